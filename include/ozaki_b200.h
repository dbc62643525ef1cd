/*
 * ozaki_b200.h -- C ABI of the B200 (sm_100a) Ozaki-scheme GEMM library
 * (liboz_b200.so).
 *
 * The library replaces the two device kernels of the reference
 * implementation WhFanatic/Ozaki_triton (ozaki_triton.py) and the wrappers
 * that launch them.  Every entry point takes plain device pointers, sizes,
 * strides and a CUDA stream.  No entry point allocates or frees device
 * memory, and only oz_device_status synchronises (the stream it is given);
 * the others only enqueue work on their stream.  State the library keeps:
 * the last-error string (thread-local), the device-side timeout word of each
 * kernel file (oz_device_status), a launch counter, and one static 32 MiB
 * device array per GPU that only oz_split_noalloc uses.  Calls are
 * re-entrant except that oz_split_noalloc calls overlapping on one GPU share
 * that array.
 *
 * Status codes: 0 = OZ_OK; negative values are errors and oz_last_error()
 * returns a message for the calling thread.  Argument errors are reported
 * before any launch.
 */
#ifndef OZAKI_B200_H
#define OZAKI_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types (matrix inputs, slices and outputs) */
enum oz_dtype {
  OZ_F64 = 0,
  OZ_F32 = 1,
  OZ_F16 = 2,
  OZ_BF16 = 3,
  OZ_I8 = 4
};

/* status codes */
enum oz_status {
  OZ_OK = 0,
  OZ_ERR_INVALID = -1,     /* bad argument (shape, stride, alignment, range) */
  OZ_ERR_UNSUPPORTED = -2, /* valid but unsupported combination */
  OZ_ERR_CUDA = -3,        /* a CUDA runtime/driver call failed */
  OZ_ERR_TIMEOUT = -4      /* a device-side wait hit its bound (see oz_device_status) */
};

/* residual handling between split levels */
enum oz_residual_mode {
  OZ_RESIDUAL_COMPAT = 0, /* round the residual to fp32 after every level, as the
                             reference's fp32 residual buffer does (bit-exact) */
  OZ_RESIDUAL_EXACT = 1   /* keep the residual in the input precision (fp64) */
};

/* flags for oz_cross_gemm */
#define OZ_GEMM_SKIP_TAIL 1u   /* drop slice pairs with i + j >= num_splits */

/*
 * Split alpha rule.  Replaces compute_split_bits (ozaki_triton.py:76-98):
 * alpha = int((acc_bits - log2 n) / 2) with acc_bits 31 (int8 slices, int32
 * accumulator) or 23 (float slices, fp32 accumulator), capped by the slice
 * mantissa bits (fp32 23, fp16 10, bf16 7, int8 7).  Returns OZ_ERR_INVALID
 * for n <= 0 or alpha < 1.
 */
int oz_compute_split_bits(int64_t n, int slice_dtype, int32_t *alpha_out);

/*
 * Bytes per slice row as the library lays slices out: k elements padded to a
 * multiple of 128 bytes (the padding is written as zeros by oz_split).
 */
int64_t oz_slice_row_bytes(int64_t k, int slice_dtype);

/*
 * Split a batch of matrices into num_splits slices along K.
 * Replaces split_matrix (ozaki_triton.py:214-256) and split_matrix_kernel
 * (ozaki_triton.py:136-211).
 *
 *   in        : element (b, line, k) at in + b*stride_b + line*stride_line + k*stride_k
 *               (element strides).  Lines are the rows of A, or the columns of B
 *               (B is split through its transposed view, ozaki_triton.py:593).
 *               Any strides.  Fast kernels: stride_k == 1 (rows); stride_line ==
 *               1 (columns) through a column kernel where one applies (fp64:
 *               pairs of columns from 2-D TMA boxes, K <= 8192, 16-byte row
 *               pitch; fp32/fp16/bf16: a cluster kernel); other layouts and
 *               int8 inputs take a generic kernel.
 *   slices    : (batch, num_splits, lines, ld) of slice_dtype, ld = row pitch in
 *               elements (oz_slice_row_bytes(k)/elem_size); k-contiguous.
 *   scales    : (batch, num_splits, lines) fp32 powers of two.
 *   residual_mode : OZ_RESIDUAL_COMPAT reproduces the reference bit for bit.
 */
int oz_split(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
             int64_t stride_b, int64_t stride_line, int64_t stride_k,
             int32_t num_splits, int32_t alpha, int slice_dtype, int residual_mode,
             void *slices, int64_t ld, float *scales, void *stream);

/*
 * Scratch bytes that oz_split_ex can use for this input layout (0 when none
 * helps).  When the lines are contiguous (stride_line == 1: the columns of a
 * row-major B) and no column kernel applies, oz_split_ex transposes them into
 * the workspace ((batch, lines, k padded to 16 bytes), input dtype) so that
 * each line is read as one contiguous row by the row kernel.
 */
int64_t oz_split_workspace_bytes(int in_dtype, int64_t batch, int64_t lines, int64_t k,
                                 int64_t stride_line, int64_t stride_k);

/*
 * oz_split with caller-provided scratch memory (device, 16-byte aligned).
 * Same results as oz_split; with workspace_bytes >= oz_split_workspace_bytes()
 * a column layout that no column kernel takes goes through the transpose
 * described above, otherwise it behaves exactly like oz_split.  Also replaces split_matrix
 * (ozaki_triton.py:214-256), whose fp32 residual buffer is a workspace too.
 */
int oz_split_ex(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
                int64_t stride_b, int64_t stride_line, int64_t stride_k,
                int32_t num_splits, int32_t alpha, int slice_dtype, int residual_mode,
                void *slices, int64_t ld, float *scales, void *workspace,
                int64_t workspace_bytes, void *stream);

/*
 * oz_split without any allocation, for callers that cannot call cudaMalloc:
 * code that reaches the library through a foreign-function binding holding
 * only the raw device pointers it was handed (no device allocator of its
 * own), and latency-critical loops in which cudaMalloc's implicit
 * device-wide synchronisation is not acceptable.  (No counterpart in the
 * reference, which allocates its residual buffer on every call.)
 *
 * Identical results to oz_split_ex.  The scratch that oz_split_ex takes from
 * the caller (column layouts only, size oz_split_workspace_bytes()) comes
 * from a fixed array of oz_split_noalloc_max_bytes() bytes (32 MiB) that the
 * library keeps in device memory of every GPU it is loaded on, until the
 * process exits.  Inputs needing more scratch are rejected with
 * OZ_ERR_INVALID before any launch, unless a column kernel takes them
 * without scratch (fp64 column pairs, or the cluster kernel).  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  All calls share the one array: calls that overlap on
 * the GPU (different streams, or different host threads on one device) race
 * and corrupt each other's slices; serialise them.  Nothing in the array has
 * to start at zero: every byte a call reads was written earlier in that call.
 */
int oz_split_noalloc(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
                     int64_t stride_b, int64_t stride_line, int64_t stride_k,
                     int32_t num_splits, int32_t alpha, int slice_dtype, int residual_mode,
                     void *slices, int64_t ld, float *scales, void *stream);

/* Size in bytes of oz_split_noalloc's fixed device scratch array. */
int64_t oz_split_noalloc_max_bytes(void);

/*
 * Fused cross-GEMM over all slice pairs.
 * Replaces cross_gemm (ozaki_triton.py:455-498) and cross_gemm_kernel
 * (ozaki_triton.py:305-452):
 *   C[b] = out( sum_i sum_j od( f32( f32(A_i B_j^T) * sa_i ) * sb_j ) )
 * summed i-major, j-minor; od = fp64 for an fp64 output, else fp32.
 *
 *   a_slices : (a_batches, s, m, ld) K-contiguous, ld as returned by oz_slice_row_bytes.
 *   b_slices : (b_batches, s, n, ld) K-contiguous (B's slices stored transposed,
 *              like B_slices_T at ozaki_triton.py:594).
 *   a_scales : (a_batches, s, m) fp32; b_scales : (b_batches, s, n) fp32.
 *   a_index / b_index : per output batch b, which A / B batch it uses (int32
 *              device arrays of length batch; NULL means identity).  This is how
 *              torch.matmul broadcasting is expressed without copying operands.
 *   c        : (batch, m, n) of out_dtype, row pitch ldc elements.
 *   flags    : OZ_GEMM_SKIP_TAIL or 0.
 */
int oz_cross_gemm(const void *a_slices, const void *b_slices, const float *a_scales,
                  const float *b_scales, int64_t batch, int64_t m, int64_t n, int64_t k,
                  int64_t ld, int32_t num_splits, int slice_dtype, int out_dtype,
                  const int32_t *a_index, const int32_t *b_index, int64_t a_batches,
                  int64_t b_batches, void *c, int64_t ldc, uint32_t flags, void *stream);

/*
 * The whole product in one call.  Replaces ozaki_matmul
 * (ozaki_triton.py:534-606) below its Python-level checks: B is split by
 * columns (its transposed view, ozaki_triton.py:593) and A by rows into the
 * workspace, then the fused cross-GEMM writes C in the input dtype
 * (ozaki_triton.py:575, 606).  alpha comes from oz_compute_split_bits(k).
 *
 *   a : element (b, i, kk) at a + b*a_sb + i*a_sm + kk*a_sk (element strides),
 *       a_batches matrices (m, k); b : element (b, kk, j) at
 *       b + b*b_sb + kk*b_sk + j*b_sn, b_batches matrices (k, n).  Any strides.
 *   batch, a_index, b_index : output batches and the operand members each uses
 *       (NULL = identity), as in oz_cross_gemm: torch.matmul broadcasting
 *       without copies of the operands.
 *   c : (batch, m, n) of in_dtype, row pitch ldc.
 *   workspace : oz_matmul_workspace_bytes() bytes of device memory, 256-byte
 *       aligned (slices, scales and the column-transpose scratch).
 * Small operand pairs (A and B together at most 4 Mi elements, k * 8 bytes
 * at most 48 KB) are split in a single launch, so the call is two kernels;
 * larger ones take the streaming split kernels (three or more).  Results are
 * bit-identical either way.
 */
int64_t oz_matmul_workspace_bytes(int in_dtype, int64_t a_batches, int64_t b_batches, int64_t m,
                                  int64_t n, int64_t k, int64_t a_sm, int64_t a_sk, int64_t b_sk,
                                  int64_t b_sn, int32_t num_splits, int slice_dtype);

int oz_matmul(const void *a, const void *b, int in_dtype, int64_t batch, int64_t a_batches,
              int64_t b_batches, const int32_t *a_index, const int32_t *b_index, int64_t m,
              int64_t n, int64_t k, int64_t a_sb, int64_t a_sm, int64_t a_sk, int64_t b_sb,
              int64_t b_sk, int64_t b_sn, int32_t num_splits, int slice_dtype, int residual_mode,
              void *c, int64_t ldc, uint32_t flags, void *workspace, int64_t workspace_bytes,
              void *stream);

/*
 * oz_cross_gemm with B's slices stored in column blocks (no counterpart in the
 * reference, which has no multi-GPU path; this is the layout an all-gather or
 * a blockwise broadcast of B's slices produces without a re-layout copy).
 *
 *   b_slices : (b_batches, blocks, num_splits, b_block_cols, ld), blocks =
 *              ceil(n / b_block_cols); column c of B lives in block
 *              c / b_block_cols at row c % b_block_cols (rows of the last
 *              block past n are never read into stored outputs).
 *   b_scales : (b_batches, blocks, num_splits, b_block_cols).
 *   b_block_cols : a multiple of 128, or >= n (one block whose rows past n
 *              are padding), or 0 for the plain layout of oz_cross_gemm.
 * All other arguments as oz_cross_gemm; results are bit-identical to it.
 */
int oz_cross_gemm_blocked(const void *a_slices, const void *b_slices, const float *a_scales,
                          const float *b_scales, int64_t batch, int64_t m, int64_t n, int64_t k,
                          int64_t ld, int32_t num_splits, int slice_dtype, int out_dtype,
                          const int32_t *a_index, const int32_t *b_index, int64_t a_batches,
                          int64_t b_batches, int64_t b_block_cols, void *c, int64_t ldc,
                          uint32_t flags, void *stream);

/*
 * oz_cross_gemm_blocked (one batch) in a single persistent launch while B's
 * column blocks are still arriving (no counterpart in the reference, which
 * has no multi-GPU path; it lets a rank multiply the blocks it pulls from its
 * peers without one launch per block).
 *
 *   ready       : device int32[blocks]; block c is read (its slices and
 *                 scales) once ready[c] == ready_value.  Write the flag with
 *                 a copy ordered after the block's own copies on the same
 *                 stream (e.g. a 4-byte copy from pinned host memory): the
 *                 kernel holds every SM while it waits, so the flag must
 *                 come from work that needs none, like a copy engine.
 *   first_block, block_count : the launch computes the output columns of
 *                 block_count blocks (0: all), first_block, first_block + 1,
 *                 .. (mod blocks), in that order; other columns of C are
 *                 left as they are.
 * The waits are bounded (about 2 s of SM clock): a block that never arrives
 * ends the launch early and oz_device_status then reports OZ_ERR_TIMEOUT
 * (code 5).  All other arguments and the results as oz_cross_gemm_blocked.
 */
int oz_cross_gemm_arrivals(const void *a_slices, const void *b_slices, const float *a_scales,
                           const float *b_scales, int64_t m, int64_t n, int64_t k, int64_t ld,
                           int32_t num_splits, int slice_dtype, int out_dtype,
                           int64_t b_block_cols, const int32_t *ready, int32_t ready_value,
                           int32_t first_block, int32_t block_count, void *c, int64_t ldc,
                           uint32_t flags, void *stream);

/*
 * Peer mappings for the multi-GPU gather (no counterpart in the reference,
 * which has no multi-GPU path).  One process per GPU: a rank exports the
 * allocation holding its slice buffer, each peer imports it once and pulls
 * blocks with oz_copy_async (copy engines over NVLink, no SMs used).
 */
#define OZ_IPC_HANDLE_BYTES 64

/* CUDA IPC handle (OZ_IPC_HANDLE_BYTES) of the allocation holding ptr, and
 * ptr's byte offset inside it. */
int oz_ipc_export(const void *ptr, void *handle, int64_t *offset);

/* Map a peer's exported allocation into this process: *ptr = base + offset. */
int oz_ipc_import(const void *handle, int64_t offset, void **ptr);

/* Unmap what oz_ipc_import returned (same ptr and offset). */
int oz_ipc_close(void *ptr, int64_t offset);

/* Stream-ordered copy (kind inferred from the addresses): device memory,
 * a peer mapping or pinned host memory on either side. */
int oz_copy_async(void *dst, const void *src, int64_t bytes, void *stream);

/*
 * Device-side status: the kernels bound every spin-wait; when a bound is hit
 * they record a code in a device flag and return early (their output is then
 * undefined).  This call synchronises `stream`, returns OZ_OK or
 * OZ_ERR_TIMEOUT, writes the recorded code (0 = none) to *code, and clears it.
 */
int oz_device_status(void *stream, int32_t *code);

/*
 * Kernel timing from the caller's side (no counterpart in the reference):
 * the next cross-GEMM launch made by this thread (through oz_cross_gemm,
 * oz_cross_gemm_blocked or oz_matmul) records begin_event just before it and
 * end_event just after it, on the launch's stream; then the pair is
 * forgotten.  Either may be NULL.  The events are the caller's cudaEvent_t.
 */
int oz_profile_next_gemm(void *begin_event, void *end_event);

/* Kernels the library has launched in this process, a running total (no
 * counterpart in the reference; lets a caller count the device work of a
 * region: the difference of two readings). */
int64_t oz_launch_count(void);

/*
 * Self-test of the device-side failure detection (no counterpart in the
 * reference): one thread waits on a barrier that nothing arrives on, with
 * the kernels' bounded wait cut to bound_cycles SM cycles (at most the
 * kernels' own bound, ~2 s).  The wait gives up, the kernel returns normally
 * and the next oz_device_status reports OZ_ERR_TIMEOUT with code 9.  No
 * fault, no trap; the context stays usable.
 */
int oz_wait_selftest(int64_t bound_cycles, void *stream);

/* Message for the last error returned on the calling thread ("" if none). */
const char *oz_last_error(void);

/* Library version string. */
const char *oz_version(void);

#ifdef __cplusplus
}
#endif

#endif /* OZAKI_B200_H */
