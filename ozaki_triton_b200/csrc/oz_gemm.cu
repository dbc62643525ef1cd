// oz_gemm.cu -- fused Ozaki cross-GEMM on the 5th-generation tensor cores
// (tcgen05, sm_100a).
//
// Replaces cross_gemm_kernel (ozaki_triton.py:305-452) and its wrapper
// cross_gemm (ozaki_triton.py:455-498):
//   C[b,m,n] = out( sum_i sum_j od( f32( f32(acc_ij[m,n]) * sa_i[m] ) * sb_j[n] ) )
//   acc_ij   = sum_k A_i[m,k] * B_j[n,k]   (int32 for int8 slices, fp32 otherwise)
// summed i-major, j-minor into od = fp64 (fp64 output) or fp32, exactly the
// epilogue order of ozaki_triton.py:426-447, so int8 results are bit-identical
// to the reference.
//
// Structure (one persistent CTA per SM, 10 warps):
//   warp 0     TMA producer: 128x128-byte K-major tiles (128-byte swizzle) of
//              A_i and B_j into two shared-memory rings (A ring, B ring).
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer.
//   warps 2-9  epilogue: tcgen05.ld of the int32/fp32 accumulators, scaling,
//              fp64/fp32 outer accumulation in registers, store of C.
// Per output tile (128 rows x NT columns) the kernel runs one "pass" per A
// slice i: a full K loop that accumulates the pair products A_i B_j for every
// j into s TMEM accumulators of NT columns each (s * NT <= 512 columns).  A_i
// is loaded once per pass and reused by all j; when 2 * s * NT <= 512 the
// accumulators are double-buffered so the epilogue of pass i overlaps the MMAs
// of pass i + 1.  The fp64/fp32 outer accumulator never leaves registers.
//
// Every spin-wait is bounded (oz_common.cuh); on a timeout the kernel records
// a code in g_device_status, drains its own asynchronous work (bounded), frees
// TMEM and returns.

#include <cstdio>
#include <cudaTypedefs.h>

#include "oz_common.cuh"

namespace oz {

constexpr int kBM = 128;          // rows per tile (UMMA M)
constexpr int kKBytes = 128;      // K bytes per pipeline stage (one swizzle row)
constexpr int kGemmThreads = 320; // 10 warps
constexpr int kEpiWarps = 8;
constexpr int kStagesA = 4;

struct GemmParams {
  const float *a_scales;
  const float *b_scales;
  const int32_t *a_index;
  const int32_t *b_index;
  void *c;
  int64_t ldc;
  int m, n, kblocks;     // kblocks = ld_bytes / 128
  int s;
  int skip_tail;
  int batch;
  int tiles_m, tiles_n, num_tiles;
  uint32_t idesc;
};

template <int NT> struct GemmCfg {
  static constexpr int kBBytes = NT * kKBytes;              // one B tile
  static constexpr int kABytes = kBM * kKBytes;             // one A tile (16 KB)
  static constexpr int kStagesB = (NT == 128) ? 8 : 12;
  static constexpr int kSmemTiles = kStagesA * kABytes + kStagesB * kBBytes;
  static constexpr int kSmemBytes = kSmemTiles + 1024 /*align*/ + 1024 /*barriers*/;
};

template <int OUTK> struct OutT;
template <> struct OutT<OZ_F64> { using acc = double; using store = double; };
template <> struct OutT<OZ_F32> { using acc = float; using store = float; };
template <> struct OutT<OZ_F16> { using acc = float; using store = __half; };
template <> struct OutT<OZ_BF16> { using acc = float; using store = __nv_bfloat16; };

template <typename ACC> __device__ __forceinline__ ACC acc_add(ACC a, float v);
template <> __device__ __forceinline__ double acc_add<double>(double a, float v) {
  return __dadd_rn(a, (double)v);
}
template <> __device__ __forceinline__ float acc_add<float>(float a, float v) {
  return __fadd_rn(a, v);
}

template <int OUTK> __device__ __forceinline__ typename OutT<OUTK>::store
to_out(typename OutT<OUTK>::acc v) {
  if constexpr (OUTK == OZ_F16) return __float2half_rn(v);
  else if constexpr (OUTK == OZ_BF16) return __float2bfloat16_rn(v);
  else return v;
}

__device__ __forceinline__ void tile_coords(const GemmParams &p, int t, int &b, int &mb, int &nb) {
  const int tpb = p.tiles_m * p.tiles_n;
  b = t / tpb;
  int local = t - b * tpb;
  // grouped raster: GM row-tiles sweep all column tiles before moving on,
  // so the A rows and B columns of concurrently running tiles stay in L2
  constexpr int GM = 16;
  int per_group = GM * p.tiles_n;
  int group = local / per_group;
  int first_m = group * GM;
  int gsz = min(p.tiles_m - first_m, GM);
  int in_group = local - group * per_group;
  mb = first_m + in_group % gsz;
  nb = in_group / gsz;
}

template <int KIND, int OUTK, int NT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    cross_gemm_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b, const GemmParams p) {
  using Cfg = GemmCfg<NT>;
  using ACC = typename OutT<OUTK>::acc;
  using STO = typename OutT<OUTK>::store;
  constexpr int SB = Cfg::kStagesB;

  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  unsigned char *ring_a = smem;
  unsigned char *ring_b = smem + kStagesA * Cfg::kABytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::kSmemTiles);
  uint64_t *full_a = bars;
  uint64_t *empty_a = full_a + kStagesA;
  uint64_t *full_b = empty_a + kStagesA;
  uint64_t *empty_b = full_b + SB;
  uint64_t *acc_full = empty_b + SB;      // [2]
  uint64_t *acc_empty = acc_full + 2;     // [2]
  uint64_t *drain = acc_empty + 2;        // [1]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int s = p.s;
  const int nbuf = (2 * s * NT <= 512) ? 2 : 1;
  int tcols = 32;
  while (tcols < nbuf * s * NT) tcols <<= 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStagesA; ++i) { mbar_init(&full_a[i], 1); mbar_init(&empty_a[i], 1); }
    for (int i = 0; i < SB; ++i) { mbar_init(&full_b[i], 1); mbar_init(&empty_b[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps * 32);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, (uint32_t)tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t ia = 0, ib = 0;   // running load counters (slot = counter % stages)
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int b, mb, nb;
        tile_coords(p, t, b, mb, nb);
        const int ai = p.a_index ? p.a_index[b] : b;
        const int bi = p.b_index ? p.b_index[b] : b;
        for (int i = 0; ok && i < s; ++i) {
          const int js = p.skip_tail ? s - i : s;
          for (int kb = 0; ok && kb < p.kblocks; ++kb) {
            {
              const int slot = ia % kStagesA;
              const uint32_t par = ((ia / kStagesA) & 1) ^ 1;
              if (!(ok = mbar_wait_bounded(&empty_a[slot], par, abort_flag, DEV_TIMEOUT_PRODUCER)))
                break;
              mbar_arrive_expect_tx(&full_a[slot], Cfg::kABytes);
              tma_load_3d(ring_a + slot * Cfg::kABytes, &tm_a, &full_a[slot], kb * kKBytes,
                          mb * kBM, ai * s + i);
              ++ia;
            }
            for (int j = 0; j < js; ++j) {
              const int slot = ib % SB;
              const uint32_t par = ((ib / SB) & 1) ^ 1;
              if (!(ok = mbar_wait_bounded(&empty_b[slot], par, abort_flag, DEV_TIMEOUT_PRODUCER)))
                break;
              mbar_arrive_expect_tx(&full_b[slot], Cfg::kBBytes);
              tma_load_3d(ring_b + slot * Cfg::kBBytes, &tm_b, &full_b[slot], kb * kKBytes,
                          nb * NT, bi * s + j);
              ++ib;
            }
          }
        }
      }
      // drain: every issued load must have landed before shared memory is released
      for (uint32_t k = (ia > kStagesA ? ia - kStagesA : 0); k < ia; ++k)
        mbar_wait_bounded(&full_a[k % kStagesA], (k / kStagesA) & 1, abort_flag,
                          DEV_TIMEOUT_PRODUCER);
      for (uint32_t k = (ib > (uint32_t)SB ? ib - SB : 0); k < ib; ++k)
        mbar_wait_bounded(&full_b[k % SB], (k / SB) & 1, abort_flag, DEV_TIMEOUT_PRODUCER);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t ia = 0, ib = 0, pass = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(ring_a), b_base = smem_u32(ring_b);
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        for (int i = 0; ok && i < s; ++i, ++pass) {
          const int js = p.skip_tail ? s - i : s;
          const int buf = pass % nbuf;
          const uint32_t use = pass / nbuf;
          if (!(ok = mbar_wait_bounded(&acc_empty[buf], (use & 1) ^ 1, abort_flag,
                                       DEV_TIMEOUT_MMA)))
            break;
          tc_fence_after();
          const uint32_t d0 = tmem_base + (uint32_t)(buf * s * NT);
          for (int kb = 0; ok && kb < p.kblocks; ++kb) {
            const int sa_slot = ia % kStagesA;
            if (!(ok = mbar_wait_bounded(&full_a[sa_slot], (ia / kStagesA) & 1, abort_flag,
                                         DEV_TIMEOUT_MMA)))
              break;
            tc_fence_after();
            const uint64_t adesc = smem_desc_sw128(a_base + sa_slot * Cfg::kABytes);
            for (int j = 0; j < js; ++j) {
              const int sb_slot = ib % SB;
              if (!(ok = mbar_wait_bounded(&full_b[sb_slot], (ib / SB) & 1, abort_flag,
                                           DEV_TIMEOUT_MMA)))
                break;
              tc_fence_after();
              const uint64_t bdesc = smem_desc_sw128(b_base + sb_slot * Cfg::kBBytes);
#pragma unroll
              for (int kk = 0; kk < kKBytes / 32; ++kk) {
                // advance 32 bytes along K inside the 128-byte swizzle row
                tc_mma<KIND>(d0 + (uint32_t)(j * NT), adesc + (uint64_t)(kk * 2),
                             bdesc + (uint64_t)(kk * 2), p.idesc, (kb | kk) != 0);
              }
              tc_commit(&empty_b[sb_slot]);
              ++ib;
            }
            if (!ok) break;
            tc_commit(&empty_a[sa_slot]);
            ++ia;
          }
          if (!ok) break;
          tc_commit(&acc_full[buf]);
        }
      }
      // wait for all issued MMAs before TMEM / shared memory go away
      tc_commit(drain);
      mbar_wait_bounded(drain, 0, abort_flag, DEV_TIMEOUT_MMA);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int sub = warp & 3;                 // TMEM lane quarter this warp may access
    const int half = e >> 2;                  // which half of the NT columns
    constexpr int NH = NT / 2;
    const int row = sub * 32 + lane;
    const uint32_t lane_addr = tmem_base + ((uint32_t)(sub * 32) << 16);
    ACC out[NH];
#pragma unroll
    for (int x = 0; x < NH; ++x) out[x] = (ACC)0;
    uint32_t pass = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
      int b, mb, nb;
      tile_coords(p, t, b, mb, nb);
      const int ai = p.a_index ? p.a_index[b] : b;
      const int bi = p.b_index ? p.b_index[b] : b;
      const int m = mb * kBM + row;
      const int n0 = nb * NT + half * NH;
      for (int i = 0; i < s; ++i, ++pass) {
        const int js = p.skip_tail ? s - i : s;
        const int buf = pass % nbuf;
        const uint32_t use = pass / nbuf;
        // every lane waits, then the warp agrees (tcgen05.ld needs a converged warp)
        ok = mbar_wait_bounded(&acc_full[buf], use & 1, abort_flag, DEV_TIMEOUT_EPILOGUE);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const float sa = (m < p.m) ? p.a_scales[((int64_t)ai * s + i) * p.m + m] : 0.f;
        for (int j = 0; j < js; ++j) {
          const float *sbp = p.b_scales + ((int64_t)bi * s + j) * p.n;
#pragma unroll
          for (int c = 0; c < NH / 16; ++c) {
            uint32_t r[16];
            tmem_ld16(lane_addr + (uint32_t)((buf * s + j) * NT + half * NH + c * 16), r);
            tmem_ld_wait();
#pragma unroll
            for (int x = 0; x < 16; ++x) {
              const int col = n0 + c * 16 + x;
              const float sb = (col < p.n) ? __ldg(sbp + col) : 0.f;
              float v;
              if constexpr (KIND == 0) v = __int2float_rn((int)r[x]);
              else v = __uint_as_float(r[x]);
              v = __fmul_rn(__fmul_rn(v, sa), sb);
              out[c * 16 + x] = acc_add<ACC>(out[c * 16 + x], v);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      // store the finished tile
      if (m < p.m) {
        STO *crow = reinterpret_cast<STO *>(p.c) + ((int64_t)b * p.m + m) * p.ldc;
#pragma unroll
        for (int x = 0; x < NH; ++x) {
          const int col = n0 + x;
          if (col < p.n) crow[col] = to_out<OUTK>(out[x]);
        }
      }
#pragma unroll
      for (int x = 0; x < NH; ++x) out[x] = (ACC)0;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, (uint32_t)tcols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

int make_map(CUtensorMap *map, const void *base, uint64_t row_bytes, uint64_t rows,
             uint64_t mats, uint32_t box_rows) {
  auto enc = get_encode();
  if (!enc) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {row_bytes, rows, mats};
  cuuint64_t strides[2] = {row_bytes, row_bytes * rows};
  cuuint32_t box[3] = {(cuuint32_t)kKBytes, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return OZ_OK;
}

uint32_t make_idesc(int slice_dtype, int nt) {
  uint32_t c_fmt, ab_fmt;
  switch (slice_dtype) {
    case OZ_I8: c_fmt = 2; ab_fmt = 1; break;    // S32 accumulate, signed 8-bit
    case OZ_F16: c_fmt = 1; ab_fmt = 0; break;   // F32 accumulate, F16
    case OZ_BF16: c_fmt = 1; ab_fmt = 1; break;  // F32 accumulate, BF16
    default: c_fmt = 1; ab_fmt = 2; break;       // F32 accumulate, TF32
  }
  uint32_t d = 0;
  d |= c_fmt << 4;
  d |= ab_fmt << 7;
  d |= ab_fmt << 10;
  // bits 15/16 = 0: both operands K-major
  d |= (uint32_t)(nt >> 3) << 17;
  d |= (uint32_t)(kBM >> 4) << 24;
  return d;
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int KIND, int OUTK, int NT>
int launch_gemm(const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p,
                cudaStream_t st) {
  using Cfg = GemmCfg<NT>;
  auto kern = cross_gemm_kernel<KIND, OUTK, NT>;
  if (int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               Cfg::kSmemBytes),
                          "cudaFuncSetAttribute(cross_gemm)"))
    return rc;
  int grid = min(p.num_tiles, sm_count());
  kern<<<grid, kGemmThreads, Cfg::kSmemBytes, st>>>(ta, tb, p);
  return check_cuda(cudaGetLastError(), "cross_gemm_kernel launch");
}

template <int KIND, int NT>
int launch_out(int out_dtype, const CUtensorMap &ta, const CUtensorMap &tb, const GemmParams &p,
               cudaStream_t st) {
  switch (out_dtype) {
    case OZ_F64: return launch_gemm<KIND, OZ_F64, NT>(ta, tb, p, st);
    case OZ_F32: return launch_gemm<KIND, OZ_F32, NT>(ta, tb, p, st);
    case OZ_F16: return launch_gemm<KIND, OZ_F16, NT>(ta, tb, p, st);
    case OZ_BF16: return launch_gemm<KIND, OZ_BF16, NT>(ta, tb, p, st);
  }
  return set_error(OZ_ERR_UNSUPPORTED, "unsupported output dtype %d", out_dtype);
}

}  // namespace
int status_gemm(int *value, bool clear) { return read_status_word(value, clear); }

}  // namespace oz

extern "C" int oz_cross_gemm(const void *a_slices, const void *b_slices, const float *a_scales,
                             const float *b_scales, int64_t batch, int64_t m, int64_t n,
                             int64_t k, int64_t ld, int32_t num_splits, int slice_dtype,
                             int out_dtype, const int32_t *a_index, const int32_t *b_index,
                             int64_t a_batches, int64_t b_batches, void *c, int64_t ldc,
                             uint32_t flags, void *stream) {
  using namespace oz;
  if (num_splits < 1 || num_splits > 8)
    return set_error(OZ_ERR_INVALID, "num_splits must be in [1, 8], got %d", num_splits);
  if (batch < 0 || m < 0 || n < 0 || k < 0)
    return set_error(OZ_ERR_INVALID, "negative size");
  if (slice_dtype != OZ_I8 && slice_dtype != OZ_F16 && slice_dtype != OZ_BF16 &&
      slice_dtype != OZ_F32)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
  if (out_dtype != OZ_F64 && out_dtype != OZ_F32 && out_dtype != OZ_F16 && out_dtype != OZ_BF16)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported output dtype %d", out_dtype);
  if (flags & ~OZ_GEMM_SKIP_TAIL) return set_error(OZ_ERR_INVALID, "unknown flags 0x%x", flags);
  if (batch == 0 || m == 0 || n == 0) return OZ_OK;
  if (!c || ldc < n) return set_error(OZ_ERR_INVALID, "bad output (ldc=%lld n=%lld)",
                                      (long long)ldc, (long long)n);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int es = dtype_size(slice_dtype);
  const int64_t ld_bytes = ld * es;
  if (k == 0) {
    // empty contraction: C = 0
    if (ldc == n)
      return check_cuda(cudaMemsetAsync(c, 0, (size_t)(batch * m * n * dtype_size(out_dtype)), st),
                        "cudaMemsetAsync");
    return set_error(OZ_ERR_UNSUPPORTED, "k == 0 with a padded output");
  }
  if (!a_slices || !b_slices || !a_scales || !b_scales)
    return set_error(OZ_ERR_INVALID, "null pointer");
  if (ld < k || ld_bytes % kKBytes != 0)
    return set_error(OZ_ERR_INVALID,
                     "slice row pitch must be >= k and a multiple of 128 bytes (ld=%lld)",
                     (long long)ld);
  if (((uintptr_t)a_slices | (uintptr_t)b_slices) % 16 != 0)
    return set_error(OZ_ERR_INVALID, "slice buffers must be 16-byte aligned");
  if (a_batches < 1 || b_batches < 1 || (!a_index && a_batches < batch) ||
      (!b_index && b_batches < batch))
    return set_error(OZ_ERR_INVALID, "bad operand batch counts");
  if (m > INT32_MAX || n > INT32_MAX || a_batches * num_splits > INT32_MAX ||
      b_batches * num_splits > INT32_MAX)
    return set_error(OZ_ERR_INVALID, "size out of range");

  const int nt = num_splits <= 4 ? 128 : 64;
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, a_slices, (uint64_t)ld_bytes, (uint64_t)m,
                        (uint64_t)(a_batches * num_splits), kBM))
    return rc;
  if (int rc = make_map(&tb, b_slices, (uint64_t)ld_bytes, (uint64_t)n,
                        (uint64_t)(b_batches * num_splits), (uint32_t)nt))
    return rc;

  GemmParams p;
  p.a_scales = a_scales;
  p.b_scales = b_scales;
  p.a_index = a_index;
  p.b_index = b_index;
  p.c = c;
  p.ldc = ldc;
  p.m = (int)m;
  p.n = (int)n;
  p.kblocks = (int)(ld_bytes / kKBytes);
  p.s = num_splits;
  p.skip_tail = (flags & OZ_GEMM_SKIP_TAIL) ? 1 : 0;
  p.batch = (int)batch;
  p.tiles_m = (int)((m + kBM - 1) / kBM);
  p.tiles_n = (int)((n + nt - 1) / nt);
  int64_t tiles = (int64_t)p.tiles_m * p.tiles_n * batch;
  if (tiles > INT32_MAX) return set_error(OZ_ERR_INVALID, "too many tiles");
  p.num_tiles = (int)tiles;
  p.idesc = make_idesc(slice_dtype, nt);

  const int kind = slice_dtype == OZ_I8 ? 0 : (slice_dtype == OZ_F32 ? 2 : 1);
  if (nt == 128) {
    if (kind == 0) return launch_out<0, 128>(out_dtype, ta, tb, p, st);
    if (kind == 1) return launch_out<1, 128>(out_dtype, ta, tb, p, st);
    return launch_out<2, 128>(out_dtype, ta, tb, p, st);
  }
  if (kind == 0) return launch_out<0, 64>(out_dtype, ta, tb, p, st);
  if (kind == 1) return launch_out<1, 64>(out_dtype, ta, tb, p, st);
  return launch_out<2, 64>(out_dtype, ta, tb, p, st);
}
