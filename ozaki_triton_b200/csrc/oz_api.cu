// oz_api.cu -- library-wide C ABI entry points: error strings, the alpha
// rule, device status and the version string.

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>

#include "oz_common.cuh"

namespace oz {

namespace {
thread_local char g_err[512] = {0};
}

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<int64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int check_cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return OZ_OK;
  return set_error(OZ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

}  // namespace oz

extern "C" const char *oz_last_error(void) { return oz::g_err; }

extern "C" const char *oz_version(void) { return "ozaki_b200 0.1 (sm_100a)"; }

// alpha = int((acc_bits - log2 n) / 2), capped by the slice mantissa bits.
// ozaki_triton.py:76-98 (acc_bits 31 for the int32 accumulator of int8
// slices, 23 for the fp32 accumulator of float slices).
extern "C" int oz_compute_split_bits(int64_t n, int slice_dtype, int32_t *alpha_out) {
  int bits, acc_bits;
  switch (slice_dtype) {
    case OZ_F32: bits = 23; acc_bits = 23; break;
    case OZ_F16: bits = 10; acc_bits = 23; break;
    case OZ_BF16: bits = 7; acc_bits = 23; break;
    case OZ_I8: bits = 7; acc_bits = 31; break;
    default: return oz::set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
  }
  if (n <= 0) return oz::set_error(OZ_ERR_INVALID, "math domain error (n=%lld)", (long long)n);
  // int() truncates toward zero, like the reference
  int alpha = (int)((acc_bits - std::log2((double)n)) / 2.0);
  if (alpha > bits) alpha = bits;
  if (alpha < 1)
    return oz::set_error(OZ_ERR_INVALID, "n=%lld too large to split safely (alpha=%d)",
                         (long long)n, alpha);
  if (alpha_out) *alpha_out = alpha;
  return OZ_OK;
}

extern "C" int oz_device_status(void *stream, int32_t *code) {
  using namespace oz;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (int rc = check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize")) return rc;
  int v1 = 0, v2 = 0;
  if (int rc = status_split(&v1, true)) return rc;
  if (int rc = status_gemm(&v2, true)) return rc;
  const int v = v1 ? v1 : v2;
  if (code) *code = v;
  if (v != 0) return set_error(OZ_ERR_TIMEOUT, "device-side wait timed out (code %d)", v);
  return OZ_OK;
}

extern "C" int64_t oz_launch_count(void) { return oz::g_launches.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
// the whole product in one call
// ---------------------------------------------------------------------------
namespace {

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// Byte offsets of the pieces of oz_matmul's workspace.  The transpose
// scratch is shared by the two splits: they run one after the other on the
// same stream.
struct MatmulLayout {
  int64_t ld, a_sl, b_sl, a_sc, b_sc, ws, ws_bytes, total;
};

MatmulLayout matmul_layout(int in_dtype, int64_t a_batches, int64_t b_batches, int64_t m,
                           int64_t n, int64_t k, int64_t a_sm, int64_t a_sk, int64_t b_sk,
                           int64_t b_sn, int32_t s, int slice_dtype) {
  MatmulLayout L{};
  const int es = oz::dtype_size(slice_dtype);
  L.ld = oz_slice_row_bytes(k, slice_dtype) / es;
  int64_t off = 0;
  L.a_sl = off;
  off += align256(a_batches * s * m * L.ld * es);
  L.b_sl = off;
  off += align256(b_batches * s * n * L.ld * es);
  L.a_sc = off;
  off += align256(a_batches * s * m * 4);
  L.b_sc = off;
  off += align256(b_batches * s * n * 4);
  const int64_t wa = oz_split_workspace_bytes(in_dtype, a_batches, m, k, a_sm, a_sk);
  const int64_t wb = oz_split_workspace_bytes(in_dtype, b_batches, n, k, b_sn, b_sk);
  L.ws = off;
  L.ws_bytes = wa > wb ? wa : wb;
  off += align256(L.ws_bytes);
  L.total = off;
  return L;
}

bool valid_dtype(int dt) {
  return dt == OZ_F64 || dt == OZ_F32 || dt == OZ_F16 || dt == OZ_BF16 || dt == OZ_I8;
}

}  // namespace

extern "C" int64_t oz_matmul_workspace_bytes(int in_dtype, int64_t a_batches, int64_t b_batches,
                                             int64_t m, int64_t n, int64_t k, int64_t a_sm,
                                             int64_t a_sk, int64_t b_sk, int64_t b_sn,
                                             int32_t num_splits, int slice_dtype) {
  if (!valid_dtype(in_dtype) || !valid_dtype(slice_dtype) || slice_dtype == OZ_F64 ||
      num_splits < 1 || num_splits > 8 || a_batches < 0 || b_batches < 0 || m < 0 || n < 0 ||
      k < 0)
    return OZ_ERR_INVALID;
  if (a_batches == 0 || b_batches == 0 || m == 0 || n == 0 || k == 0) return 0;
  return matmul_layout(in_dtype, a_batches, b_batches, m, n, k, a_sm, a_sk, b_sk, b_sn,
                       num_splits, slice_dtype)
      .total;
}

extern "C" int oz_matmul(const void *a, const void *b, int in_dtype, int64_t batch,
                         int64_t a_batches, int64_t b_batches, const int32_t *a_index,
                         const int32_t *b_index, int64_t m, int64_t n, int64_t k, int64_t a_sb,
                         int64_t a_sm, int64_t a_sk, int64_t b_sb, int64_t b_sk, int64_t b_sn,
                         int32_t num_splits, int slice_dtype, int residual_mode, void *c,
                         int64_t ldc, uint32_t flags, void *workspace, int64_t workspace_bytes,
                         void *stream) {
  using namespace oz;
  if (!valid_dtype(in_dtype)) return set_error(OZ_ERR_UNSUPPORTED, "unsupported input dtype %d", in_dtype);
  if (!valid_dtype(slice_dtype) || slice_dtype == OZ_F64)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
  if (num_splits < 1 || num_splits > 8)
    return set_error(OZ_ERR_INVALID, "num_splits must be in [1, 8], got %d", num_splits);
  if (batch < 0 || a_batches < 0 || b_batches < 0 || m < 0 || n < 0 || k < 0)
    return set_error(OZ_ERR_INVALID, "negative size");
  if (batch == 0 || m == 0 || n == 0) return OZ_OK;
  if (k == 0)   // empty contraction: C = 0
    return oz_cross_gemm(nullptr, nullptr, nullptr, nullptr, batch, m, n, 0, 0, num_splits,
                         slice_dtype, in_dtype, a_index, b_index, a_batches, b_batches, c, ldc,
                         flags, stream);
  if (!a || !b || !c) return set_error(OZ_ERR_INVALID, "null pointer");
  int32_t alpha = 0;
  if (int rc = oz_compute_split_bits(k, slice_dtype, &alpha)) return rc;
  const MatmulLayout L = matmul_layout(in_dtype, a_batches, b_batches, m, n, k, a_sm, a_sk, b_sk,
                                       b_sn, num_splits, slice_dtype);
  if (!workspace || workspace_bytes < L.total || (uintptr_t)workspace % 256 != 0)
    return set_error(OZ_ERR_INVALID,
                     "workspace of %lld bytes (256-byte aligned) needed, got %lld at %p",
                     (long long)L.total, (long long)workspace_bytes, workspace);
  unsigned char *w = static_cast<unsigned char *>(workspace);
  void *a_sl = w + L.a_sl, *b_sl = w + L.b_sl, *ws = L.ws_bytes ? w + L.ws : nullptr;
  float *a_sc = reinterpret_cast<float *>(w + L.a_sc);
  float *b_sc = reinterpret_cast<float *>(w + L.b_sc);
  bool done = false;
  if (int rc = split_two_small_impl(in_dtype, a, a_batches, m, a_sb, a_sm, a_sk, b, b_batches, n,
                                    b_sb, b_sn, b_sk, k, num_splits, alpha, slice_dtype,
                                    residual_mode, a_sl, a_sc, b_sl, b_sc, L.ld, stream, &done))
    return rc;
  if (!done) {
    // B is split by columns (its transposed view, ozaki_triton.py:593), then A by rows
    if (int rc = oz_split_ex(b, in_dtype, b_batches, n, k, b_sb, b_sn, b_sk, num_splits, alpha,
                             slice_dtype, residual_mode, b_sl, L.ld, b_sc, ws, L.ws_bytes,
                             stream))
      return rc;
    if (int rc = oz_split_ex(a, in_dtype, a_batches, m, k, a_sb, a_sm, a_sk, num_splits, alpha,
                             slice_dtype, residual_mode, a_sl, L.ld, a_sc, ws, L.ws_bytes,
                             stream))
      return rc;
  }
  return oz_cross_gemm(a_sl, b_sl, a_sc, b_sc, batch, m, n, k, L.ld, num_splits, slice_dtype,
                       in_dtype, a_index, b_index, a_batches, b_batches, c, ldc, flags, stream);
}
