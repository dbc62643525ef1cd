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
