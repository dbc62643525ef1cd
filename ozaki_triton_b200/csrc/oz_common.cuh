// oz_common.cuh -- shared device helpers for the sm_100a Ozaki kernels:
// dtype traits, exact power-of-two scale arithmetic, bounded mbarrier waits,
// TMA and tcgen05 (5th-generation tensor core / tensor memory) PTX wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <unordered_map>

#include "../../include/ozaki_b200.h"

namespace oz {

// ---------------------------------------------------------------------------
// error state (host)
// ---------------------------------------------------------------------------
int set_error(int code, const char *fmt, ...);
int check_cuda(cudaError_t e, const char *what);
// Kernel launches issued by the library (oz_launch_count), counted at each
// launch site.
void count_launch();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for a kernel, issued only
// when this device has not yet allowed the kernel that much shared memory
// (the attribute is an upper bound, so a larger earlier value covers smaller
// launches).  Saves a driver call per launch on small, launch-bound products.
inline int set_smem_once(const void *kern, int smem, const char *what) {
  constexpr int kDevs = 64;
  static std::mutex mu;
  static std::unordered_map<const void *, int> allowed[kDevs];
  int dev = -1;
  const bool cached = cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kDevs;
  if (cached) {
    std::lock_guard<std::mutex> lk(mu);
    const auto it = allowed[dev].find(kern);
    if (it != allowed[dev].end() && it->second >= smem) return 0;
  }
  const int rc =
      check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), what);
  if (rc == 0 && cached) {
    std::lock_guard<std::mutex> lk(mu);
    int &v = allowed[dev][kern];
    if (v < smem) v = smem;
  }
  return rc;
}

// Device-side status word of this translation unit: kernels write a nonzero
// code here when a bounded wait gives up.  Each .cu file exposes it through a
// host accessor (status_split / status_gemm) that oz_device_status() reads and
// clears.
static __device__ int g_device_status = 0;

int status_split(int *value, bool clear);
int status_gemm(int *value, bool clear);

// Split of both operands of a product in one launch (oz_split.cu): A's rows
// (a_sm, a_sk: line and k strides) and B's columns (b_sn, b_sk), each into
// its own slices (batch, s, lines, ld) and scales.  Sets *done only when the
// operands are small enough for it; otherwise nothing is launched.
int split_two_small_impl(int in_dtype, const void *a, int64_t a_batches, int64_t m, int64_t a_sb,
                         int64_t a_sm, int64_t a_sk, const void *b, int64_t b_batches, int64_t n,
                         int64_t b_sb, int64_t b_sn, int64_t b_sk, int64_t k, int32_t s,
                         int32_t alpha, int slice_dtype, int residual_mode, void *a_slices,
                         float *a_scales, void *b_slices, float *b_scales, int64_t ld,
                         void *stream, bool *done);

// Read (and optionally clear) this translation unit's status word.
static inline int read_status_word(int *value, bool clear) {
  int v = 0;
  if (int rc = check_cuda(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)),
                          "read device status"))
    return rc;
  if (clear && v != 0) {
    const int zero = 0;
    if (int rc = check_cuda(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)),
                            "clear device status"))
      return rc;
  }
  *value = v;
  return OZ_OK;
}

enum DeviceCode : int {
  DEV_OK = 0,
  DEV_TIMEOUT_PRODUCER = 1,
  DEV_TIMEOUT_MMA = 2,
  DEV_TIMEOUT_EPILOGUE = 3,
  DEV_TIMEOUT_CLUSTER = 4,
  DEV_TIMEOUT_ARRIVAL = 5,    // oz_cross_gemm_arrivals: a column block never arrived
  DEV_TIMEOUT_SELFTEST = 9,   // oz_wait_selftest: a wait that nothing satisfies
};

// Upper bound for any spin-wait, in SM clock cycles (~2 s at 1.9 GHz).
constexpr long long kWaitBoundCycles = 4000000000LL;

// ---------------------------------------------------------------------------
// element helpers
// ---------------------------------------------------------------------------
__host__ __device__ inline int dtype_size(int dt) {
  return dt == OZ_F64 ? 8 : dt == OZ_F32 ? 4 : (dt == OZ_F16 || dt == OZ_BF16) ? 2 : 1;
}

template <typename T> struct InTraits;
template <> struct InTraits<double> {
  static __device__ __forceinline__ double to_double(double v) { return v; }
  static __device__ __forceinline__ float to_float(double v) { return __double2float_rn(v); }
};
template <> struct InTraits<float> {
  static __device__ __forceinline__ double to_double(float v) { return (double)v; }
  static __device__ __forceinline__ float to_float(float v) { return v; }
};
template <> struct InTraits<__half> {
  static __device__ __forceinline__ double to_double(__half v) { return (double)__half2float(v); }
  static __device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
};
template <> struct InTraits<int8_t> {
  static __device__ __forceinline__ double to_double(int8_t v) { return (double)v; }
  static __device__ __forceinline__ float to_float(int8_t v) { return (float)v; }
};
template <> struct InTraits<__nv_bfloat16> {
  static __device__ __forceinline__ double to_double(__nv_bfloat16 v) {
    return (double)__bfloat162float(v);
  }
  static __device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
};

// The residual lives in fp64 for fp64 inputs and in fp32 otherwise
// (the reference's RESIDUAL_DTYPE, ozaki_triton.py:227).
template <typename TIn> struct RdOf { using type = float; };
template <> struct RdOf<double> { using type = double; };

template <typename TIn, typename RD> __device__ __forceinline__ RD in_to_rd(TIn v) {
  if constexpr (sizeof(RD) == 8) return InTraits<TIn>::to_double(v);
  else return InTraits<TIn>::to_float(v);
}

// Exact float32 2**e for e in [-149, 127] (normal and subnormal).
__device__ __forceinline__ float pow2f(int e) {
  return e >= -126 ? __int_as_float((e + 127) << 23) : __int_as_float(1 << (e + 149));
}
// Exact float64 2**e for e in [-1022, 1023].
__device__ __forceinline__ double pow2d(int e) {
  return __longlong_as_double((long long)(e + 1023) << 52);
}

// ceil(float32(log2(m))) for positive float32 m, including subnormal m.
// The float64 log2 is ~1 ulp (2^-52 relative) accurate; rounding it to
// float32 reproduces the correctly rounded float32 log2 wherever ceil can
// change (the nearest float32 rounding boundary there is >= 2e-10 relative
// away), which is what the reference's tl.ceil(tl.log2(row_max)) computes
// (ozaki_triton.py:174).
__device__ __forceinline__ int ceil_log2_f32(float m) {
  return (int)ceilf(__double2float_rn(log2((double)m)));
}

// ---------------------------------------------------------------------------
// PTX wrappers: mbarrier, fences, TMA, clusters
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and raises *abort) when
// the bound is hit or another role already aborted; never traps.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  volatile int *abort, int code,
                                                  long long bound = kWaitBoundCycles) {
  uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  long long t0 = clock64();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*abort) return false;
      if (clock64() - t0 > bound) {
        *abort = code;
        atomicCAS(&g_device_status, 0, code);
        return false;
      }
    }
  }
}

// 3-D tiled TMA load global -> shared, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// cluster helpers (distributed shared memory)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// Asynchronous remote store of one float into a CTA of the cluster; its 4
// bytes complete on that CTA's mbarrier (both given as shared::cluster addresses).
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                   addr),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Pair (cta_group::2) variants: one MMA spans the two CTAs of a cluster pair.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Arrive on an mbarrier (given as a shared::cluster address, possibly in the
// peer CTA) once every previously issued pair MMA of this thread completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster_addr)
      : "memory");
}
// Arrive on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}
// 3-D TMA load into this CTA's shared memory whose completion is counted on
// the pair leader's mbarrier (bar_cluster_addr).
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map,
                                                 uint32_t bar_cluster_addr, int c0, int c1,
                                                 int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, one instruction, issued by one thread.
template <int KIND>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

template <int KIND>
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
// Wait for the warp's TMEM loads, with the destination registers passed
// through the wait so that no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_ld16_at(uint32_t taddr, uint32_t *r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}


// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row / 1024-byte swizzle atoms).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);        // start address, bits [0,14)
  d |= (uint64_t)1 << 16;                          // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                          // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                          // layout: 128-byte swizzle
  return d;
}

}  // namespace oz
