// oz_split.cu -- single-pass split of FP64/FP32/FP16/BF16 lines into
// num_splits low-precision slices plus power-of-two scales (sm_100a).
//
// Replaces split_matrix_kernel (ozaki_triton.py:136-211) and its wrapper
// split_matrix (ozaki_triton.py:214-256).  The reference sweeps K twice per
// level and round-trips an fp32 residual through HBM; here every line is read
// from HBM once, its residual stays in registers for all levels, and every
// slice is written once.  Per level and line the arithmetic is the
// reference's, operation for operation:
//   row_max = max(float32(1e-38), float32(max_k |res|))          (:172, :192)
//   scale   = float32(2^(ceil(log2(row_max)) - alpha))            (:174)
//   x       = res / scale  (in the residual precision rd)          (:196)
//   int8  : q = trunc(clamp(x >= 0 ? x + 0.5 : x - 0.5, -128, 127))   (:199-200)
//   float : q = slice_dtype(x), round to nearest even              (:202)
//   res     = res - q * scale, then rounded to fp32 because the reference's
//             residual buffer is fp32 (:210-211, :233); OZ_RESIDUAL_EXACT keeps rd.
// Division by the power of two is done as an exact multiplication by its
// reciprocal (same correctly rounded result).
//
// Three kernels:
//   split_rows_kernel : the split axis is contiguous (rows of A).  A group of
//                       T threads owns a line; coalesced 16-byte loads.
//   split_cols_kernel : the lines are contiguous (columns of B, split through
//                       B's transposed view like ozaki_triton.py:593).  A
//                       cluster of up to 8 CTAs shares one panel of W columns
//                       along K; per-level column maxima are combined through
//                       distributed shared memory; slices are transposed in
//                       shared memory and written K-contiguous.
//   split_any_kernel  : any strides / any K.  Recomputes the residual chain
//                       from the input on each level instead of holding it
//                       (s + 1 reads of the line); used only when the two
//                       fast kernels do not apply.

#include <cstdio>

#include "oz_common.cuh"

namespace oz {

// ---------------------------------------------------------------------------
// per-level quantisation (shared by all split kernels)
// ---------------------------------------------------------------------------
template <int SK> struct SliceT;
template <> struct SliceT<OZ_I8> { using type = int8_t; };
template <> struct SliceT<OZ_F16> { using type = __half; };
template <> struct SliceT<OZ_BF16> { using type = __nv_bfloat16; };
template <> struct SliceT<OZ_F32> { using type = float; };

template <typename RD> struct Level {
  float scale;   // stored scale (fp32 power of two)
  RD scale_rd;   // the same value in rd
  RD inv1, inv2; // 1/scale == inv1 * inv2, each factor exact in rd
  __device__ __forceinline__ void init(float row_max, int alpha) {
    float m = fmaxf(1e-38f, row_max);
    int e = ceil_log2_f32(m) - alpha;     // scale = 2^e, e in [-149, 127]
    scale = pow2f(e);
    scale_rd = (RD)scale;
    if constexpr (sizeof(RD) == 8) {
      inv1 = 1.0;
      inv2 = pow2d(-e);
    } else {
      // 2^-e may exceed the float range (e < -127): split it in two factors
      if (-e > 127) {
        inv1 = 18446744073709551616.0f;   // 2^64
        inv2 = pow2f(-e - 64);
      } else {
        inv1 = 1.0f;
        inv2 = pow2f(-e);               // -e >= -127 (2^-127 is a float subnormal)
      }
    }
  }
};

__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double sub_rn(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float sub_rn(float a, float b) { return __fsub_rn(a, b); }

template <typename RD> __device__ __forceinline__ int trunc_to_int(RD v);
template <> __device__ __forceinline__ int trunc_to_int<double>(double v) { return __double2int_rz(v); }
template <> __device__ __forceinline__ int trunc_to_int<float>(float v) { return __float2int_rz(v); }

template <int SK, typename RD>
__device__ __forceinline__ typename SliceT<SK>::type to_slice(RD x, RD &q_back) {
  if constexpr (SK == OZ_I8) {
    // round half away from zero in rd, clamp to [-128, 127], truncate
    RD half = (RD)0.5;
    RD t = (x >= (RD)0) ? add_rn(x, half) : sub_rn(x, half);
    t = t < (RD)-128 ? (RD)-128 : t;
    t = t > (RD)127 ? (RD)127 : t;
    int q = trunc_to_int<RD>(t);
    q_back = (RD)q;
    return (int8_t)q;
  } else if constexpr (SK == OZ_F16) {
    unsigned short h;
    if constexpr (sizeof(RD) == 8) asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(x));
    else asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(x));
    __half r = __ushort_as_half(h);
    q_back = (RD)__half2float(r);
    return r;
  } else if constexpr (SK == OZ_BF16) {
    unsigned short h;
    if constexpr (sizeof(RD) == 8) asm("cvt.rn.bf16.f64 %0, %1;" : "=h"(h) : "d"(x));
    else asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(x));
    __nv_bfloat16 r = __ushort_as_bfloat16(h);
    q_back = (RD)__bfloat162float(r);
    return r;
  } else {
    float r;
    if constexpr (sizeof(RD) == 8) r = __double2float_rn(x);
    else r = x;
    q_back = (RD)r;
    return r;
  }
}

// One level applied to one residual value: returns the slice element and,
// when `update`, replaces r by the next level's residual.
template <int SK, typename RD, bool EXACT>
__device__ __forceinline__ typename SliceT<SK>::type quant_step(RD &r, const Level<RD> &lv,
                                                                bool update) {
  RD x;
  if constexpr (sizeof(RD) == 8) x = mul_rn(r, lv.inv2);
  else x = mul_rn(mul_rn(r, lv.inv1), lv.inv2);
  RD qb;
  auto q = to_slice<SK, RD>(x, qb);
  if (update) {
    r = sub_rn(r, mul_rn(qb, lv.scale_rd));
    if constexpr (sizeof(RD) == 8 && !EXACT) r = (double)__double2float_rn(r);
  }
  return q;
}

template <typename RD> __device__ __forceinline__ float abs_to_f32(RD v);
template <> __device__ __forceinline__ float abs_to_f32<double>(double v) {
  return __double2float_rn(fabs(v));
}
template <> __device__ __forceinline__ float abs_to_f32<float>(float v) { return fabsf(v); }

template <typename T, int N> struct alignas(sizeof(T) * N) Pack { T e[N]; };

// ---------------------------------------------------------------------------
// rows: the split axis is contiguous
// ---------------------------------------------------------------------------
constexpr int kRowThreads = 256;

template <typename TIn, int SK, int VEC, int NCH, bool EXACT>
__global__ void __launch_bounds__(kRowThreads)
    split_rows_kernel(const TIn *__restrict__ in, int64_t stride_b, int64_t stride_line, int lines,
                      int K, int ld, int s, int alpha, typename SliceT<SK>::type *__restrict__ out,
                      float *__restrict__ scales, int T) {
  using RD = typename RdOf<TIn>::type;
  using ST = typename SliceT<SK>::type;
  __shared__ float red[2][kRowThreads / 32];

  const int lpb = kRowThreads / T;                 // lines per block
  const int grp = threadIdx.x / T;
  const int tl = threadIdx.x % T;                  // thread within the line group
  const int line = blockIdx.x * lpb + grp;
  const int b = blockIdx.y;
  const bool active = line < lines;

  RD v[NCH][VEC];
  const TIn *src = in + (int64_t)b * stride_b + (int64_t)(active ? line : 0) * stride_line;
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch) {
    int k0 = (ch * T + tl) * VEC;
    if (active && k0 < K) {
      if constexpr (VEC > 1) {
        Pack<TIn, VEC> p = *reinterpret_cast<const Pack<TIn, VEC> *>(src + k0);
#pragma unroll
        for (int e = 0; e < VEC; ++e) v[ch][e] = in_to_rd<TIn, RD>(p.e[e]);
      } else {
        v[ch][0] = in_to_rd<TIn, RD>(src[k0]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) v[ch][e] = (RD)0;
    }
  }

  ST *dst_base = out + ((int64_t)b * s * lines + (active ? line : 0)) * (int64_t)ld;
  for (int l = 0; l < s; ++l) {
    // ---- line max of |res| (max commutes with the monotone rd->fp32 rounding)
    float m = 0.f;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch)
#pragma unroll
      for (int e = 0; e < VEC; ++e) m = fmaxf(m, abs_to_f32<RD>(v[ch][e]));
    const int w = (T < 32) ? T : 32;
    for (int o = w / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (T > 32) {
      if ((threadIdx.x & 31) == 0) red[l & 1][threadIdx.x >> 5] = m;
      __syncthreads();
      const int nw = T / 32, w0 = (grp * T) / 32;
      m = red[l & 1][w0];
      for (int i = 1; i < nw; ++i) m = fmaxf(m, red[l & 1][w0 + i]);
    }
    Level<RD> lv;
    lv.init(m, alpha);
    if (active && tl == 0) scales[((int64_t)b * s + l) * lines + line] = lv.scale;

    ST *dst = dst_base + (int64_t)l * lines * ld;
    const bool upd = l < s - 1;
#pragma unroll
    for (int ch = 0; ch < NCH; ++ch) {
      int k0 = (ch * T + tl) * VEC;
      Pack<ST, VEC> q;
#pragma unroll
      for (int e = 0; e < VEC; ++e) q.e[e] = quant_step<SK, RD, EXACT>(v[ch][e], lv, upd);
      if (active && k0 < ld) *reinterpret_cast<Pack<ST, VEC> *>(dst + k0) = q;
    }
  }
}

// ---------------------------------------------------------------------------
// columns: the lines are contiguous, the split axis is strided
// ---------------------------------------------------------------------------
constexpr int kColThreads = 256;
constexpr int kMaxCluster = 8;

template <typename TIn, int SK, int W, int V, bool EXACT>
__global__ void __launch_bounds__(kColThreads)
    split_cols_kernel(const TIn *__restrict__ in, int64_t stride_b, int64_t stride_k, int lines,
                      int K, int ld, int s, int alpha, typename SliceT<SK>::type *__restrict__ out,
                      float *__restrict__ scales) {
  using RD = typename RdOf<TIn>::type;
  using ST = typename SliceT<SK>::type;
  constexpr int G = kColThreads / W;                 // row groups
  constexpr int KC = G * V;                          // rows of K per CTA
  constexpr int PITCH = KC * (int)sizeof(ST) + 16;   // staging row pitch in bytes
  static_assert(V % 4 == 0, "V must be a multiple of 4");

  extern __shared__ __align__(16) unsigned char smem[];
  float *red = reinterpret_cast<float *>(smem);                 // [G][W]
  float *peer = red + G * W;                                    // [2][kMaxCluster][W]
  unsigned char *stage = smem + ((G * W + 2 * kMaxCluster * W) * 4 + 15) / 16 * 16;

  const int CL = (int)cluster_nctarank();
  const int rank = (int)cluster_ctarank();
  const int panel = blockIdx.x / CL;
  const int b = blockIdx.y;
  const int c = threadIdx.x % W;
  const int g = threadIdx.x / W;
  const int n = panel * W + c;
  const bool col_ok = n < lines;
  const int kbase = rank * KC;

  RD v[V / 4][4];
  const TIn *src = in + (int64_t)b * stride_b + (col_ok ? n : 0);
#pragma unroll
  for (int i = 0; i < V / 4; ++i)
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      int k = kbase + 4 * (g + G * i) + u;
      v[i][u] = (col_ok && k < K) ? in_to_rd<TIn, RD>(src[(int64_t)k * stride_k]) : (RD)0;
    }

  for (int l = 0; l < s; ++l) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < V / 4; ++i)
#pragma unroll
      for (int u = 0; u < 4; ++u) m = fmaxf(m, abs_to_f32<RD>(v[i][u]));
    red[g * W + c] = m;
    __syncthreads();
    if (threadIdx.x < W) {
      float mm = red[threadIdx.x];
      for (int gg = 1; gg < G; ++gg) mm = fmaxf(mm, red[gg * W + threadIdx.x]);
      float *slot = peer + ((l & 1) * kMaxCluster + rank) * W + threadIdx.x;
      if (CL > 1) {
        uint32_t a = smem_u32(slot);
        for (int r = 0; r < CL; ++r) st_cluster_f32(map_to_cta(a, r), mm);
      } else {
        *slot = mm;
      }
    }
    if (CL > 1) cluster_sync();
    else __syncthreads();
    m = peer[((l & 1) * kMaxCluster) * W + c];
    for (int r = 1; r < CL; ++r) m = fmaxf(m, peer[((l & 1) * kMaxCluster + r) * W + c]);

    Level<RD> lv;
    lv.init(m, alpha);
    if (rank == 0 && g == 0 && col_ok) scales[((int64_t)b * s + l) * lines + n] = lv.scale;

    const bool upd = l < s - 1;
#pragma unroll
    for (int i = 0; i < V / 4; ++i) {
      Pack<ST, 4> q;
#pragma unroll
      for (int u = 0; u < 4; ++u) q.e[u] = quant_step<SK, RD, EXACT>(v[i][u], lv, upd);
      *reinterpret_cast<Pack<ST, 4> *>(stage + c * PITCH + 4 * (g + G * i) * sizeof(ST)) = q;
    }
    __syncthreads();
    // coalesced 16-byte stores of W K-contiguous rows
    constexpr int CPL = KC * (int)sizeof(ST) / 16;   // 16-byte chunks per line
    ST *dst = out + ((int64_t)b * s + l) * lines * (int64_t)ld;
    for (int id = threadIdx.x; id < W * CPL; id += kColThreads) {
      int cc = id / CPL, off = id % CPL;
      int nn = panel * W + cc;
      int k0 = kbase + off * 16 / (int)sizeof(ST);
      if (nn < lines && k0 < ld) {
        uint4 val = *reinterpret_cast<const uint4 *>(stage + cc * PITCH + off * 16);
        *reinterpret_cast<uint4 *>(reinterpret_cast<unsigned char *>(dst + (int64_t)nn * ld + k0)) =
            val;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// any layout: recompute the residual chain per level
// ---------------------------------------------------------------------------
constexpr int kAnyThreads = 256;
constexpr int kMaxSplits = 8;

template <typename TIn, int SK, bool EXACT>
__global__ void __launch_bounds__(kAnyThreads)
    split_any_kernel(const TIn *__restrict__ in, int64_t stride_b, int64_t stride_line,
                     int64_t stride_k, int lines, int K, int ld, int s, int alpha,
                     typename SliceT<SK>::type *__restrict__ out, float *__restrict__ scales) {
  using RD = typename RdOf<TIn>::type;
  __shared__ float red[kAnyThreads / 32];
  __shared__ float sm_max[kMaxSplits];
  const int line = blockIdx.x, b = blockIdx.y;
  const TIn *src = in + (int64_t)b * stride_b + (int64_t)line * stride_line;
  Level<RD> lv[kMaxSplits];
  for (int l = 0; l < s; ++l) {
    float m = 0.f;
    for (int k = threadIdx.x; k < K; k += kAnyThreads) {
      RD r = in_to_rd<TIn, RD>(src[(int64_t)k * stride_k]);
      for (int j = 0; j < l; ++j) (void)quant_step<SK, RD, EXACT>(r, lv[j], true);
      m = fmaxf(m, abs_to_f32<RD>(r));
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
      float mm = red[0];
      for (int i = 1; i < kAnyThreads / 32; ++i) mm = fmaxf(mm, red[i]);
      sm_max[l] = mm;
    }
    __syncthreads();
    lv[l].init(sm_max[l], alpha);
    if (threadIdx.x == 0) scales[((int64_t)b * s + l) * lines + line] = lv[l].scale;
  }
  using ST = typename SliceT<SK>::type;
  for (int k = threadIdx.x; k < ld; k += kAnyThreads) {
    RD r = k < K ? in_to_rd<TIn, RD>(src[(int64_t)k * stride_k]) : (RD)0;
    for (int l = 0; l < s; ++l) {
      ST q = quant_step<SK, RD, EXACT>(r, lv[l], l < s - 1);
      out[(((int64_t)b * s + l) * lines + line) * (int64_t)ld + k] = q;
    }
  }
}

// ---------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------
namespace {

template <typename TIn, int SK, bool EXACT, int NC>
int launch_rows_nc(const TIn *in, int64_t sb, int64_t sl, int64_t batch, int lines, int K, int ld,
                   int s, int alpha, void *slices, float *scales, cudaStream_t st, int T) {
  constexpr int VEC = 16 / (int)sizeof(TIn);
  using ST = typename SliceT<SK>::type;
  dim3 grid((unsigned)((lines + (kRowThreads / T) - 1) / (kRowThreads / T)), (unsigned)batch);
  split_rows_kernel<TIn, SK, VEC, NC, EXACT><<<grid, kRowThreads, 0, st>>>(
      in, sb, sl, lines, K, ld, s, alpha, reinterpret_cast<ST *>(slices), scales, T);
  return check_cuda(cudaGetLastError(), "split_rows_kernel launch");
}

template <typename TIn, int SK, bool EXACT>
int launch_rows(const TIn *in, int64_t sb, int64_t sl, int64_t batch, int lines, int K, int ld,
                int s, int alpha, void *slices, float *scales, cudaStream_t st, bool *done) {
  using ST = typename SliceT<SK>::type;
  constexpr int VEC = 16 / (int)sizeof(TIn);
  // 16-byte vector loads need 16-byte aligned rows
  const bool vec_ok = ((uintptr_t)in % 16 == 0) && (sl * (int64_t)sizeof(TIn)) % 16 == 0 &&
                      (sb * (int64_t)sizeof(TIn)) % 16 == 0 && K % VEC == 0 && ld % VEC == 0 &&
                      ((int64_t)ld * (int64_t)sizeof(ST)) % 16 == 0;
  *done = false;
  if (!vec_ok) return OZ_OK;
  // Threads per line T in [32, 256] and chunks per thread NC so that the
  // coverage T * VEC * NC reaches ld (the tail up to ld is written as zeros).
  // At most 64 values per thread are held in registers.
  constexpr int NC_MAX = 64 / VEC;
  int T = 32, nch = 1;
  for (;;) {
    nch = (ld + T * VEC - 1) / (T * VEC);
    if (nch <= NC_MAX || T == 256) break;
    T *= 2;
  }
  if (nch > NC_MAX) return OZ_OK;  // line too long for the register-resident kernel
  *done = true;
  if (nch <= 1) return launch_rows_nc<TIn, SK, EXACT, 1>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales, st, T);
  if (nch <= 2) return launch_rows_nc<TIn, SK, EXACT, 2>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales, st, T);
  if (nch <= 4) return launch_rows_nc<TIn, SK, EXACT, 4>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales, st, T);
  if (nch <= 8) return launch_rows_nc<TIn, SK, EXACT, 8>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales, st, T);
  if constexpr (NC_MAX >= 16)
    if (nch <= 16) return launch_rows_nc<TIn, SK, EXACT, 16>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales, st, T);
  if constexpr (NC_MAX >= 32)
    return launch_rows_nc<TIn, SK, EXACT, (NC_MAX >= 32 ? 32 : 16)>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales, st, T);
  *done = false;
  return OZ_OK;
}

template <typename TIn, int SK, bool EXACT, int W, int V>
int launch_cols_wv(const TIn *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K,
                   int ld, int s, int alpha, void *slices, float *scales, cudaStream_t st,
                   bool *done) {
  using ST = typename SliceT<SK>::type;
  constexpr int G = kColThreads / W, KC = G * V;
  const int CL = (ld + KC - 1) / KC;
  if (*done || CL > kMaxCluster) return OZ_OK;
  *done = true;
  const size_t smem = ((size_t)(G * W + 2 * kMaxCluster * W) * 4 + 15) / 16 * 16 +
                      (size_t)W * (KC * sizeof(ST) + 16);
  auto kern = split_cols_kernel<TIn, SK, W, V, EXACT>;
  if (int rc = check_cuda(
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
          "cudaFuncSetAttribute(split_cols)"))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(CL * ((lines + W - 1) / W)), (unsigned)batch);
  cfg.blockDim = dim3(kColThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ST *o = reinterpret_cast<ST *>(slices);
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, in, sb, sk, lines, K, ld, s, alpha, o, scales),
                    "split_cols_kernel launch");
}

template <typename TIn, int SK, bool EXACT>
int launch_cols(const TIn *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K, int ld,
                int s, int alpha, void *slices, float *scales, cudaStream_t st, bool *done) {
  using ST = typename SliceT<SK>::type;
  *done = false;
  if (((int64_t)ld * (int64_t)sizeof(ST)) % 16 != 0) return OZ_OK;
  // W lines per CTA (row segments of W * sizeof(TIn) bytes), V values per
  // thread, K rows per CTA = (256 / W) * V, cluster of <= 8 CTAs along K.
  // The first shape whose cluster covers ld wins: wide segments first, then
  // short per-thread runs (more CTAs in flight).
  constexpr int WA = 128 / (int)sizeof(TIn);   // 128-byte row segments
  constexpr int WB = WA / 2, WC = WA / 4;
  int rc = OZ_OK;
#define OZ_C(W, V)                                                                          \
  if (rc == OZ_OK && !*done && (W) >= 8)                                                    \
    rc = launch_cols_wv<TIn, SK, EXACT, ((W) >= 8 ? (W) : 8), V>(in, sb, sk, batch, lines, K, ld, \
                                                               s, alpha, slices, scales, st, done);
  OZ_C(WA, 16) OZ_C(WA, 32) OZ_C(WA, 64) OZ_C(WB, 64) OZ_C(WC, 64)
  if constexpr (sizeof(TIn) == 8) { OZ_C(8, 64) }
#undef OZ_C
  return rc;
}

template <typename TIn, int SK, bool EXACT>
int dispatch(const void *in_v, int64_t batch, int64_t lines, int64_t K, int64_t sb, int64_t sl,
             int64_t sk, int s, int alpha, void *slices, int64_t ld, float *scales,
             cudaStream_t st) {
  const TIn *in = reinterpret_cast<const TIn *>(in_v);
  bool done = false;
  int rc = OZ_OK;
  if (sk == 1) {
    rc = launch_rows<TIn, SK, EXACT>(in, sb, sl, batch, (int)lines, (int)K, (int)ld, s, alpha,
                                     slices, scales, st, &done);
  } else if (sl == 1) {
    rc = launch_cols<TIn, SK, EXACT>(in, sb, sk, batch, (int)lines, (int)K, (int)ld, s, alpha,
                                     slices, scales, st, &done);
  }
  if (rc != OZ_OK || done) return rc;
  using ST = typename SliceT<SK>::type;
  dim3 grid((unsigned)lines, (unsigned)batch);
  split_any_kernel<TIn, SK, EXACT><<<grid, kAnyThreads, 0, st>>>(
      in, sb, sl, sk, (int)lines, (int)K, (int)ld, s, alpha, reinterpret_cast<ST *>(slices), scales);
  return check_cuda(cudaGetLastError(), "split_any_kernel launch");
}

template <typename TIn>
int dispatch_slice(int slice_dtype, int residual_mode, const void *in, int64_t batch,
                   int64_t lines, int64_t K, int64_t sb, int64_t sl, int64_t sk, int s, int alpha,
                   void *slices, int64_t ld, float *scales, cudaStream_t st) {
  // a float32 residual is identical in both modes
  const bool exact = residual_mode == OZ_RESIDUAL_EXACT && sizeof(TIn) == 8;
#define OZ_D(SK)                                                                               \
  return exact ? dispatch<TIn, SK, true>(in, batch, lines, K, sb, sl, sk, s, alpha, slices, ld,   \
                                         scales, st)                                           \
               : dispatch<TIn, SK, false>(in, batch, lines, K, sb, sl, sk, s, alpha, slices, ld,  \
                                          scales, st);
  switch (slice_dtype) {
    case OZ_I8: OZ_D(OZ_I8)
    case OZ_F16: OZ_D(OZ_F16)
    case OZ_BF16: OZ_D(OZ_BF16)
    case OZ_F32: OZ_D(OZ_F32)
  }
#undef OZ_D
  return set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
}

}  // namespace
int status_split(int *value, bool clear) { return read_status_word(value, clear); }

}  // namespace oz

extern "C" int64_t oz_slice_row_bytes(int64_t k, int slice_dtype) {
  int64_t bytes = k * oz::dtype_size(slice_dtype);
  return (bytes + 127) / 128 * 128;
}

extern "C" int oz_split(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
                        int64_t stride_b, int64_t stride_line, int64_t stride_k,
                        int32_t num_splits, int32_t alpha, int slice_dtype, int residual_mode,
                        void *slices, int64_t ld, float *scales, void *stream) {
  using namespace oz;
  if (num_splits < 1 || num_splits > kMaxSplits)
    return set_error(OZ_ERR_INVALID, "num_splits must be in [1, %d], got %d", kMaxSplits,
                     num_splits);
  if (batch < 0 || lines < 0 || k < 0)
    return set_error(OZ_ERR_INVALID, "negative size (batch=%lld lines=%lld k=%lld)",
                     (long long)batch, (long long)lines, (long long)k);
  if (alpha < 1 || alpha > 23) return set_error(OZ_ERR_INVALID, "alpha out of range: %d", alpha);
  if (slice_dtype != OZ_I8 && slice_dtype != OZ_F16 && slice_dtype != OZ_BF16 &&
      slice_dtype != OZ_F32)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
  if (residual_mode != OZ_RESIDUAL_COMPAT && residual_mode != OZ_RESIDUAL_EXACT)
    return set_error(OZ_ERR_INVALID, "unknown residual mode %d", residual_mode);
  if (ld < k) return set_error(OZ_ERR_INVALID, "slice row pitch %lld < k %lld", (long long)ld,
                               (long long)k);
  if (batch == 0 || lines == 0) return OZ_OK;
  if (!in || !slices || !scales) return set_error(OZ_ERR_INVALID, "null pointer");
  if (lines > INT32_MAX || ld > INT32_MAX || batch > 65535)
    return set_error(OZ_ERR_INVALID, "size out of range (lines=%lld ld=%lld batch=%lld)",
                     (long long)lines, (long long)ld, (long long)batch);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (in_dtype) {
    case OZ_F64:
      return dispatch_slice<double>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                    stride_line, stride_k, num_splits, alpha, slices, ld, scales, st);
    case OZ_F32:
      return dispatch_slice<float>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                   stride_line, stride_k, num_splits, alpha, slices, ld, scales, st);
    case OZ_F16:
      return dispatch_slice<__half>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                    stride_line, stride_k, num_splits, alpha, slices, ld, scales, st);
    case OZ_BF16:
      return dispatch_slice<__nv_bfloat16>(slice_dtype, residual_mode, in, batch, lines, k,
                                           stride_b, stride_line, stride_k, num_splits, alpha,
                                           slices, ld, scales, st);
  }
  return set_error(OZ_ERR_UNSUPPORTED, "unsupported input dtype %d", in_dtype);
}
