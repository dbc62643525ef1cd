// oz_split.cu -- single-pass split of FP64/FP32/FP16/BF16/INT8 lines into
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
// Kernels:
//   split_rows_f64s    : fp64 rows of 4097..8192 elements with the fp32
//                        residual: three CTAs per SM, level 0 read from
//                        shared memory, later levels from registers.
//   split_rows_tma     : the split axis is contiguous (rows of A, or rows of a
//                        transposed workspace).  512 threads own a line;
//                        whole lines arrive by bulk TMA copies.
//   split_colpairs_tma : fp64 lines that are contiguous columns of a row-major
//                        B (split through B's transposed view like
//                        ozaki_triton.py:593), two per iteration, from 2-D TMA
//                        boxes; no transposed copy.
//   split_cols_tma     : contiguous columns of other dtypes: a cluster of up
//                        to 8 CTAs shares one panel of W columns along K;
//                        per-level column maxima are combined through
//                        distributed shared memory; slices are transposed in
//                        shared memory and written K-contiguous.
//   transpose_lines    : columns into a K-contiguous workspace where neither
//                        column kernel applies (then split_rows_tma).
//   split_any_kernel   : any strides / any K, and int8 inputs.  Recomputes
//                        the residual chain from the input on each level
//                        instead of holding it (s + 1 reads of the line).

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <cudaTypedefs.h>

#include "oz_common.cuh"
#include "oz_log2_table.h"

namespace oz {

// ---------------------------------------------------------------------------
// per-level quantisation (shared by all split kernels)
// ---------------------------------------------------------------------------
template <int SK> struct SliceT;
template <> struct SliceT<OZ_I8> { using type = int8_t; };
template <> struct SliceT<OZ_F16> { using type = __half; };
template <> struct SliceT<OZ_BF16> { using type = __nv_bfloat16; };
template <> struct SliceT<OZ_F32> { using type = float; };

// What a quantisation step hands to the store: the slice value itself, or
// for int8 slices a 32-bit word whose low byte is the int8 value (a
// magic-number float's bits or the clamped integer), so that four of them
// pack into one word with byte permutes.
template <int SK> struct QOut { using type = typename SliceT<SK>::type; };
template <> struct QOut<OZ_I8> { using type = uint32_t; };
template <int SK>
__device__ __forceinline__ typename SliceT<SK>::type to_slice(typename QOut<SK>::type q) {
  if constexpr (SK == OZ_I8) return (int8_t)(q & 0xFFu);
  else return q;
}

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
// fast per-level quantisation for the streaming kernels
//
// Level 0 of an fp64 input (and every level in OZ_RESIDUAL_EXACT mode) works
// on the fp64 residual.  After level 0 the reference's residual is an fp32
// value (its residual buffer is fp32), so levels >= 1 run in fp32 registers:
// x = r * 2^-e is then exact, and the reference's fp64 "x + 0.5, truncate"
// equals exact rounding half away from zero (x + 0.5 needs at most 33 bits
// whenever the result can be nonzero).  Inputs other than fp64 have an fp32
// residual from the start and follow the reference's fp32 arithmetic
// (x + 0.5 rounded to fp32, then truncated).  Rounding to an integer uses the
// 1.5 * 2^23 (fp32) / 1.5 * 2^52 (fp64) magic-number identities instead of
// conversion instructions where that is exact.
// ---------------------------------------------------------------------------
// ceil(float32(log2(m))) for positive float32 m (ozaki_triton.py:174): the
// binade's exponent plus one once the mantissa reaches the binade's
// threshold (oz_log2_table.h); subnormal m (the 1e-38 floor) take the
// float64 log2 route.
__device__ __forceinline__ int ceil_log2_table(float m) {
  const uint32_t b = __float_as_uint(m);
  const uint32_t B = b >> 23;
  if (B == 0) return ceil_log2_f32(m);
  return (int)B - 127 + ((int)(b & 0x7FFFFFu) >= kCeilLog2Thr[B] ? 1 : 0);
}

struct LevelP {
  float scale;      // stored scale 2^e
  int e;
  __device__ __forceinline__ void init(float row_max, int alpha) {
    const float m = fmaxf(1e-38f, row_max);
    e = ceil_log2_table(m) - alpha;               // e in [-149, 127]
    scale = pow2f(e);
  }
  __device__ __forceinline__ double inv_d() const { return pow2d(-e); }   // 2^-e
  // 2^-e is not a float when -e > 127: then it is 2^64 * 2^(-e-64)
  __device__ __forceinline__ bool big() const { return -e > 127; }
  __device__ __forceinline__ float inv2() const { return pow2f(big() ? -e - 64 : -e); }
};

constexpr float kMagicF = 12582912.0f;            // 1.5 * 2^23
constexpr double kMagicD = 6755399441055744.0;    // 1.5 * 2^52

// exact double(n) for any 32-bit n: 1.5 * 2^52 + n, minus 1.5 * 2^52
__device__ __forceinline__ double int_to_double_exact(int n) {
  return __dsub_rn(__hiloint2double(0x43380000 + (n >> 31), n), 6755399441055744.0);
}
// |x| < 128.5 for every level (the scale is at least the line maximum / 2^7,
// up to float32 rounding of the maximum and of its log2), so rounding half
// away from zero gives at least -128 and at most +128: only +128 needs the
// reference's clamp to 127.
__device__ __forceinline__ int clamp_i8(int n) { return min(127, n); }

template <int SK> __device__ __forceinline__ typename SliceT<SK>::type slice_from_f64(double x) {
  if constexpr (SK == OZ_F16) {
    unsigned short h;
    asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(x));
    return __ushort_as_half(h);
  } else if constexpr (SK == OZ_BF16) {
    unsigned short h;
    asm("cvt.rn.bf16.f64 %0, %1;" : "=h"(h) : "d"(x));
    return __ushort_as_bfloat16(h);
  } else {
    return __double2float_rn(x);
  }
}
template <int SK> __device__ __forceinline__ typename SliceT<SK>::type slice_from_f32(float x) {
  if constexpr (SK == OZ_F16) return __float2half_rn(x);
  else if constexpr (SK == OZ_BF16) return __float2bfloat16_rn(x);
  else return x;
}
template <int SK> __device__ __forceinline__ float slice_to_f32(typename SliceT<SK>::type q) {
  if constexpr (SK == OZ_F16) return __half2float(q);
  else if constexpr (SK == OZ_BF16) return __bfloat162float(q);
  else return q;
}

// level on an fp64 residual; the next residual goes to rn_d (EXACT) or,
// rounded to fp32 like the reference's residual buffer, to rn_f.  CLAMP:
// the line maximum reaches 127.25 * scale, so +128 may occur and is clamped
// to 127 (otherwise no element can round to 128).
template <int SK, bool EXACT, bool CLAMP>
__device__ __forceinline__ typename QOut<SK>::type step_f64(double r, double inv_d,
                                                            double nscale, bool upd,
                                                            double &rn_d, float &rn_f) {
  const double x = __dmul_rn(r, inv_d);
  double qd;
  typename QOut<SK>::type q;
  if constexpr (SK == OZ_I8) {
    // the reference's fp64 t = x +- 0.5 (rounded), then trunc(t) =
    // sign(x) * floor(|t|) with floor(|t|) from the magic add rounded toward
    // zero: fl_rz(|t| + 1.5 * 2^52) = 1.5 * 2^52 + floor(|t|), whose low word
    // is floor(|t|) (no conversion instruction; integer sign handling keeps
    // the fp64 temporaries, two registers each, few)
    const double t = __dadd_rn(x, copysign(0.5, x));
    const int qa = __double2loint(__dadd_rz(fabs(t), kMagicD));
    const int sgn = __double2hiint(x) >> 31;
    int n = (qa ^ sgn) - sgn;
    if constexpr (CLAMP) n = clamp_i8(n);
    q = (uint32_t)n;
    qd = int_to_double_exact(n);
  } else {
    q = slice_from_f64<SK>(x);
    qd = (double)slice_to_f32<SK>(q);
  }
  if (upd) {
    // q * scale is exact, so one fused rounding equals the reference's r - q*s
    const double d = __fma_rn(qd, nscale, r);
    if constexpr (EXACT) rn_d = d;
    else rn_f = __double2float_rn(d);
  }
  return q;
}

// Integer rounding of an fp32 x (|x| < 2^22) to q in [-128, 127], returned
// as a float.  floor(t) for t >= 0 is the magic add rounded toward zero:
// fl_rz(t + 1.5 * 2^23) = 1.5 * 2^23 + floor(t).
//   EXACT_HALF (fp64 reference arithmetic, exact "|x| + 0.5"): t =
//     fl_rz(|x| + 0.5) never rounds up across an integer, so floor(t) =
//     floor(|x| + 0.5) exactly.
//   otherwise (fp32 reference arithmetic): t = fl_rn(|x| + 0.5), exactly the
//     reference's rounded sum, then truncated.
template <bool EXACT_HALF>
__device__ __forceinline__ float round_q(float x) {
  const float a = fabsf(x);
  const float t = EXACT_HALF ? __fadd_rz(a, 0.5f) : __fadd_rn(a, 0.5f);
  const float qa = __fsub_rn(__fadd_rz(t, kMagicF), kMagicF);   // floor(t), exact
  return fminf(copysignf(qa, x), 127.0f);     // floor(t) <= 128: see clamp_i8
}
// a word whose low byte is the int8 bit pattern of an integer-valued float q
// in [-128, 127]: 1.5 * 2^23 + q has q's two's complement in its low bits
__device__ __forceinline__ uint32_t q_word(float q) {
  return __float_as_uint(__fadd_rn(q, kMagicF));
}

// x = r * 2^-e in fp32: one multiply, or two when 2^-e exceeds the float range
template <bool BIG>
__device__ __forceinline__ float scale_down(float r, float inv2) {
  if constexpr (BIG) return __fmul_rn(__fmul_rn(r, 18446744073709551616.0f), inv2);   // 2^64
  else return __fmul_rn(r, inv2);
}

// level >= 1 of an fp64 input (fp32-valued residual, fp64 reference
// arithmetic): x is exact and the reference's fp64 "x + 0.5, truncate" is
// exact rounding half away from zero (x + 0.5 needs at most 33 bits whenever
// the result can be nonzero)
template <int SK, bool BIG>
__device__ __forceinline__ typename QOut<SK>::type step_f32_exact(float &r, float inv2,
                                                                  float scale, bool upd) {
  const float x = scale_down<BIG>(r, inv2);
  if constexpr (SK == OZ_I8) {
    const float q = round_q<true>(x);
    if (upd) r = __fmaf_rn(-q, scale, r);   // exact
    return q_word(q);
  } else {
    const auto q = slice_from_f32<SK>(x);
    if (upd) r = __fmaf_rn(-slice_to_f32<SK>(q), scale, r);
    return q;
  }
}

// every level of a non-fp64 input (fp32 residual, fp32 reference arithmetic):
// trunc(fl32(x +- 0.5)) = sign(x) * floor(fl32(|x| + 0.5))
template <int SK, bool BIG>
__device__ __forceinline__ typename QOut<SK>::type step_f32_rd(float &r, float inv2, float scale,
                                                               bool upd) {
  const float x = scale_down<BIG>(r, inv2);   // == r / scale, rounded once
  if constexpr (SK == OZ_I8) {
    const float q = round_q<false>(x);
    if (upd) r = __fsub_rn(r, __fmul_rn(q, scale));
    return q_word(q);
  } else {
    const auto q = slice_from_f32<SK>(x);
    if (upd) r = __fsub_rn(r, __fmul_rn(slice_to_f32<SK>(q), scale));
    return q;
  }
}

// Two int8 steps at once with the packed fp32 instructions of sm_100
// (__fmul2/__fadd2/__ffma2: per component exactly the scalar operations
// above).  |x| + 0.5 is two scalar adds, whose operand takes the absolute
// value for free; the sign goes back on with one bit operation per element.
// EXACT_HALF selects the fp64-input (step_f32_exact) or fp32-input
// (step_f32_rd) rounding of |x| + 0.5; both residual updates are one fused
// r + q * (-scale): q * scale is exact, so this rounds once like r - q*s.
// CLAMP as in step_f64.
template <bool BIG, bool EXACT_HALF, bool CLAMP>
__device__ __forceinline__ void step2_i8(float2 &r, float inv2, float2 nscale, bool upd,
                                         uint32_t &w0, uint32_t &w1) {
  float2 x = r;
  if constexpr (BIG) x = __fmul2_rn(x, make_float2(18446744073709551616.0f, 18446744073709551616.0f));
  x = __fmul2_rn(x, make_float2(inv2, inv2));
  const float2 t = EXACT_HALF ? make_float2(__fadd_rz(fabsf(x.x), 0.5f), __fadd_rz(fabsf(x.y), 0.5f))
                              : make_float2(__fadd_rn(fabsf(x.x), 0.5f), __fadd_rn(fabsf(x.y), 0.5f));
  const float2 f = __fadd2_rz(t, make_float2(kMagicF, kMagicF));
  const float2 qa = __fadd2_rn(f, make_float2(-kMagicF, -kMagicF));   // floor(t), exact
  float2 q = make_float2(copysignf(qa.x, x.x), copysignf(qa.y, x.y));
  if constexpr (CLAMP) q = make_float2(fminf(q.x, 127.0f), fminf(q.y, 127.0f));
  const float2 m = __fadd2_rn(q, make_float2(kMagicF, kMagicF));
  w0 = __float_as_uint(m.x);
  w1 = __float_as_uint(m.y);
  if (upd) r = __ffma2_rn(q, nscale, r);
}

// max(|a|, |b|, |c|) in one instruction (three-input max of sm_100)
__device__ __forceinline__ float max_abs3(float a, float b, float c) {
  float d;
  asm("max.abs.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// bulk (non-tensor) TMA copy global -> shared, completion counted on `bar`
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Per-thread storage of one line's values and the level loop, shared by the
// streaming kernels.  NV values per thread; `emit(l, idx, q)` stores slice
// element idx of level l; `reduce(m, l)` returns the line max over the
// threads of the line.
// REG64 = false: an fp64 line whose level 0 the caller runs itself (from
// shared memory, split_rows_f64s): no fp64 registers, levels from `first`.
template <typename TIn, int SK, int NV, bool EXACT, bool REG64 = true> struct LineLevels {
  using ST = typename SliceT<SK>::type;
  using QT = typename QOut<SK>::type;
  static constexpr bool F64IN = sizeof(TIn) == 8;
  static_assert(REG64 || (F64IN && !EXACT), "only fp64 lines with an fp32 residual drop vd");
  double vd[F64IN && REG64 ? NV : 1];
  // fp32 values as register pairs (the packed f32x2 steps take both halves)
  float2 vf2[(NV + 1) / 2];
  __device__ __forceinline__ float &vf(int i) { return (i & 1) ? vf2[i >> 1].y : vf2[i >> 1].x; }

  __device__ __forceinline__ void set(int i, TIn v) {
    if constexpr (F64IN && REG64) vd[i] = v;
    else vf(i) = InTraits<TIn>::to_float(v);
  }

  // emit(l, i, q) stores one slice element (q as QOut: see there) and must
  // not synchronise (it runs inside data-dependent branches); end_level(l)
  // runs once per level on every thread, after all of that level's emits.
  template <typename Reduce, typename Emit, typename Scale, typename EndLevel>
  __device__ __forceinline__ void run(int s, int alpha, Reduce reduce, Emit emit, Scale put_scale,
                                      EndLevel end_level, int first = 0) {
    for (int l = first; l < s; ++l) {
      const bool upd = l < s - 1;
      const bool on_f64 = REG64 && F64IN && (EXACT || l == 0);
      float m;
      if (on_f64) {
        double md = 0.0;
        if constexpr (REG64) {
#pragma unroll
          for (int i = 0; i < NV; ++i) md = fmax(md, fabs(vd[i]));
        }
        m = __double2float_rn(md);
      } else {
        m = 0.f;
#pragma unroll
        for (int i = 0; i + 1 < NV; i += 2) m = max_abs3(m, vf(i), vf(i + 1));
        if constexpr (NV % 2 == 1) m = fmaxf(m, fabsf(vf(NV - 1)));
      }
      m = reduce(m, l);
      LevelP lv;
      lv.init(m, alpha);
      put_scale(l, lv.scale);
      // int8: only a line whose maximum reaches 127.25 * scale (exact in
      // fp32 for every int8 scale) can round an element to +128; the clamp
      // is skipped on the others (fp64 maxima are rounded to fp32 at most
      // 2^-24 below the true maximum, far from the 127.5 that rounds up)
      const bool clamp = SK == OZ_I8 && m >= 127.25f * lv.scale;
      if (on_f64) {
        if constexpr (F64IN && REG64) {
          const double inv_d = lv.inv_d();
          const double nscale = -(double)lv.scale;
          auto level = [&](auto clamp_tag) {
            constexpr bool C = decltype(clamp_tag)::value;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
              double nd = 0.0;
              float nf = 0.f;
              QT q = step_f64<SK, EXACT, C>(vd[i], inv_d, nscale, upd, nd, nf);
              if constexpr (EXACT) vd[i] = nd;
              else vf(i) = nf;
              emit(l, i, q);
            }
          };
          if (clamp) level(std::true_type{});
          else level(std::false_type{});
        }
      } else if constexpr (SK == OZ_I8 && NV % 2 == 0) {
        const float inv2 = lv.inv2();
        const float2 nscale = make_float2(-lv.scale, -lv.scale);
        auto level = [&](auto big_tag, auto clamp_tag) {
          constexpr bool BIG = decltype(big_tag)::value, C = decltype(clamp_tag)::value;
#pragma unroll
          for (int i = 0; i < NV; i += 2) {
            uint32_t w0, w1;
            step2_i8<BIG, F64IN, C>(vf2[i >> 1], inv2, nscale, upd, w0, w1);
            emit(l, i, w0);
            emit(l, i + 1, w1);
          }
        };
        if (!lv.big()) {
          if (clamp) level(std::false_type{}, std::true_type{});
          else level(std::false_type{}, std::false_type{});
        } else {
          if (clamp) level(std::true_type{}, std::true_type{});
          else level(std::true_type{}, std::false_type{});
        }
      } else if (!lv.big()) {
        const float inv2 = lv.inv2();
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          QT q;
          if constexpr (F64IN) q = step_f32_exact<SK, false>(vf(i), inv2, lv.scale, upd);
          else q = step_f32_rd<SK, false>(vf(i), inv2, lv.scale, upd);
          emit(l, i, q);
        }
      } else {
        const float inv2 = lv.inv2();
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          QT q;
          if constexpr (F64IN) q = step_f32_exact<SK, true>(vf(i), inv2, lv.scale, upd);
          else q = step_f32_rd<SK, true>(vf(i), inv2, lv.scale, upd);
          emit(l, i, q);
        }
      }
      end_level(l);
    }
  }
};

// ---------------------------------------------------------------------------
// rows: the split axis is contiguous (rows of A)
// ---------------------------------------------------------------------------
constexpr int kRowCTA = 512;
constexpr int kRowMaxStages = 4;
constexpr int kRowSmem = 200 * 1024;

// (batch, line) of a flat row index without a 64-bit division where that is
// avoidable (a 64-bit division is a long instruction sequence, paid per row)
__device__ __forceinline__ void row_coords(int64_t row, int lines, bool one_batch, int64_t &b,
                                           int64_t &line) {
  if (one_batch) {
    b = 0;
    line = row;
  } else if (row <= (int64_t)0xFFFFFFFFu) {
    const uint32_t r = (uint32_t)row, q = r / (uint32_t)lines;
    b = q;
    line = r - q * (uint32_t)lines;
  } else {
    b = row / lines;
    line = row - b * lines;
  }
}

// Elements per thread and chunk of the row kernel: 16-byte chunks of the
// input, except fp64, whose 32-byte chunks (two 16-byte reads) give int8
// slices 4-byte stores.
template <typename TIn> __host__ __device__ constexpr int row_vec() {
  return sizeof(TIn) == 8 ? 4 : 16 / (int)sizeof(TIn);
}

// VEC slice values -> one store.  int8: the low bytes of VEC QOut words,
// packed with byte permutes (3 per 4 values).
template <int SK, int VEC>
__device__ __forceinline__ void store_slices(typename SliceT<SK>::type *dst,
                                             const typename QOut<SK>::type (&q)[VEC]) {
  if constexpr (SK == OZ_I8) {
    static_assert(VEC % 4 == 0, "int8 slices are stored 4 at a time");
    uint32_t w[VEC / 4];
#pragma unroll
    for (int j = 0; j < VEC / 4; ++j)
      w[j] = __byte_perm(__byte_perm(q[4 * j], q[4 * j + 1], 0x0040),
                         __byte_perm(q[4 * j + 2], q[4 * j + 3], 0x0040), 0x5410);
    if constexpr (VEC == 4) *reinterpret_cast<uint32_t *>(dst) = w[0];
    else *reinterpret_cast<uint2 *>(dst) = make_uint2(w[0], w[1]);
  } else {
    Pack<typename SliceT<SK>::type, VEC> pq;
#pragma unroll
    for (int j = 0; j < VEC; ++j) pq.e[j] = q[j];
    *reinterpret_cast<Pack<typename SliceT<SK>::type, VEC> *>(dst) = pq;
  }
}

// Persistent kernel: each iteration takes RPS = 512 / T whole rows; a group
// of T threads owns a row.  Rows arrive by bulk TMA copies into a ring of NS
// stages, are moved to registers, and the stage is refilled with a later
// iteration's rows while the levels are computed.  Thread `tl` of a row
// holds elements [(c*T + tl)*VEC, +VEC) for c < NCH (16- or 32-byte chunks:
// the shared-memory reads are conflict-free or 2-way, the slice stores
// coalesce).
template <typename TIn, int SK, int T, int NCH, bool EXACT, int CTA = kRowCTA>
__global__ void __launch_bounds__(CTA, kRowCTA / CTA)
    split_rows_tma(const TIn *__restrict__ in, int64_t stride_b, int64_t stride_line, int lines,
                   int64_t total, int K, int ld, int s, int alpha,
                   typename SliceT<SK>::type *__restrict__ out, float *__restrict__ scales, int NS,
                   int rowp) {
  using ST = typename SliceT<SK>::type;
  using QT = typename QOut<SK>::type;
  constexpr int VEC = row_vec<TIn>();
  constexpr int NV = NCH * VEC;
  constexpr int RPS = CTA / T;
  extern __shared__ __align__(128) unsigned char smem[];
  const int stage = RPS * rowp;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + NS * stage);
  float *red = reinterpret_cast<float *>(full + kRowMaxStages);   // [2][16]
  const int grp = threadIdx.x / T, tl = threadIdx.x % T;
  const int64_t groups = (total + RPS - 1) / RPS;
  const uint32_t row_bytes = (uint32_t)K * (uint32_t)sizeof(TIn);

  const bool one_batch = total == lines;
  auto issue = [&](int64_t g, int st) {
    int nrows = (int)min((int64_t)RPS, total - g * RPS);
    mbar_arrive_expect_tx(&full[st], (uint32_t)nrows * row_bytes);
    for (int r = 0; r < nrows; ++r) {
      int64_t b, line;
      row_coords(g * RPS + r, lines, one_batch, b, line);
      bulk_load(smem + st * stage + r * rowp, in + b * stride_b + line * stride_line, row_bytes,
                &full[st]);
    }
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < NS && blockIdx.x + (int64_t)i * gridDim.x < groups; ++i)
      issue(blockIdx.x + (int64_t)i * gridDim.x, i);

  // which of this thread's chunks lie inside the row pitch (written), wholly
  // inside K (read as a vector), or straddle K (read element by element);
  // fixed for the whole kernel
  uint32_t in_ld = 0, in_k = 0, part_k = 0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int k0 = (c * T + tl) * VEC;
    in_ld |= (uint32_t)(k0 < ld) << c;
    in_k |= (uint32_t)(k0 + VEC <= K) << c;
    part_k |= (uint32_t)(k0 < K && k0 + VEC > K) << c;
  }

  volatile int abort_flag = 0;
  int it = 0;
  for (int64_t g = blockIdx.x; g < groups; g += gridDim.x, ++it) {
    const int st = it % NS;
    // a timeout is recorded and the loop keeps going so that every thread
    // reaches the same barriers; the output is then reported as undefined
    mbar_wait_bounded(&full[st], (it / NS) & 1, (volatile int *)&abort_flag, DEV_TIMEOUT_PRODUCER);
    const int64_t row = g * RPS + grp;
    const bool active = row < total;
    LineLevels<TIn, SK, NV, EXACT> ll;
    const TIn *srow = reinterpret_cast<const TIn *>(smem + st * stage + grp * rowp) + tl * VEC;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      Pack<TIn, VEC> pk;
      if (active && ((in_k >> c) & 1)) {
        pk = *reinterpret_cast<const Pack<TIn, VEC> *>(srow + c * T * VEC);
      } else {
        const int k0 = (c * T + tl) * VEC;
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          pk.e[e] = (active && ((part_k >> c) & 1) && k0 + e < K) ? srow[c * T * VEC + e]
                                                                  : (TIn)0.0f;
      }
#pragma unroll
      for (int e = 0; e < VEC; ++e) ll.set(c * VEC + e, pk.e[e]);
    }
    __syncthreads();                       // stage consumed by every thread
    if (threadIdx.x == 0) {
      const int64_t gn = g + (int64_t)NS * gridDim.x;
      if (gn < groups) issue(gn, st);
    }
    int64_t b = 0, line = 0;
    if (active) row_coords(row, lines, one_batch, b, line);
    ST *dst = out + (b * s * lines + line) * (int64_t)ld + tl * VEC;
    const uint32_t wmask = active ? in_ld : 0u;
    const int64_t level_stride = (int64_t)lines * ld;
    auto reduce = [&](float m, int l) -> float {
      constexpr int w = T < 32 ? T : 32;
#pragma unroll
      for (int o = w / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if constexpr (T > 32) {
        if ((threadIdx.x & 31) == 0) red[(l & 1) * 16 + (threadIdx.x >> 5)] = m;
        __syncthreads();
        constexpr int nw = T / 32;
        const int lane = threadIdx.x & 31;
        float v = lane < nw ? red[(l & 1) * 16 + (grp * T) / 32 + lane] : 0.f;
#pragma unroll
        for (int o = nw / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        m = __shfl_sync(0xffffffffu, v, 0);
      }
      return m;
    };
    // slices are stored VEC elements at a time, to dl = this level's row
    QT pq[VEC];
    ST *dl = dst;
    auto put_scale = [&](int l, float sc) {
      if (active && tl == 0) scales[(b * s + l) * lines + line] = sc;
      dl = dst + l * level_stride;
    };
    auto emit = [&](int l, int i, QT q) {
      (void)l;
      pq[i % VEC] = q;
      if (i % VEC == VEC - 1) {
        const int c = i / VEC;
        if ((wmask >> c) & 1) store_slices<SK, VEC>(dl + c * T * VEC, pq);
      }
    };
    ll.run(s, alpha, reduce, emit, put_scale, [](int) {});
  }
}

// ---------------------------------------------------------------------------
// fp64 rows with an fp32 residual: level 0 straight from shared memory
// ---------------------------------------------------------------------------
// Three 256-thread CTAs per SM, one row each.  Level 0 reads the row's fp64
// values from the ring stage twice (maximum, then quantisation into the fp32
// residual, which stays in registers); the stage is then handed back to the
// next row's bulk copy while levels 1.. run from registers.  No fp64 value
// is held in registers, so three rows fit per SM instead of two, with three
// barrier domains.  Same element mapping, arithmetic and stores as
// split_rows_tma (thread tl holds elements [(c*T + tl)*4, +4), c < NCH).
constexpr int kRowsSCTA = 256;
constexpr int kRowsSPerSM = 3;

// FULL: the row holds exactly NCH * T * 4 elements and so does its slice row
// (K = ld = 8192 with NCH = 8), so no chunk needs a bound check.
template <int SK, int NCH, bool FULL>
__global__ void __launch_bounds__(kRowsSCTA, kRowsSPerSM)
    split_rows_f64s(const double *__restrict__ in, int64_t stride_b, int64_t stride_line,
                    int lines, int64_t total, int K, int ld, int s, int alpha,
                    typename SliceT<SK>::type *__restrict__ out, float *__restrict__ scales,
                    int rowp) {
  using ST = typename SliceT<SK>::type;
  using QT = typename QOut<SK>::type;
  constexpr int T = kRowsSCTA, VEC = 4, NV = NCH * VEC;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + rowp);
  float *red = reinterpret_cast<float *>(full + 1);   // [2][8]
  const int tl = threadIdx.x;
  const uint32_t row_bytes = (uint32_t)K * 8u;
  const bool one_batch = total == lines;
  auto issue = [&](int64_t row) {
    int64_t b, line;
    row_coords(row, lines, one_batch, b, line);
    mbar_arrive_expect_tx(full, row_bytes);
    bulk_load(smem, in + b * stride_b + line * stride_line, row_bytes, full);
  };
  if (tl == 0) {
    mbar_init(full, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tl == 0 && blockIdx.x < total) issue(blockIdx.x);

  // which chunks lie inside the row pitch (written), wholly inside K (read
  // as a vector) or straddle K (read element by element); fixed per thread
  uint32_t in_ld = 0, in_k = 0, part_k = 0;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int k0 = (c * T + tl) * VEC;
    in_ld |= (uint32_t)(k0 < ld) << c;
    in_k |= (uint32_t)(k0 + VEC <= K) << c;
    part_k |= (uint32_t)(k0 < K && k0 + VEC > K) << c;
  }
  const double *srow = reinterpret_cast<const double *>(smem) + tl * VEC;
  auto chunk = [&](int c) -> Pack<double, VEC> {
    Pack<double, VEC> pk;
    if (FULL || ((in_k >> c) & 1)) {
      pk = *reinterpret_cast<const Pack<double, VEC> *>(srow + c * T * VEC);
    } else {
      const int k0 = (c * T + tl) * VEC;
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        pk.e[e] = (((part_k >> c) & 1) && k0 + e < K) ? srow[c * T * VEC + e] : 0.0;
    }
    return pk;
  };
  // consecutive reductions alternate between two slots (also across rows,
  // where no other barrier separates one row's last level from the next
  // row's first): a slot is rewritten only after the barrier of the
  // reduction in between, which every thread passes after reading it
  int nred = 0;
  auto reduce = [&](float m, int) -> float {
    const int slot = (nred++ & 1) * 8;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tl & 31) == 0) red[slot + (tl >> 5)] = m;
    __syncthreads();
    const int lane = tl & 31;
    float v = lane < T / 32 ? red[slot + lane] : 0.f;
#pragma unroll
    for (int o = T / 64; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return __shfl_sync(0xffffffffu, v, 0);
  };

  volatile int abort_flag = 0;
  int it = 0;
  for (int64_t row = blockIdx.x; row < total; row += gridDim.x, ++it) {
    mbar_wait_bounded(full, it & 1, (volatile int *)&abort_flag, DEV_TIMEOUT_PRODUCER);
    int64_t b, line;
    row_coords(row, lines, one_batch, b, line);
    ST *dst = out + (b * s * lines + line) * (int64_t)ld + tl * VEC;
    const int64_t level_stride = (int64_t)lines * ld;
    QT pq[VEC];
    ST *dl = dst;
    auto put_scale = [&](int l, float sc) {
      if (tl == 0) scales[(b * s + l) * lines + line] = sc;
      dl = dst + l * level_stride;
    };
    auto emit = [&](int l, int i, QT q) {
      (void)l;
      pq[i % VEC] = q;
      if (i % VEC == VEC - 1) {
        const int c = i / VEC;
        if (FULL || ((in_ld >> c) & 1)) store_slices<SK, VEC>(dl + c * T * VEC, pq);
      }
    };
    LineLevels<double, SK, NV, false, false> ll;
    // level 0 from shared memory: the maximum, then the quantisation
    double md = 0.0;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const Pack<double, VEC> pk = chunk(c);
#pragma unroll
      for (int e = 0; e < VEC; ++e) md = fmax(md, fabs(pk.e[e]));
    }
    const float m = reduce(__double2float_rn(md), 0);
    LevelP lv;
    lv.init(m, alpha);
    put_scale(0, lv.scale);
    const bool upd = s > 1;
    const double inv_d = lv.inv_d();
    const double nscale = -(double)lv.scale;
    auto level0 = [&](auto clamp_tag) {
      constexpr bool C = decltype(clamp_tag)::value;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const Pack<double, VEC> pk = chunk(c);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          double nd = 0.0;
          float nf = 0.f;
          const QT q = step_f64<SK, false, C>(pk.e[e], inv_d, nscale, upd, nd, nf);
          ll.vf(c * VEC + e) = nf;
          emit(0, c * VEC + e, q);
        }
      }
    };
    if (SK == OZ_I8 && m >= 127.25f * lv.scale) level0(std::true_type{});
    else level0(std::false_type{});
    __syncthreads();                     // the stage is read by every thread
    if (tl == 0 && row + gridDim.x < total) issue(row + gridDim.x);
    ll.run(s, alpha, reduce, emit, put_scale, [](int) {}, 1);
  }
}

// ---------------------------------------------------------------------------
// fp64 column pairs: the columns of a row-major B without a transposed copy
// ---------------------------------------------------------------------------
// Persistent kernel, one panel of 2 adjacent columns (lines) per iteration.
// The panel's K rows arrive by 2-D TMA boxes of 2 columns x 256 rows (16
// bytes per row, zero-filled past N and K) in chunks of 2048 rows -- one
// ring stage per chunk -- so no transposed fp64 copy of B is written and
// read back.  Each half of the CTA (256 threads) splits one column of the
// panel, so the two columns' levels run side by side with a barrier domain
// each (named barriers 1 and 2; barrier 0 only joins the halves once per
// panel, when the ring stages are handed back).  Thread t of a half holds
// rows c*2048 + t + 256*e (e < 8) of chunk c: lane-consecutive rows, so the
// shared-memory reads of one column are 2-way conflicted at most, and each
// store of a warp writes 32 consecutive slice elements of the K-contiguous
// slice row (rows past K are zero from the TMA fill, which writes the row's
// padding).
constexpr int kPairRows = 2048;                 // rows per chunk (= ring stage)
constexpr int kPairStage = kPairRows * 16;      // 32 KB
constexpr int kPairMaxStages = 6;
constexpr int kPairSmem = 224 * 1024;
constexpr int kPairHalf = kRowCTA / 2;          // threads per column

// barrier over the NT threads of one half of the CTA (ids 1 and 2)
template <int NT = kPairHalf>
__device__ __forceinline__ void half_sync(int half) {
  // immediate barrier ids, so that the kernel reserves three barriers, not all
  if (half == 0) asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
  else asm volatile("bar.sync 2, %0;" ::"n"(NT) : "memory");
}

// FULL: the slice row is exactly the chunks' length (ld == NCH * 2048), so
// no store needs a bound (a per-element bound keeps a predicate per element
// live through the levels).
template <int SK, int NCH, bool EXACT, bool FULL>
__global__ void __launch_bounds__(kRowCTA, 1)
    split_colpairs_tma(const __grid_constant__ CUtensorMap tm_in, int lines, int64_t panels,
                       int ppb, int K, int ld, int s, int alpha,
                       typename SliceT<SK>::type *__restrict__ out, float *__restrict__ scales,
                       int NS) {
  using ST = typename SliceT<SK>::type;
  using QT = typename QOut<SK>::type;
  constexpr int T = kPairHalf, VEC = 8, NV = NCH * VEC;
  static_assert(NV <= 32, "one bit per element in the store mask");
  extern __shared__ __align__(128) unsigned char smem[];
  const int half = threadIdx.x / T, tl = threadIdx.x % T;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + NS * kPairStage);
  float *red = reinterpret_cast<float *>(full + kPairMaxStages) + half * 16;   // [2][8]

  // chunk q (running index over this CTA's chunks) lives in ring slot q % NS
  auto issue = [&](int64_t panel, int c, int slot) {
    const int b = (int)(panel / ppb), n0 = (int)(panel % ppb) * 2;
    mbar_arrive_expect_tx(&full[slot], (uint32_t)kPairStage);
    unsigned char *dst = smem + slot * kPairStage;
#pragma unroll 1
    for (int r = 0; r < kPairRows; r += 256)
      tma_load_3d(dst + r * 16, &tm_in, &full[slot], n0, c * kPairRows + r, b);
  };
  const int64_t my_panels = panels > blockIdx.x ? (panels - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t my_chunks = my_panels * NCH;
  auto chunk_panel = [&](int64_t q) { return blockIdx.x + (q / NCH) * gridDim.x; };
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    prefetch_tmap(&tm_in);
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int64_t q = 0; q < NS && q < my_chunks; ++q) issue(chunk_panel(q), (int)(q % NCH), (int)q);

  // element i = c*VEC + e is slice element k = c*2048 + tl + 256*e; bit i
  // set when k lies inside the slice row (k < ld)
  uint32_t in_ld = 0;
#pragma unroll
  for (int i = 0; i < NV; ++i)
    in_ld |= (uint32_t)((i / VEC) * kPairRows + tl + (i % VEC) * T < ld) << i;

  volatile int abort_flag = 0;
  int64_t q = 0;
  for (int64_t pi = 0; pi < my_panels; ++pi) {
    const int64_t panel = blockIdx.x + pi * gridDim.x;
    const int b = (int)(panel / ppb), n0 = (int)(panel % ppb) * 2;
    const int line = n0 + half;
    LineLevels<double, SK, NV, EXACT> ll;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int64_t qc = q + c;
      const int slot = (int)(qc % NS);
      mbar_wait_bounded(&full[slot], (uint32_t)((qc / NS) & 1), (volatile int *)&abort_flag,
                        DEV_TIMEOUT_PRODUCER);
      const double *src = reinterpret_cast<const double *>(smem + slot * kPairStage) + half;
#pragma unroll
      for (int e = 0; e < VEC; ++e) ll.set(c * VEC + e, src[2 * (tl + e * T)]);
    }
    __syncthreads();                     // the panel's stages consumed by both halves
    if (threadIdx.x == 0)
      for (int c = 0; c < NCH; ++c) {
        const int64_t qn = q + c + NS;
        if (qn < my_chunks) issue(chunk_panel(qn), (int)(qn % NCH), (int)((q + c) % NS));
      }
    q += NCH;
    if (line >= lines) continue;         // odd N: the last panel's second column
    // consecutive reductions alternate between two slots; a slot is
    // rewritten only after the barrier of the reduction in between (and the
    // panels are separated by the barrier above)
    auto reduce = [&](float m, int l) -> float {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if ((tl & 31) == 0) red[(l & 1) * 8 + (tl >> 5)] = m;
      half_sync(half);
      const int lane = tl & 31;
      float v = lane < T / 32 ? red[(l & 1) * 8 + lane] : 0.f;
#pragma unroll
      for (int o = T / 64; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      return __shfl_sync(0xffffffffu, v, 0);
    };
    ST *row0 = out + ((int64_t)b * s * lines + line) * (int64_t)ld + tl;
    ST *dl = row0;
    auto put_scale = [&](int l, float sc) {
      if (tl == 0) scales[((int64_t)b * s + l) * lines + line] = sc;
      dl = row0 + (int64_t)l * lines * ld;
    };
    auto emit = [&](int, int i, QT qv) {
      if (FULL || ((in_ld >> i) & 1)) dl[(i / VEC) * kPairRows + (i % VEC) * T] = to_slice<SK>(qv);
    };
    ll.run(s, alpha, reduce, emit, put_scale, [](int) {});
  }
}

// ---------------------------------------------------------------------------
// fp64 column pairs with K split over a CTA pair (cluster of 2)
// ---------------------------------------------------------------------------
// For columns of 4097..8192 rows whose slice rows are 8192 elements long
// (B of C3), with the fp32 residual.  A cluster of two CTAs takes a panel of
// 2 columns; CTA r holds rows [r*4096, r*4096 + 4096) of it (64 KB, one
// stage), so three CTAs fit per SM.  Each CTA half (128 threads) splits one
// column: level 0 from shared memory (maximum, then quantisation into the
// fp32 residual in registers), then the stage goes to the next panel's copy
// and levels 1.. run from registers.  Per level each half reduces its part
// of the column, writes its partial maximum into its own slot and sends it
// to the peer CTA with an asynchronous remote store that completes on the
// peer's exchange barrier; the exchange barriers and slots alternate by level
// parity, so a value of level l + 1 can never complete level l's barrier.
// Thread t of a half holds rows c*2048 + t + 128*e (c < 2, e < 16) of its
// CTA's part: lane-consecutive rows for the shared-memory reads and stores.
constexpr int kPairKRows = 4096;                // rows per CTA of the pair
constexpr int kPairKThreads = 256;              // 128 per column
constexpr int kPairKPerSM = 3;

template <int SK>
__global__ void __launch_bounds__(kPairKThreads, kPairKPerSM)
    split_colpairs_kx(const __grid_constant__ CUtensorMap tm_in, int lines, int64_t panels,
                      int ppb, int ld, int s, int alpha,
                      typename SliceT<SK>::type *__restrict__ out, float *__restrict__ scales) {
  using ST = typename SliceT<SK>::type;
  using QT = typename QOut<SK>::type;
  constexpr int T = kPairKThreads / 2, VEC = 16, NCH = kPairKRows / kPairRows, NV = NCH * VEC;
  constexpr int STAGE = kPairKRows * 16;        // 64 KB: 2 columns x 4096 rows of fp64
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGE);
  uint64_t *xbar = full + 1;                                   // [2 halves][2 parities]
  float *slot = reinterpret_cast<float *>(xbar + 4);           // [2 halves][2 parities][2 ranks]
  float *red = slot + 8;                                       // [2 halves][2 parities][4 warps]
  const uint32_t rank = cluster_ctarank();
  const int cid = blockIdx.x / 2, ncl = gridDim.x / 2;
  const int half = threadIdx.x / T, tl = threadIdx.x % T;
  const int kbase = (int)rank * kPairKRows;

  auto issue = [&](int64_t panel) {
    const int b = (int)(panel / ppb), n0 = (int)(panel % ppb) * 2;
    mbar_arrive_expect_tx(full, (uint32_t)STAGE);
#pragma unroll 1
    for (int r = 0; r < kPairKRows; r += 256)
      tma_load_3d(smem + r * 16, &tm_in, full, n0, kbase + r, b);
  };
  if (threadIdx.x == 0) {
    mbar_init(full, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 1);
    fence_mbar_init();
    prefetch_tmap(&tm_in);
  }
  cluster_sync();                       // the peer's barriers exist before any remote store
  if (threadIdx.x == 0 && cid < panels) issue(cid);

  volatile int abort_flag = 0;
  uint32_t lc = 0;                      // reductions of this half so far
  auto reduce = [&](float m, int) -> float {
    const int par = (int)(lc & 1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tl & 31) == 0) red[(half * 2 + par) * 4 + (tl >> 5)] = m;
    half_sync<T>(half);
    float *my = slot + (half * 2 + par) * 2;
    uint64_t *xb = &xbar[half * 2 + par];
    if (tl == 0) {
      const float *r4 = red + (half * 2 + par) * 4;
      const float v = fmaxf(fmaxf(r4[0], r4[1]), fmaxf(r4[2], r4[3]));
      my[rank] = v;
      mbar_arrive_expect_tx(xb, 4u);    // the peer's value; the own one is local
      st_async_f32(map_to_cta(smem_u32(my + rank), rank ^ 1u), v,
                   map_to_cta(smem_u32(xb), rank ^ 1u));
    }
    mbar_wait_bounded(xb, (lc >> 1) & 1, (volatile int *)&abort_flag, DEV_TIMEOUT_CLUSTER);
    ++lc;
    return fmaxf(my[0], my[1]);
  };

  int it = 0;
  for (int64_t pw = cid; pw < panels; pw += ncl, ++it) {
    mbar_wait_bounded(full, it & 1, (volatile int *)&abort_flag, DEV_TIMEOUT_PRODUCER);
    const int b = (int)(pw / ppb), n0 = (int)(pw % ppb) * 2;
    const int line = n0 + half;
    const bool col_ok = line < lines;   // odd N: both CTAs still run the exchange
    ST *row0 = out + ((int64_t)b * s * lines + (col_ok ? line : 0)) * (int64_t)ld + kbase + tl;
    ST *dl = row0;
    auto put_scale = [&](int l, float sc) {
      if (rank == 0 && tl == 0 && col_ok) scales[((int64_t)b * s + l) * lines + line] = sc;
      dl = row0 + (int64_t)l * lines * ld;
    };
    auto emit = [&](int, int i, QT qv) {
      if (col_ok) dl[(i / VEC) * kPairRows + (i % VEC) * T] = to_slice<SK>(qv);
    };
    const double *src = reinterpret_cast<const double *>(smem) + half;
    LineLevels<double, SK, NV, false, false> ll;
    // level 0 from shared memory: the maximum, then the quantisation
    double md = 0.0;
#pragma unroll
    for (int i = 0; i < NV; ++i)
      md = fmax(md, fabs(src[2 * ((i / VEC) * kPairRows + tl + (i % VEC) * T)]));
    const float m = reduce(__double2float_rn(md), 0);
    LevelP lv;
    lv.init(m, alpha);
    put_scale(0, lv.scale);
    const bool upd = s > 1;
    const double inv_d = lv.inv_d();
    const double nscale = -(double)lv.scale;
    auto level0 = [&](auto clamp_tag) {
      constexpr bool C = decltype(clamp_tag)::value;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        double nd = 0.0;
        float nf = 0.f;
        const QT q = step_f64<SK, false, C>(src[2 * ((i / VEC) * kPairRows + tl + (i % VEC) * T)],
                                            inv_d, nscale, upd, nd, nf);
        ll.vf(i) = nf;
        emit(0, i, q);
      }
    };
    if (SK == OZ_I8 && m >= 127.25f * lv.scale) level0(std::true_type{});
    else level0(std::false_type{});
    __syncthreads();                     // the stage is read by both halves
    if (threadIdx.x == 0 && pw + ncl < panels) issue(pw + ncl);
    ll.run(s, alpha, reduce, emit, put_scale, [](int) {}, 1);
  }
  cluster_sync();                       // no CTA leaves while the peer may still address it
}

// ---------------------------------------------------------------------------
// columns: the lines are contiguous, the split axis is strided (columns of B)
// ---------------------------------------------------------------------------
constexpr int kColCTA = 512;
constexpr int kMaxCluster = 8;
constexpr int kColSmem = 200 * 1024;

// Persistent cluster kernel: a cluster of CL CTAs owns one panel of W columns
// (W * sizeof(TIn) = 64 bytes) at a time; CTA `rank` holds K rows
// [rank*KC, rank*KC + KC) of it, KC = G * V with G = 512 / W row groups.
// Panels arrive by TMA tiles into a ring of NS stages; per-level column
// maxima are combined across the cluster through distributed shared memory;
// slices are transposed in shared memory and written K-contiguous.
template <typename TIn, int SK, int V, bool EXACT>
__global__ void __launch_bounds__(kColCTA, 1)
    split_cols_tma(const __grid_constant__ CUtensorMap tm_in, int lines, int batch, int K,
                   int ld, int s, int alpha, typename SliceT<SK>::type *__restrict__ out,
                   float *__restrict__ scales, int NS) {
  using ST = typename SliceT<SK>::type;
  constexpr int W = 64 / (int)sizeof(TIn);
  constexpr int G = kColCTA / W;
  constexpr int KC = G * V;
  constexpr int BOXR = KC < 256 ? KC : 256;
  constexpr int STAGE = KC * 64;
  constexpr int PITCH = KC * (int)sizeof(ST) + 16;   // staging row pitch, bytes
  static_assert(V % 4 == 0, "V must be a multiple of 4");

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *outst = smem + NS * STAGE;                         // [W][PITCH]
  float *red = reinterpret_cast<float *>(outst + W * PITCH);        // [G][W]
  float *peer = red + G * W;                                        // [2][kMaxCluster][W]
  uint64_t *full = reinterpret_cast<uint64_t *>(peer + 2 * kMaxCluster * W);
  uint64_t *xbar = full + 4;            // [2] per-level exchange of column maxima, by parity

  const int CL = (int)cluster_nctarank();
  const int rank = (int)cluster_ctarank();
  const int cid = blockIdx.x / CL, ncl = gridDim.x / CL;
  const int npan = (lines + W - 1) / W;
  const int64_t work = (int64_t)npan * batch;
  const int c = threadIdx.x % W, g = threadIdx.x / W;
  const int kbase = rank * KC;

  auto issue = [&](int64_t pw, int st) {
    const int b = (int)(pw / npan), pn = (int)(pw % npan);
    mbar_arrive_expect_tx(&full[st], STAGE);
    for (int r0 = 0; r0 < KC; r0 += BOXR)
      tma_load_3d(smem + st * STAGE + r0 * 64, &tm_in, &full[st], pn * W, kbase + r0, b);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) mbar_init(&full[i], 1);
    mbar_init(&xbar[0], 1);
    mbar_init(&xbar[1], 1);
    fence_mbar_init();
    prefetch_tmap(&tm_in);
  }
  if (CL > 1) cluster_sync();   // peers' barriers exist before any remote store
  else __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < NS && cid + (int64_t)i * ncl < work; ++i) issue(cid + (int64_t)i * ncl, i);
  uint32_t lc = 0;              // levels exchanged so far (exchange barrier phase)

  volatile int abort_flag = 0;
  int it = 0;
  for (int64_t pw = cid; pw < work; pw += ncl, ++it) {
    const int st = it % NS;
    // a timeout here is recorded and the loop keeps going: the cluster must
    // stay in step, and the output is reported as undefined by the status
    mbar_wait_bounded(&full[st], (it / NS) & 1, (volatile int *)&abort_flag, DEV_TIMEOUT_PRODUCER);
    const int b = (int)(pw / npan), pn = (int)(pw % npan);
    const int n = pn * W + c;
    const bool col_ok = n < lines;
    LineLevels<TIn, SK, V, EXACT> ll;
    const TIn *sp = reinterpret_cast<const TIn *>(smem + st * STAGE);
#pragma unroll
    for (int i = 0; i < V / 4; ++i)
#pragma unroll
      for (int u = 0; u < 4; ++u) ll.set(i * 4 + u, sp[(4 * (g + G * i) + u) * W + c]);
    __syncthreads();                       // stage consumed by every thread
    if (threadIdx.x == 0) {
      const int64_t pn2 = pw + (int64_t)NS * ncl;
      if (pn2 < work) issue(pn2, st);
    }
    // Column maxima: CTA-local reduction, then every CTA sends its W partial
    // maxima to every CTA of the cluster with asynchronous remote stores that
    // complete on the receiver's exchange barrier (no cluster-wide barrier
    // per level).  Slots and barriers alternate by level parity: a CTA can
    // only be one level ahead of a peer that still reads the other buffer,
    // and a value of level l + 1 cannot complete level l's barrier.
    auto reduce = [&](float m, int l) -> float {
      (void)l;
      const int pb = (int)(lc & 1);
      red[g * W + c] = m;
      __syncthreads();
      if (threadIdx.x < W) {
        float mm = red[threadIdx.x];
        for (int gg = 1; gg < G; ++gg) mm = fmaxf(mm, red[gg * W + threadIdx.x]);
        float *slot = peer + (pb * kMaxCluster + rank) * W + threadIdx.x;
        if (CL > 1) {
          if (threadIdx.x == 0) mbar_arrive_expect_tx(&xbar[pb], (uint32_t)(CL * W * 4));
          const uint32_t a = smem_u32(slot), xb = smem_u32(&xbar[pb]);
          for (int r = 0; r < CL; ++r)
            st_async_f32(map_to_cta(a, r), mm, map_to_cta(xb, r));
        } else {
          *slot = mm;
        }
      }
      if (CL > 1)
        mbar_wait_bounded(&xbar[pb], (lc >> 1) & 1, (volatile int *)&abort_flag,
                          DEV_TIMEOUT_CLUSTER);
      else __syncthreads();
      ++lc;
      float mm = peer[(pb * kMaxCluster) * W + c];
      for (int r = 1; r < CL; ++r) mm = fmaxf(mm, peer[(pb * kMaxCluster + r) * W + c]);
      return mm;
    };
    auto put_scale = [&](int l, float sc) {
      if (rank == 0 && g == 0 && col_ok) scales[((int64_t)b * s + l) * lines + n] = sc;
    };
    Pack<ST, 4> pq;
    auto emit = [&](int l, int i, typename QOut<SK>::type q) {
      pq.e[i & 3] = to_slice<SK>(q);
      if ((i & 3) == 3)
        *reinterpret_cast<Pack<ST, 4> *>(outst + c * PITCH + 4 * (g + G * (i >> 2)) * sizeof(ST)) =
            pq;
    };
    auto end_level = [&](int l) {
      // level complete in shared memory: coalesced 16-byte stores
      __syncthreads();
      constexpr int CPL = KC * (int)sizeof(ST) / 16;
      ST *dst = out + ((int64_t)b * s + l) * lines * (int64_t)ld;
      for (int id = threadIdx.x; id < W * CPL; id += kColCTA) {
        const int cc = id / CPL, off = id % CPL;
        const int nn = pn * W + cc;
        const int k0 = kbase + off * 16 / (int)sizeof(ST);
        if (nn < lines && k0 < ld)
          *reinterpret_cast<uint4 *>(reinterpret_cast<unsigned char *>(dst + (int64_t)nn * ld + k0)) =
              *reinterpret_cast<const uint4 *>(outst + cc * PITCH + off * 16);
      }
      __syncthreads();
    };
    ll.run(s, alpha, reduce, emit, put_scale, end_level);
  }
  if (CL > 1) cluster_sync();   // no CTA leaves while peers may still address it
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
// both operands of a small product in one launch
// ---------------------------------------------------------------------------
// One CTA per line of A (rows) or of B (columns), in one grid: blocks
// [0, a.batch * a.lines) take A's lines, the rest B's.  The line is read once
// into shared memory in the residual precision and every level works there
// with the generic kernel's per-element arithmetic (quant_step), so the
// slices are the same bits as every other split kernel's.  Used for products
// whose operands are small (launch latency, not bandwidth, is their cost).
struct LineSet {
  const void *in;
  int64_t stride_b, stride_line, stride_k;
  int64_t batch, lines;
  void *slices;
  float *scales;
};
constexpr int kPairSmallThreads = 256;

template <typename TIn, int SK, bool EXACT>
__global__ void __launch_bounds__(kPairSmallThreads)
    split_two_small(const LineSet a, const LineSet b, int K, int ld, int s, int alpha) {
  using RD = typename RdOf<TIn>::type;
  using ST = typename SliceT<SK>::type;
  extern __shared__ __align__(16) unsigned char smem_small[];
  RD *res = reinterpret_cast<RD *>(smem_small);
  __shared__ float red[kPairSmallThreads / 32];
  const int64_t na = a.batch * a.lines;
  const bool is_a = (int64_t)blockIdx.x < na;
  const LineSet &op = is_a ? a : b;
  const int64_t flat = is_a ? (int64_t)blockIdx.x : (int64_t)blockIdx.x - na;
  const int64_t bb = flat / op.lines, line = flat - bb * op.lines;
  const TIn *src = reinterpret_cast<const TIn *>(op.in) + bb * op.stride_b + line * op.stride_line;
  for (int k = threadIdx.x; k < K; k += kPairSmallThreads)
    res[k] = in_to_rd<TIn, RD>(src[(int64_t)k * op.stride_k]);
  __syncthreads();
  ST *dst = reinterpret_cast<ST *>(op.slices) + (bb * s * op.lines + line) * (int64_t)ld;
  for (int l = 0; l < s; ++l) {
    float m = 0.f;
    for (int k = threadIdx.x; k < K; k += kPairSmallThreads) m = fmaxf(m, abs_to_f32<RD>(res[k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
#pragma unroll
    for (int i = 1; i < kPairSmallThreads / 32; ++i) m = fmaxf(m, red[i]);
    Level<RD> lv;
    lv.init(m, alpha);
    if (threadIdx.x == 0) op.scales[(bb * s + l) * op.lines + line] = lv.scale;
    ST *dl = dst + (int64_t)l * op.lines * ld;
    for (int k = threadIdx.x; k < ld; k += kPairSmallThreads) {
      if (k < K) {
        RD r = res[k];
        dl[k] = quant_step<SK, RD, EXACT>(r, lv, l < s - 1);
        res[k] = r;
      } else {
        dl[k] = ST(0.0f);
      }
    }
    __syncthreads();   // red[] and res[] reused by the next level
  }
}

// ---------------------------------------------------------------------------
// transpose of contiguous lines into a K-contiguous workspace
// ---------------------------------------------------------------------------
// ws[(b * lines + n) * kp + k] = in[b * stride_b + k * stride_k + n] for k < K,
// 0 for K <= k < kp.  32 x 32 tiles through padded shared memory; reads and
// writes are coalesced along n and k respectively.
template <typename T>
__global__ void __launch_bounds__(256)
    transpose_lines(const T *__restrict__ in, int64_t stride_b, int64_t stride_k, int lines, int K,
                    int kp, T *__restrict__ ws) {
  __shared__ T tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32, b = blockIdx.z;
  const T *src = in + (int64_t)b * stride_b;
#pragma unroll
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int k = k0 + r, n = n0 + threadIdx.x;
    tile[r][threadIdx.x] = (k < K && n < lines) ? src[(int64_t)k * stride_k + n] : (T)0.0f;
  }
  __syncthreads();
  T *dst = ws + (int64_t)b * lines * kp;
#pragma unroll
  for (int r = threadIdx.y; r < 32; r += 8) {
    const int n = n0 + r, k = k0 + threadIdx.x;
    if (n < lines && k < kp) dst[(int64_t)n * kp + k] = tile[threadIdx.x][r];
  }
}

// ---------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------
namespace {

int sm_count_split() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <typename TIn, int SK, bool EXACT, int T, int NC, int CTA = kRowCTA>
int launch_rows_nc(const TIn *in, int64_t sb, int64_t sl, int64_t batch, int lines, int K, int ld,
                   int s, int alpha, void *slices, float *scales, cudaStream_t st, int NS,
                   int rowp) {
  using ST = typename SliceT<SK>::type;
  auto kern = split_rows_tma<TIn, SK, T, NC, EXACT, CTA>;
  const int smem = NS * (CTA / T) * rowp + kRowMaxStages * 8 + 2 * 16 * 4;
  if (int rc = set_smem_once((const void *)kern, smem, "cudaFuncSetAttribute(split_rows)"))
    return rc;
  const int64_t total = batch * (int64_t)lines;
  const int64_t groups = (total + (CTA / T) - 1) / (CTA / T);
  const int grid =
      (int)std::min<int64_t>(groups, (int64_t)sm_count_split() * (kRowCTA / CTA));
  count_launch();
  kern<<<grid, CTA, smem, st>>>(in, sb, sl, lines, total, K, ld, s, alpha,
                                reinterpret_cast<ST *>(slices), scales, NS, rowp);
  return check_cuda(cudaGetLastError(), "split_rows_tma launch");
}

// Whether two CTAs of the 256-thread fp64 row kernel are resident on one SM
// with the largest dynamic shared memory that path requests (then any
// smaller request fits too).  Asked once per kernel instance: every GPU this
// library runs on is a B200.
template <typename TIn, int SK, bool EXACT>
bool rows_two_ctas_resident() {
  static const bool ok = [] {
    auto kern = split_rows_tma<TIn, SK, 256, 8, EXACT, 256>;
    const int smem = kRowSmem / 2 + kRowMaxStages * 8 + 2 * 16 * 4;
    int blocks = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, 256, smem) != cudaSuccess) {
      (void)cudaGetLastError();   // the failed query's error, not a kernel's
      return false;
    }
    return blocks >= 2;
  }();
  return ok;
}

// fp64 rows, fp32 residual, up to 8192 elements: split_rows_f64s when three
// of its CTAs are resident on one SM (asked once per instance).
template <int SK>
bool rows_f64s_resident(int smem) {
  static int blocks = -1;
  if (blocks < 0) {
    auto kern = split_rows_f64s<SK, 8, false>;
    const int max_smem = 64 * 1024 + 256;
    int b = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, kern, kRowsSCTA, max_smem) !=
            cudaSuccess) {
      (void)cudaGetLastError();
      b = 0;
    }
    blocks = b;
  }
  return smem <= 64 * 1024 + 256 && blocks >= kRowsSPerSM;
}

template <int SK>
int launch_rows_f64s(const double *in, int64_t sb, int64_t sl, int64_t batch, int lines, int K,
                     int ld, int s, int alpha, void *slices, float *scales, cudaStream_t st,
                     int rowp) {
  using ST = typename SliceT<SK>::type;
  const int smem = rowp + 8 + 2 * 8 * 4;
  const int64_t total = batch * (int64_t)lines;
  const int grid = (int)std::min<int64_t>(total, (int64_t)sm_count_split() * kRowsSPerSM);
  auto go = [&](auto kern) -> int {
    if (int rc = set_smem_once((const void *)kern, smem, "cudaFuncSetAttribute(split_rows_f64s)"))
      return rc;
    count_launch();
    kern<<<grid, kRowsSCTA, smem, st>>>(in, sb, sl, lines, total, K, ld, s, alpha,
                                         reinterpret_cast<ST *>(slices), scales, rowp);
    return check_cuda(cudaGetLastError(), "split_rows_f64s launch");
  };
  if (K == 8 * kRowsSCTA * 4 && ld == K) return go(split_rows_f64s<SK, 8, true>);
  return go(split_rows_f64s<SK, 8, false>);
}

template <typename TIn, int SK, bool EXACT>
int launch_rows(const TIn *in, int64_t sb, int64_t sl, int64_t batch, int lines, int K, int ld,
                int s, int alpha, void *slices, float *scales, cudaStream_t st, bool *done) {
  using ST = typename SliceT<SK>::type;
  constexpr int VEC = row_vec<TIn>();
  *done = false;
  // bulk copies need 16-byte aligned rows whose size is a multiple of 16
  // (a last chunk that straddles K is read element by element)
  const bool ok = ((uintptr_t)in % 16 == 0) && (sl * (int64_t)sizeof(TIn)) % 16 == 0 &&
                  (sb * (int64_t)sizeof(TIn)) % 16 == 0 &&
                  (K * (int64_t)sizeof(TIn)) % 16 == 0 && K > 0 && ld % VEC == 0 &&
                  ((int64_t)ld * (int64_t)sizeof(ST)) % 16 == 0;
  if (!ok) return OZ_OK;
  const int rowp = (K * (int)sizeof(TIn) + 127) / 128 * 128;
  auto go = [&](auto t_tag, auto nc_tag) -> int {
    constexpr int T = decltype(t_tag)::value, NC = decltype(nc_tag)::value;
    const int NS = std::min(kRowMaxStages, kRowSmem / ((kRowCTA / T) * rowp));
    if (NS < 1) return OZ_OK;
    *done = true;
    return launch_rows_nc<TIn, SK, EXACT, T, NC>(in, sb, sl, batch, lines, K, ld, s, alpha, slices,
                                                 scales, st, NS, rowp);
  };
  using I = std::integral_constant<int, 0>;
  (void)sizeof(I);
  // short rows: 64 threads per row (8 rows per iteration), long rows: 512
  constexpr int NC_MAX = 32 / VEC;            // at most 32 values per thread
  const int c64 = (ld + 64 * VEC - 1) / (64 * VEC);
  const int c512 = (ld + 512 * VEC - 1) / (512 * VEC);
  if (c64 <= 1) return go(std::integral_constant<int, 64>{}, std::integral_constant<int, 1>{});
  if (c64 <= 2) return go(std::integral_constant<int, 64>{}, std::integral_constant<int, 2>{});
  if (c64 <= 4) return go(std::integral_constant<int, 64>{}, std::integral_constant<int, 4>{});
  if (c512 <= 1) return go(std::integral_constant<int, 512>{}, std::integral_constant<int, 1>{});
  if (c512 <= 2) return go(std::integral_constant<int, 512>{}, std::integral_constant<int, 2>{});
  if constexpr (sizeof(TIn) == 8) {
    // fp64 rows of up to 8192 elements: two 256-thread CTAs per SM, one row
    // each -- two independent barrier domains per SM instead of one (0.228
    // vs 0.264 ms for 8192^2 with 4 int8 slices).  The kernel needs 128
    // registers per thread (ptxas, 20 bytes of spill), so two CTAs fill the
    // register file exactly; if fewer than two are resident, or
    // OZ_SPLIT_ROWS_CTA=512 is set (read on every call), the single
    // 512-thread CTA per SM runs instead.
    const char *env = getenv("OZ_SPLIT_ROWS_CTA");
    const bool two = !(env && atoi(env) == 512);
    // default: level 0 from shared memory, three rows per SM (fp32 residual,
    // rows longer than 4096 elements); OZ_SPLIT_ROWS_CTA=256 or 512 (read on
    // every call) selects the register-resident kernels
    if constexpr (!EXACT) {
      if (!env && c512 > 2 && c512 <= 4 && rows_f64s_resident<SK>(rowp + 8 + 2 * 8 * 4)) {
        *done = true;
        return launch_rows_f64s<SK>(in, sb, sl, batch, lines, K, ld, s, alpha, slices, scales,
                                    st, rowp);
      }
    }
    if (two && c512 <= 4) {
      const int NS = std::min(kRowMaxStages, (kRowSmem / 2) / rowp);
      if (NS >= 1 && rows_two_ctas_resident<TIn, SK, EXACT>()) {
        *done = true;
        return launch_rows_nc<TIn, SK, EXACT, 256, 8, 256>(in, sb, sl, batch, lines, K, ld, s,
                                                          alpha, slices, scales, st, NS, rowp);
      }
    }
  }
  if (c512 <= 4 && NC_MAX >= 4)
    return go(std::integral_constant<int, 512>{}, std::integral_constant<int, (NC_MAX >= 4 ? 4 : 2)>{});
  if (c512 <= 8 && NC_MAX >= 8)
    return go(std::integral_constant<int, 512>{}, std::integral_constant<int, (NC_MAX >= 8 ? 8 : 2)>{});
  if (c512 <= 16 && NC_MAX >= 16)
    return go(std::integral_constant<int, 512>{}, std::integral_constant<int, (NC_MAX >= 16 ? 16 : 2)>{});
  return OZ_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 split_encode_fn() {
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

template <typename TIn, int SK, bool EXACT, int V>
int launch_cols_v(const TIn *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K, int ld,
                  int s, int alpha, void *slices, float *scales, cudaStream_t st, bool *done) {
  using ST = typename SliceT<SK>::type;
  constexpr int W = 64 / (int)sizeof(TIn);
  constexpr int G = kColCTA / W, KC = G * V;
  constexpr int STAGE = KC * 64;
  constexpr int PITCH = KC * (int)sizeof(ST) + 16;
  const int CL = (ld + KC - 1) / KC;
  if (*done || CL > kMaxCluster) return OZ_OK;
  const int fixed = W * PITCH + (G * W + 2 * kMaxCluster * W) * 4 + 8 * 6;
  const int NS = min(4, (kColSmem - fixed) / STAGE);
  if (NS < 1) return OZ_OK;
  *done = true;
  auto enc = split_encode_fn();
  if (!enc) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  const CUtensorMapDataType dt = sizeof(TIn) == 8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT64
                                 : sizeof(TIn) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                    : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  cuuint64_t dims[3] = {(cuuint64_t)lines, (cuuint64_t)K, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(sk * (int64_t)sizeof(TIn)),
                           (cuuint64_t)(sb * (int64_t)sizeof(TIn))};
  cuuint32_t box[3] = {(cuuint32_t)W, (cuuint32_t)(KC < 256 ? KC : 256), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&map, dt, 3, const_cast<TIn *>(in), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled (split) failed (%d)", (int)r);
  const int smem = NS * STAGE + fixed;
  auto kern = split_cols_tma<TIn, SK, V, EXACT>;
  if (int rc = set_smem_once((const void *)kern, smem, "cudaFuncSetAttribute(split_cols)"))
    return rc;
  const int64_t work = (int64_t)((lines + W - 1) / W) * batch;
  const int clusters = (int)std::min<int64_t>(work, (int64_t)std::max(1, sm_count_split() / CL));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * CL));
  cfg.blockDim = dim3(kColCTA);
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
  count_launch();
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, map, lines, (int)batch, K, ld, s, alpha, o,
                                       scales, NS),
                    "split_cols_tma launch");
}

// fp64 columns by panels of 2 (split_colpairs_tma): K <= 4 chunks of 2048
// rows, 16-byte aligned row pitch.  Sets *done when it launched.
template <int SK, bool EXACT>
int launch_colpairs(const double *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K,
                    int ld, int s, int alpha, void *slices, float *scales, cudaStream_t st,
                    bool *done) {
  using ST = typename SliceT<SK>::type;
  *done = false;
  if (((uintptr_t)in % 16) != 0 || (sk * 8) % 16 != 0 || (sb * 8) % 16 != 0 || K <= 0 ||
      K > 4 * kPairRows || ld % 4 != 0 || ((int64_t)ld * (int64_t)sizeof(ST)) % 16 != 0 ||
      ld > 4 * kPairRows || lines < 1)
    return OZ_OK;
  const int nch0 = (std::max(K, ld) + kPairRows - 1) / kPairRows;
  const int nch = nch0 <= 1 ? 1 : nch0 <= 2 ? 2 : 4;
  const int NS = std::min(kPairMaxStages, (kPairSmem - 1024) / kPairStage);
  if (NS < nch) return OZ_OK;                    // a panel's chunks must fit the ring
  auto enc = split_encode_fn();
  if (!enc) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)lines, (cuuint64_t)K, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(sk * 8), (cuuint64_t)(sb * 8)};
  cuuint32_t box[3] = {2, 256, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 3, const_cast<double *>(in), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled (column pairs) failed (%d)", (int)r);
  const int ppb = (lines + 1) / 2;
  const int64_t panels = (int64_t)ppb * batch;
  const int smem = NS * kPairStage + kPairMaxStages * 8 + 2 * 16 * 4;
  const int grid = (int)std::min<int64_t>(panels, (int64_t)sm_count_split());
  ST *o = reinterpret_cast<ST *>(slices);
  auto go = [&](auto kern) -> int {
    if (int rc = set_smem_once((const void *)kern, smem, "cudaFuncSetAttribute(split_colpairs)"))
      return rc;
    count_launch();
    kern<<<grid, kRowCTA, smem, st>>>(map, lines, panels, ppb, K, ld, s, alpha, o, scales, NS);
    *done = true;
    return check_cuda(cudaGetLastError(), "split_colpairs_tma launch");
  };
  const bool full = ld == nch * kPairRows;
  if (nch <= 1)
    return full ? go(split_colpairs_tma<SK, 1, EXACT, true>) : go(split_colpairs_tma<SK, 1, EXACT, false>);
  if (nch <= 2)
    return full ? go(split_colpairs_tma<SK, 2, EXACT, true>) : go(split_colpairs_tma<SK, 2, EXACT, false>);
  return full ? go(split_colpairs_tma<SK, 4, EXACT, true>) : go(split_colpairs_tma<SK, 4, EXACT, false>);
}

// fp64 columns of 4097..8192 rows with 8192-element slice rows and the fp32
// residual: split_colpairs_kx (K split over a CTA pair, three CTAs per SM)
// when its clusters can be resident three CTAs per SM; OZ_SPLIT_COLS=pairs
// (read on every call) selects split_colpairs_tma.  Sets *done when it
// launched.
template <int SK>
int launch_colpairs_kx(const double *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K,
                       int ld, int s, int alpha, void *slices, float *scales, cudaStream_t st,
                       bool *done) {
  using ST = typename SliceT<SK>::type;
  *done = false;
  const char *env = getenv("OZ_SPLIT_COLS");
  if (env && strcmp(env, "pairs") == 0) return OZ_OK;
  if (((uintptr_t)in % 16) != 0 || (sk * 8) % 16 != 0 || (sb * 8) % 16 != 0 ||
      K <= kPairKRows || K > 2 * kPairKRows || ld != 2 * kPairKRows || lines < 1)
    return OZ_OK;
  const int smem = kPairKRows * 16 + 8 * 5 + 4 * 8 + 4 * 16;
  static int resident = -1;
  auto kern = split_colpairs_kx<SK>;
  if (resident < 0) {
    int nb = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kPairKThreads, smem) !=
            cudaSuccess) {
      (void)cudaGetLastError();
      nb = 0;
    }
    resident = nb;
  }
  if (resident < kPairKPerSM) return OZ_OK;
  auto enc = split_encode_fn();
  if (!enc) return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)lines, (cuuint64_t)K, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(sk * 8), (cuuint64_t)(sb * 8)};
  cuuint32_t box[3] = {2, 256, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 3, const_cast<double *>(in), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(OZ_ERR_CUDA, "cuTensorMapEncodeTiled (column pairs, K split) failed (%d)",
                     (int)r);
  const int ppb = (lines + 1) / 2;
  const int64_t panels = (int64_t)ppb * batch;
  const int clusters =
      (int)std::min<int64_t>(panels, (int64_t)sm_count_split() * kPairKPerSM / 2);
  if (int rc = set_smem_once((const void *)kern, smem, "cudaFuncSetAttribute(split_colpairs_kx)"))
    return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * 2));
  cfg.blockDim = dim3(kPairKThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  *done = true;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, map, lines, panels, ppb, ld, s, alpha,
                                       reinterpret_cast<ST *>(slices), scales),
                    "split_colpairs_kx launch");
}

// fp64 columns: the K-split pair kernel where it applies, else the column-pair
// kernel.  Sets *done when one of them launched.
template <int SK, bool EXACT>
int launch_fp64_cols(const double *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K,
                     int ld, int s, int alpha, void *slices, float *scales, cudaStream_t st,
                     bool *done) {
  if constexpr (!EXACT) {
    int rc = launch_colpairs_kx<SK>(in, sb, sk, batch, lines, K, ld, s, alpha, slices, scales, st,
                                    done);
    if (rc != OZ_OK || *done) return rc;
  }
  return launch_colpairs<SK, EXACT>(in, sb, sk, batch, lines, K, ld, s, alpha, slices, scales,
                                    st, done);
}

template <typename TIn, int SK, bool EXACT>
int launch_cols(const TIn *in, int64_t sb, int64_t sk, int64_t batch, int lines, int K, int ld,
                int s, int alpha, void *slices, float *scales, cudaStream_t st, bool *done) {
  using ST = typename SliceT<SK>::type;
  *done = false;
  // TMA: 16-byte aligned base and row pitch; slices rows in 16-byte chunks
  if (((uintptr_t)in % 16) != 0 || (sk * (int64_t)sizeof(TIn)) % 16 != 0 ||
      (sb * (int64_t)sizeof(TIn)) % 16 != 0 || ((int64_t)ld * (int64_t)sizeof(ST)) % 16 != 0 ||
      K <= 0)
    return OZ_OK;
  if constexpr (sizeof(TIn) == 8) {
    int rc = launch_fp64_cols<SK, EXACT>(in, sb, sk, batch, lines, K, ld, s, alpha, slices,
                                         scales, st, done);
    if (rc != OZ_OK || *done) return rc;
  }
  // values per thread: the smallest V whose cluster of <= 8 CTAs covers ld
  int rc = OZ_OK;
  rc = launch_cols_v<TIn, SK, EXACT, 4>(in, sb, sk, batch, lines, K, ld, s, alpha, slices, scales, st, done);
  if (rc == OZ_OK && !*done) rc = launch_cols_v<TIn, SK, EXACT, 8>(in, sb, sk, batch, lines, K, ld, s, alpha, slices, scales, st, done);
  if (rc == OZ_OK && !*done) rc = launch_cols_v<TIn, SK, EXACT, 16>(in, sb, sk, batch, lines, K, ld, s, alpha, slices, scales, st, done);
  if (rc == OZ_OK && !*done) rc = launch_cols_v<TIn, SK, EXACT, 32>(in, sb, sk, batch, lines, K, ld, s, alpha, slices, scales, st, done);
  return rc;
}

// try_only != nullptr: launch the row or column kernel if it applies and
// report that in *try_only; never fall back to split_any_kernel.
template <typename TIn, int SK, bool EXACT>
int dispatch(const void *in_v, int64_t batch, int64_t lines, int64_t K, int64_t sb, int64_t sl,
             int64_t sk, int s, int alpha, void *slices, int64_t ld, float *scales,
             cudaStream_t st, bool *try_only) {
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
  if (try_only) *try_only = done;
  if (rc != OZ_OK || done || try_only) return rc;
  using ST = typename SliceT<SK>::type;
  dim3 grid((unsigned)lines, (unsigned)batch);
  count_launch();
  split_any_kernel<TIn, SK, EXACT><<<grid, kAnyThreads, 0, st>>>(
      in, sb, sl, sk, (int)lines, (int)K, (int)ld, s, alpha, reinterpret_cast<ST *>(slices), scales);
  return check_cuda(cudaGetLastError(), "split_any_kernel launch");
}

template <typename TIn>
int dispatch_slice(int slice_dtype, int residual_mode, const void *in, int64_t batch,
                   int64_t lines, int64_t K, int64_t sb, int64_t sl, int64_t sk, int s, int alpha,
                   void *slices, int64_t ld, float *scales, cudaStream_t st,
                   bool *try_only = nullptr) {
  // a float32 residual is identical in both modes
  const bool exact = residual_mode == OZ_RESIDUAL_EXACT && sizeof(TIn) == 8;
#define OZ_D(SK)                                                                               \
  return exact ? dispatch<TIn, SK, true>(in, batch, lines, K, sb, sl, sk, s, alpha, slices, ld,   \
                                         scales, st, try_only)                                 \
               : dispatch<TIn, SK, false>(in, batch, lines, K, sb, sl, sk, s, alpha, slices, ld,  \
                                          scales, st, try_only);
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

namespace oz {
namespace {

// padded row length (elements) of the transposed workspace: 16-byte rows
int64_t ws_row(int in_dtype, int64_t k) {
  const int es = dtype_size(in_dtype);
  const int64_t vec = 16 / es;
  return (k + vec - 1) / vec * vec;
}

bool ws_applies(int in_dtype, int64_t lines, int64_t k, int64_t stride_line, int64_t stride_k) {
  return stride_line == 1 && stride_k != 1 && k > 0 && lines > 0 &&
         (in_dtype == OZ_F64 || in_dtype == OZ_F32 || in_dtype == OZ_F16 || in_dtype == OZ_BF16);
}

template <typename T>
int transpose_into(const void *in, int64_t batch, int64_t lines, int64_t k, int64_t sb,
                   int64_t sk, int64_t kp, void *ws, cudaStream_t st) {
  dim3 grid((unsigned)((lines + 31) / 32), (unsigned)((kp + 31) / 32), (unsigned)batch);
  count_launch();
  transpose_lines<T><<<grid, dim3(32, 8), 0, st>>>(reinterpret_cast<const T *>(in), sb, sk,
                                                   (int)lines, (int)k, (int)kp,
                                                   reinterpret_cast<T *>(ws));
  return check_cuda(cudaGetLastError(), "transpose_lines launch");
}

// int8 inputs (accepted by the reference, ozaki_triton.py:43-49; an fp32
// residual like every non-fp64 input) take the generic kernel: a rare input
// type that does not need its own streaming instantiations.
int dispatch_int8_input(int slice_dtype, const void *in_v, int64_t batch, int64_t lines,
                        int64_t K, int64_t sb, int64_t sl, int64_t sk, int s, int alpha,
                        void *slices, int64_t ld, float *scales, cudaStream_t st) {
  const int8_t *in = reinterpret_cast<const int8_t *>(in_v);
  dim3 grid((unsigned)lines, (unsigned)batch);
#define OZ_A(SK)                                                                             \
  count_launch();                                                                             \
  split_any_kernel<int8_t, SK, false><<<grid, kAnyThreads, 0, st>>>(                          \
      in, sb, sl, sk, (int)lines, (int)K, (int)ld, s, alpha,                                  \
      reinterpret_cast<typename SliceT<SK>::type *>(slices), scales);                         \
  break;
  switch (slice_dtype) {
    case OZ_I8: OZ_A(OZ_I8)
    case OZ_F16: OZ_A(OZ_F16)
    case OZ_BF16: OZ_A(OZ_BF16)
    default: OZ_A(OZ_F32)
  }
#undef OZ_A
  return check_cuda(cudaGetLastError(), "split_any_kernel launch");
}

// fast_only != nullptr: launch only a row or column kernel and report in
// *fast_only whether one applied (never the generic kernel).
int split_impl(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
               int64_t stride_b, int64_t stride_line, int64_t stride_k, int32_t num_splits,
               int32_t alpha, int slice_dtype, int residual_mode, void *slices, int64_t ld,
               float *scales, void *workspace, int64_t workspace_bytes, void *stream,
               bool *fast_only = nullptr) {
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
  // int8 slices saturate at 2^7 anyway; the rounding needs |x| < 2^22
  if (slice_dtype == OZ_I8 && alpha > 21)
    return set_error(OZ_ERR_INVALID, "alpha %d too large for int8 slices (at most 21)", alpha);
  if (in_dtype != OZ_F64 && in_dtype != OZ_F32 && in_dtype != OZ_F16 && in_dtype != OZ_BF16 &&
      in_dtype != OZ_I8)
    return set_error(OZ_ERR_UNSUPPORTED, "unsupported input dtype %d", in_dtype);
  if (residual_mode != OZ_RESIDUAL_COMPAT && residual_mode != OZ_RESIDUAL_EXACT)
    return set_error(OZ_ERR_INVALID, "unknown residual mode %d", residual_mode);
  if (ld < k) return set_error(OZ_ERR_INVALID, "slice row pitch %lld < k %lld", (long long)ld,
                               (long long)k);
  if (batch == 0 || lines == 0) return OZ_OK;
  if (!in || !slices || !scales) return set_error(OZ_ERR_INVALID, "null pointer");
  if (lines > INT32_MAX || ld > INT32_MAX || k > INT32_MAX || batch > 65535)
    return set_error(OZ_ERR_INVALID, "size out of range (lines=%lld ld=%lld batch=%lld)",
                     (long long)lines, (long long)ld, (long long)batch);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  // contiguous lines (columns of a row-major B).  fp32/fp16/bf16 inputs: the
  // cluster column kernel where it applies (measured faster than transpose +
  // rows for them, e.g. 0.25 vs 0.31 ms for fp32 8192^2 with 2 fp16 slices).
  // fp64 inputs, or where the cluster kernel does not apply: transpose into
  // the workspace, then split the transposed rows with the row kernel
  // (0.51 vs 0.75 ms for fp64 8192^2 with 4 int8 slices).
  if (workspace && in_dtype != OZ_F64 && ws_applies(in_dtype, lines, k, stride_line, stride_k)) {
    bool done = false;
    int rc;
    switch (in_dtype) {
      case OZ_F32:
        rc = dispatch_slice<float>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                   stride_line, stride_k, num_splits, alpha, slices, ld, scales,
                                   st, &done);
        break;
      case OZ_F16:
        rc = dispatch_slice<__half>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                    stride_line, stride_k, num_splits, alpha, slices, ld, scales,
                                    st, &done);
        break;
      default:
        rc = dispatch_slice<__nv_bfloat16>(slice_dtype, residual_mode, in, batch, lines, k,
                                           stride_b, stride_line, stride_k, num_splits, alpha,
                                           slices, ld, scales, st, &done);
        break;
    }
    if (rc != OZ_OK || done) return rc;
  }
  if (workspace && in_dtype == OZ_F64 && ws_applies(in_dtype, lines, k, stride_line, stride_k)) {
    // fp64: the column-pair kernel needs no transposed copy (0.29 vs 0.51 ms
    // with the transpose for 8192^2, 4 int8 slices); the workspace serves
    // the cases it does not take (K > 8192, unaligned pitches)
    bool done = false;
    const bool exact = residual_mode == OZ_RESIDUAL_EXACT;
    const double *ind = reinterpret_cast<const double *>(in);
    int rc;
#define OZ_P(SK)                                                                             \
  rc = exact ? launch_fp64_cols<SK, true>(ind, stride_b, stride_k, batch, (int)lines, (int)k,   \
                                          (int)ld, num_splits, alpha, slices, scales, st, &done) \
             : launch_fp64_cols<SK, false>(ind, stride_b, stride_k, batch, (int)lines, (int)k,  \
                                           (int)ld, num_splits, alpha, slices, scales, st,       \
                                           &done);                                               \
  break;
    switch (slice_dtype) {
      case OZ_I8: OZ_P(OZ_I8)
      case OZ_F16: OZ_P(OZ_F16)
      case OZ_BF16: OZ_P(OZ_BF16)
      default: OZ_P(OZ_F32)
    }
#undef OZ_P
    if (rc != OZ_OK || done) return rc;
  }
  if (workspace && ws_applies(in_dtype, lines, k, stride_line, stride_k)) {
    const int64_t kp = ws_row(in_dtype, k);
    const int64_t need = batch * lines * kp * dtype_size(in_dtype);
    if (workspace_bytes >= need && kp <= ld && (uintptr_t)workspace % 16 == 0) {
      int rc;
      switch (in_dtype) {
        case OZ_F64: rc = transpose_into<double>(in, batch, lines, k, stride_b, stride_k, kp, workspace, st); break;
        case OZ_F32: rc = transpose_into<float>(in, batch, lines, k, stride_b, stride_k, kp, workspace, st); break;
        default: rc = transpose_into<unsigned short>(in, batch, lines, k, stride_b, stride_k, kp, workspace, st); break;
      }
      if (rc) return rc;
      in = workspace;
      stride_b = lines * kp;
      stride_line = kp;
      stride_k = 1;
      k = kp;
    }
  }
  switch (in_dtype) {
    case OZ_I8:
      if (fast_only) {
        *fast_only = false;
        return OZ_OK;
      }
      return dispatch_int8_input(slice_dtype, in, batch, lines, k, stride_b, stride_line,
                                 stride_k, num_splits, alpha, slices, ld, scales, st);
    case OZ_F64:
      return dispatch_slice<double>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                    stride_line, stride_k, num_splits, alpha, slices, ld, scales,
                                    st, fast_only);
    case OZ_F32:
      return dispatch_slice<float>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                   stride_line, stride_k, num_splits, alpha, slices, ld, scales,
                                   st, fast_only);
    case OZ_F16:
      return dispatch_slice<__half>(slice_dtype, residual_mode, in, batch, lines, k, stride_b,
                                    stride_line, stride_k, num_splits, alpha, slices, ld, scales,
                                    st, fast_only);
    default:
      return dispatch_slice<__nv_bfloat16>(slice_dtype, residual_mode, in, batch, lines, k,
                                           stride_b, stride_line, stride_k, num_splits, alpha,
                                           slices, ld, scales, st, fast_only);
  }
}

template <typename TIn, int SK, bool EXACT>
int launch_two_small(const LineSet &a, const LineSet &b, int K, int ld, int s, int alpha,
                     cudaStream_t st) {
  using RD = typename RdOf<TIn>::type;
  const int64_t blocks = a.batch * a.lines + b.batch * b.lines;
  const int smem = K * (int)sizeof(RD);
  count_launch();
  split_two_small<TIn, SK, EXACT><<<(unsigned)blocks, kPairSmallThreads, smem, st>>>(
      a, b, K, ld, s, alpha);
  return check_cuda(cudaGetLastError(), "split_two_small launch");
}

template <typename TIn>
int two_small_slice(int slice_dtype, bool exact, const LineSet &a, const LineSet &b, int K, int ld,
                    int s, int alpha, cudaStream_t st) {
#define OZ_T(SK)                                                                              \
  return exact ? launch_two_small<TIn, SK, true>(a, b, K, ld, s, alpha, st)                    \
               : launch_two_small<TIn, SK, false>(a, b, K, ld, s, alpha, st);
  switch (slice_dtype) {
    case OZ_I8: OZ_T(OZ_I8)
    case OZ_F16: OZ_T(OZ_F16)
    case OZ_BF16: OZ_T(OZ_BF16)
    case OZ_F32: OZ_T(OZ_F32)
  }
#undef OZ_T
  return set_error(OZ_ERR_UNSUPPORTED, "unsupported slice dtype %d", slice_dtype);
}

}  // namespace

// Largest operand pair (elements of A and B together) and line length the
// one-launch split takes: below this the split is launch-bound, and a line
// of the residual fits the default 48 KB of shared memory.
constexpr int64_t kTwoSmallMaxElems = 1ll << 22;
constexpr int64_t kTwoSmallMaxLineBytes = 48 * 1024;

int split_two_small_impl(int in_dtype, const void *a, int64_t a_batches, int64_t m, int64_t a_sb,
                         int64_t a_sm, int64_t a_sk, const void *b, int64_t b_batches, int64_t n,
                         int64_t b_sb, int64_t b_sn, int64_t b_sk, int64_t k, int32_t s,
                         int32_t alpha, int slice_dtype, int residual_mode, void *a_slices,
                         float *a_scales, void *b_slices, float *b_scales, int64_t ld,
                         void *stream, bool *done) {
  *done = false;
  const int rd_bytes = in_dtype == OZ_F64 ? 8 : 4;
  const int64_t lines = a_batches * m + b_batches * n;
  if (k < 1 || k * rd_bytes > kTwoSmallMaxLineBytes || lines * k > kTwoSmallMaxElems ||
      lines > INT32_MAX || ld > INT32_MAX || s < 1 || s > kMaxSplits)
    return OZ_OK;
  LineSet la{a, a_sb, a_sm, a_sk, a_batches, m, a_slices, a_scales};
  LineSet lb{b, b_sb, b_sn, b_sk, b_batches, n, b_slices, b_scales};
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool exact = residual_mode == OZ_RESIDUAL_EXACT && in_dtype == OZ_F64;
  *done = true;
  switch (in_dtype) {
    case OZ_F64: return two_small_slice<double>(slice_dtype, exact, la, lb, (int)k, (int)ld, s, alpha, st);
    case OZ_F32: return two_small_slice<float>(slice_dtype, exact, la, lb, (int)k, (int)ld, s, alpha, st);
    case OZ_F16: return two_small_slice<__half>(slice_dtype, exact, la, lb, (int)k, (int)ld, s, alpha, st);
    case OZ_BF16: return two_small_slice<__nv_bfloat16>(slice_dtype, exact, la, lb, (int)k, (int)ld, s, alpha, st);
    case OZ_I8: return two_small_slice<int8_t>(slice_dtype, exact, la, lb, (int)k, (int)ld, s, alpha, st);
  }
  *done = false;
  return set_error(OZ_ERR_UNSUPPORTED, "unsupported input dtype %d", in_dtype);
}

}  // namespace oz

extern "C" int oz_split(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
                        int64_t stride_b, int64_t stride_line, int64_t stride_k,
                        int32_t num_splits, int32_t alpha, int slice_dtype, int residual_mode,
                        void *slices, int64_t ld, float *scales, void *stream) {
  return oz::split_impl(in, in_dtype, batch, lines, k, stride_b, stride_line, stride_k,
                        num_splits, alpha, slice_dtype, residual_mode, slices, ld, scales, nullptr,
                        0, stream);
}

extern "C" int64_t oz_split_workspace_bytes(int in_dtype, int64_t batch, int64_t lines,
                                            int64_t k, int64_t stride_line, int64_t stride_k) {
  if (!oz::ws_applies(in_dtype, lines, k, stride_line, stride_k) || batch <= 0) return 0;
  return batch * lines * oz::ws_row(in_dtype, k) * oz::dtype_size(in_dtype);
}

extern "C" int oz_split_ex(const void *in, int in_dtype, int64_t batch, int64_t lines, int64_t k,
                           int64_t stride_b, int64_t stride_line, int64_t stride_k,
                           int32_t num_splits, int32_t alpha, int slice_dtype, int residual_mode,
                           void *slices, int64_t ld, float *scales, void *workspace,
                           int64_t workspace_bytes, void *stream) {
  return oz::split_impl(in, in_dtype, batch, lines, k, stride_b, stride_line, stride_k,
                        num_splits, alpha, slice_dtype, residual_mode, slices, ld, scales,
                        workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// allocation-free variant of oz_split_ex
// ---------------------------------------------------------------------------
// Scratch for the column transpose of oz_split_noalloc: a fixed array in
// device memory, present on every GPU that loads the library until the
// process exits.  Host code must not hand the symbol itself to a kernel (on
// the host it is only a stand-in); the device address is looked up once per
// device with cudaGetSymbolAddress.
namespace oz {
constexpr int64_t kNoAllocScratchBytes = 32ll << 20;   // 32 MiB
}
static __device__ __align__(256) unsigned char g_split_scratch[oz::kNoAllocScratchBytes];

namespace oz {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// device address of g_split_scratch on the current device (looked up on the
// first call for that device)
int scratch_address(void **out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= kMaxDevices) return set_error(OZ_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_split_scratch),
                            "cudaGetSymbolAddress(g_split_scratch)"))
      return rc;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return OZ_OK;
}
}  // namespace
}  // namespace oz

extern "C" int64_t oz_split_noalloc_max_bytes(void) { return oz::kNoAllocScratchBytes; }

extern "C" int oz_split_noalloc(const void *in, int in_dtype, int64_t batch, int64_t lines,
                                int64_t k, int64_t stride_b, int64_t stride_line, int64_t stride_k,
                                int32_t num_splits, int32_t alpha, int slice_dtype,
                                int residual_mode, void *slices, int64_t ld, float *scales,
                                void *stream) {
  using namespace oz;
  const int64_t need =
      oz_split_workspace_bytes(in_dtype, batch, lines, k, stride_line, stride_k);
  if (need > kNoAllocScratchBytes) {
    // a column kernel that needs no scratch (fp64 column pairs, the cluster
    // kernel) still takes it; otherwise the input is rejected
    bool fast = false;
    if (int rc = split_impl(in, in_dtype, batch, lines, k, stride_b, stride_line, stride_k,
                            num_splits, alpha, slice_dtype, residual_mode, slices, ld, scales,
                            nullptr, 0, stream, &fast))
      return rc;
    if (fast) return OZ_OK;
    return set_error(OZ_ERR_INVALID,
                     "oz_split_noalloc: this input needs %lld bytes of scratch, more than the "
                     "library's fixed %lld-byte device array; use oz_split_ex with a workspace",
                     (long long)need, (long long)kNoAllocScratchBytes);
  }
  void *scratch = nullptr;
  if (need > 0)
    if (int rc = scratch_address(&scratch)) return rc;
  // the transpose writes every workspace byte the split then reads (zero
  // padding included), so the array needs no clearing between calls
  return split_impl(in, in_dtype, batch, lines, k, stride_b, stride_line, stride_k, num_splits,
                    alpha, slice_dtype, residual_mode, slices, ld, scales, scratch, need, stream);
}
