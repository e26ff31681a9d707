// Exact element step of the row-wise INT8 quantiser, shared by the stand-alone
// quantiser and the fused small-M linear.
//
// The reference computes q = clamp(rne(T(x / T(scale))), -128, 127) with an
// IEEE fp32 divide (inference/src/eager.rs:159-171, torch's bf16 `div`;
// native/comfy-port/kitchen/int8_linear.cu:47-51).  A divide per element is
// the dominant cost of a bandwidth-bound kernel.  For bf16/f16 inputs the
// quotient is computed exactly with one FMA correction (div_exact_short,
// proof at its definition); the vectorised bf16 paths need only the product
// x * RN(1/d), which rounds to the same bf16 (proof at quant8_bf16).  For fp32
// inputs it is formed as x * r with
// r = RN(1 / T(scale)):
//   |x*r - x/s| <= 2^-23 |x/s| (r and the product each round once), i.e. the
//   product is within 2 ulp of the correctly rounded quotient.
// Rounding that fp32 value to T can only differ from rounding the correctly
// rounded quotient if a T rounding midpoint lies within those ulps; the
// midpoint of bf16 (f16) rounding is low 16 (13) bits == 0x8000 (0x1000), so
// any product whose discarded bits sit within +-8 ulp of the midpoint takes the
// exact divide.  For fp32 inputs (no intermediate rounding) the same guard is
// applied around the half-integer boundaries of rne.  Results are therefore
// bit-identical to the divide; the slow path is taken for ~0.03% of elements.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

namespace w8a8 {

// Round an fp32 value to the nearest bf16 (ties to even) with integer ops,
// returned as the fp32 value of that bf16.  Bit-identical to
// __float2bfloat16_rn for every finite input (NaN is not produced by the
// callers); keeps the conversion off the XU pipe.
__device__ __forceinline__ float round_bf16_alu(float v) {
  const uint32_t u = __float_as_uint(v);
  const uint32_t r = u + 0x7FFFu + ((u >> 16) & 1u);
  return __uint_as_float(r & 0xFFFF0000u);
}

// rne(t) for |t| < 2^22 as an int, on the FMA pipe: adding 1.5 * 2^23 makes
// the FPU round t to an integer (ties to even) in the low mantissa bits.
__device__ __forceinline__ int rne_small_int(float t) {
  return __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
}

template <typename T>
struct QuantTraits;

template <>
struct QuantTraits<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  static constexpr float kFiniteMax = 3.3895313892515355e38f;
  static constexpr float kTiny = 1.1754943508222875e-38f;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ float round_t(float v) { return round_bf16_alu(v); }
  // true if rounding v to bf16 is insensitive to an error of a few fp32 ulp
  static __device__ __forceinline__ bool safe(float v) {
    const uint32_t low = __float_as_uint(v) & 0xFFFFu;
    return (low - 0x7FF8u) > 16u;  // unsigned: outside [0x7FF8, 0x8008]
  }
};

template <>
struct QuantTraits<__half> {
  static constexpr int kPerVec = 8;
  static constexpr float kFiniteMax = 65504.0f;
  static constexpr float kTiny = 6.103515625e-05f;
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ float round_t(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ bool safe(float v) {
    const uint32_t low = __float_as_uint(v) & 0x1FFFu;
    // f16 is normal for |v| >= 2^-14; below 0.25 the code is 0 either way
    return (low - 0x0FF8u) > 16u || fabsf(v) < 0.25f;
  }
};

template <>
struct QuantTraits<float> {
  static constexpr int kPerVec = 4;
  static constexpr float kFiniteMax = 3.4028234663852886e38f;
  static constexpr float kTiny = 1.1754943508222875e-38f;
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float round_t(float v) { return v; }
  // rne(v) is insensitive to a few ulp unless v is near k + 0.5
  static __device__ __forceinline__ bool safe(float v) {
    const float f = fabsf(v - truncf(v));
    return fabsf(f - 0.5f) > 8.0f * 1.1920929e-07f * fmaxf(fabsf(v), 1.0f);
  }
};

// Row scale (fp32) from the row's absmax.
//   eager   (inference/src/eager.rs:163-166):      max(amax / 127, 1e-30)
//   kitchen (native/.../int8_linear.cu:206-208):   max(min(amax, finite) * (1/127), 1e-30)
template <typename T>
__device__ __forceinline__ float quant_row_scale(float amax, int kitchen_mode) {
  if (kitchen_mode) {
    return fmaxf(__fmul_rn(fminf(amax, QuantTraits<T>::kFiniteMax), 1.0f / 127.0f), 1.0e-30f);
  }
  return fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-30f);
}

// Scale modes (W8A8_SCALE_* of the public header): 0 eager, 1 kitchen,
// 2 kitchen with the element numerics of the reference's Kitchen CUDA build.
constexpr int kScaleKitchenCuda = 2;

// Divisor actually applied to the elements: the scale rounded to T, with an
// exact zero replaced by T's smallest normal (inference/src/eager.rs:94-109).
// The Kitchen CUDA kernels keep the zero (int8_linear.cu:48-51): a row whose
// scale rounds to 0 in T (an all-zero f16 row: 1e-30 underflows) divides by
// zero there, and quant_code reproduces what its clamp makes of that.
template <typename T>
__device__ __forceinline__ float quant_divisor(float scale, int scale_mode = 0) {
  const float s = QuantTraits<T>::round_t(scale);
  return (s == 0.0f && scale_mode != kScaleKitchenCuda) ? QuantTraits<T>::kTiny : s;
}

// One code: clamp(rne(T(x / div)), -128, 127), given recip = RN(1 / div).
// |x / div| <= 127 * (1 + 2^-7) for every element of the row, so the value
// handed to rne_small_int is far inside its exact range.
__device__ __forceinline__ float div_exact_short(float x, float d, float r);

// With `fast` (the Kitchen CUDA build's numerics, f16 / f32 inputs): the
// approximate divide that --use_fast_math compiles `x / scale` to, then the
// reference's clamp(nearbyint(.)) in float, under which a NaN quotient (0 / 0)
// codes to -128 and +-inf to 127 / -128 (fmaxf returns the non-NaN operand).
// For bf16 the exact quotient rounds to the same bf16 as any quotient within
// 2 fp32 ulp (see the W8A8_SCALE_KITCHEN_CUDA note), so bf16 ignores `fast`.
template <typename T>
__device__ __forceinline__ int quant_code(float x, float div, float recip, bool fast = false) {
  float y;
  if constexpr (!std::is_same<T, __nv_bfloat16>::value) {
    if (fast) {
      const float t = QuantTraits<T>::round_t(__fdividef(x, div));
      return static_cast<int>(fminf(127.0f, fmaxf(-128.0f, rintf(t))));
    }
  }
  if constexpr (std::is_same<T, float>::value) {
    y = __fmul_rn(x, recip);
    if (!QuantTraits<T>::safe(y)) y = __fdiv_rn(x, div);
  } else {
    y = div_exact_short(x, div, recip);  // 16-bit x and divisor: exact
  }
  const int q = rne_small_int(QuantTraits<T>::round_t(y));
  return min(127, max(-128, q));
}

// Correctly rounded x / d for x, d with at most 11 significant bits (bf16 or
// f16 values), from r = RN(1/d), using one FMA correction step:
//   y0 = RN(x r), e = x - y0 d (exact by FMA), y1 = RN(y0 + e r).
// y0 is within 2 ulp of q = x/d, so |e r - (q - y0)| <= |e| |r - 1/d| is
// below 2^-22 ulp(q).  q = (mx/md) 2^k with md <= 2047 odd-part > 1 (else q is
// exact), so q is at least ulp(q) / (4 md) >= 2^-13 ulp(q) away from every
// fp32 rounding midpoint; the single rounding of y0 + e r therefore equals
// RN(q).  Quotients below the fp32 normal range quantise to 0 either way.
__device__ __forceinline__ float div_exact_short(float x, float d, float r) {
  const float y0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-y0, d, x);
  return __fmaf_rn(e, r, y0);
}

// ---- packed fp32 pairs (sm_100 add/sub/mul/fma.rn.f32x2): two elements in
// one 64-bit register pair, one instruction for both; each lane rounds as
// the scalar instruction would.
__device__ __forceinline__ uint64_t pk(float a, float b) {
  return static_cast<uint64_t>(__float_as_uint(a)) | (static_cast<uint64_t>(__float_as_uint(b)) << 32);
}
__device__ __forceinline__ float lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// bf16(x / d) for bf16 values x and d (d > 0 finite) from one product with
// r = RN(1/d): RN(x r) is within 2^-23 |x/d| (relative) of the quotient, while a
// quotient of two 8-bit significands mx / md lies at least 2^-18 |x/d| from every
// bf16 rounding midpoint (|mx 2^9 - m md| / (md 2^9) with md < 2^8, and it is
// never exactly on one: a finite binary expansion of mx / md has at most 8
// significant bits).  So RN_bf16(RN(x r)) == RN_bf16(x / d) for every such pair;
// f16 (11-bit significands) leaves no such margin and keeps div_exact_short.
//
// Eight codes from one 16-byte vector of bf16 (the hot path of the
// quantiser): the product above on packed pairs, paired hardware bf16
// rounding, rne via the 1.5*2^23 trick (packed), and saturating packs (the
// clamp to [-128, 127]).
__device__ __forceinline__ uint2 quant8_bf16(const uint4& v, float div, float recip) {
  (void)div;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const uint64_t r2 = pk(recip, recip);
  const uint64_t magic = pk(12582912.0f, 12582912.0f);
  int q[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t x = pk(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
    const uint64_t y = mul2(x, r2);
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo(y), hi(y));  // .x = lo
    const uint32_t bits = *reinterpret_cast<const uint32_t*>(&b);
    const uint64_t t = add2(pk(__uint_as_float(bits << 16), __uint_as_float(bits & 0xFFFF0000u)), magic);
    q[2 * i] = __float_as_int(lo(t)) - 0x4B400000;
    q[2 * i + 1] = __float_as_int(hi(t)) - 0x4B400000;
  }
  // cvt.pack.sat.s8.s32.b32 d, a, b, c: d = c[15:0] << 16 | sat(a) << 8 | sat(b)
  uint32_t t0, t1, lo, hi;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(t0) : "r"(q[3]), "r"(q[2]));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(lo) : "r"(q[1]), "r"(q[0]), "r"(t0));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(t1) : "r"(q[7]), "r"(q[6]));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(q[5]), "r"(q[4]), "r"(t1));
  return make_uint2(lo, hi);
}

}  // namespace w8a8
