// Per-token (row-wise) dynamic INT8 quantiser, bf16/f16/f32 -> int8 + fp32
// row scale.  Replaces the reference's quantize_int8_rowwise_kernel
// (native/comfy-port/kitchen/int8_linear.cu:184-227, launcher :1322-1371) and
// its Triton twin (KSRC backends/triton/quantization.py:771-816), with the
// numerics of the eager path (inference/src/eager.rs:159-171) by default.
//
// Layout: a group of WPR warps owns one row.  Each thread loads up to MAXV
// 16-byte vectors of the row into registers (one HBM read of x), the group
// reduces |x| with shuffles (+ shared memory across warps), and the same
// registers are scaled, rounded and written as int8.  Rows whose byte length or
// base are not 16-byte aligned, or that do not fit in registers, take a
// scalar two-pass path (second pass hits L2).
#include <cuda_bf16.h>
#include <algorithm>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "quant_common.cuh"
#include "sm100_ptx.cuh"
#include "w8a8_internal.h"

namespace w8a8 {
namespace {

constexpr int kQuantThreads = 256;   // threads per CTA

template <typename T>
using InTraits = QuantTraits<T>;

// PCG-hash stochastic rounding noise of the reference's CUDA quantiser
// (native/comfy-port/kitchen/int8_linear.cu:82-95): uniform in [0,1) with 24
// bits, rounded to T, added in T, then floor.
__device__ __forceinline__ uint32_t pcg_hash(uint32_t x) {
  const uint32_t state = x * 747796405u + 2891336453u;
  const uint32_t word = ((state >> ((state >> 28u) + 4u)) ^ state) * 277803737u;
  return (word >> 22u) ^ word;
}

template <typename T, bool kStochastic>
__device__ __forceinline__ int quant_elem(float xv, float div, float recip, int64_t idx,
                                          uint64_t seed, bool fast) {
  if constexpr (!kStochastic) {
    return quant_code<T>(xv, div, recip, fast);
  } else {
    const float scaled = InTraits<T>::round_t(fast ? __fdividef(xv, div) : __fdiv_rn(xv, div));
    const uint64_t key = static_cast<uint64_t>(idx) + seed;
    const uint32_t folded = static_cast<uint32_t>(key) ^ static_cast<uint32_t>(key >> 32);
    const float noise = InTraits<T>::round_t(static_cast<float>(pcg_hash(folded) >> 8) * 0x1.0p-24f);
    const float r = floorf(InTraits<T>::round_t(__fadd_rn(scaled, noise)));
    return static_cast<int>(fminf(127.0f, fmaxf(-128.0f, r)));
  }
}

// |x| max of one 16-byte vector, packed two-at-a-time for 16-bit types.
template <typename T>
__device__ __forceinline__ float vec_absmax(const uint4& v);
template <>
__device__ __forceinline__ float vec_absmax<__nv_bfloat16>(const uint4& v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  __nv_bfloat162 m = __hmax2(__habs2(h[0]), __habs2(h[1]));
  m = __hmax2(m, __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(__low2float(m), __high2float(m));
}
template <>
__device__ __forceinline__ float vec_absmax<__half>(const uint4& v) {
  const __half2* h = reinterpret_cast<const __half2*>(&v);
  __half2 m = __hmax2(__habs2(h[0]), __habs2(h[1]));
  m = __hmax2(m, __hmax2(__habs2(h[2]), __habs2(h[3])));
  return fmaxf(__low2float(m), __high2float(m));
}
template <>
__device__ __forceinline__ float vec_absmax<float>(const uint4& v) {
  return fmaxf(fmaxf(fabsf(__uint_as_float(v.x)), fabsf(__uint_as_float(v.y))),
               fmaxf(fabsf(__uint_as_float(v.z)), fabsf(__uint_as_float(v.w))));
}

// A group of WPR warps owns one row; each thread holds up to MAXV 16-byte
// vectors of it in registers.
// kMode: 0 quantise, 1 write the row absmax only (to `scales`), 2 quantise
// with the row absmax read from `amax_in` (a K-sharded row whose absmax was
// reduced across ranks) instead of the local one.
template <typename T, int WPR, int MAXV, bool kStochastic, int kMode>
__global__ void __launch_bounds__(kQuantThreads) quantize_rowwise_vec_kernel(
    const T* __restrict__ x, int64_t ldx, int8_t* __restrict__ q, int64_t ldq,
    float* __restrict__ scales, int rows, int cols, int scale_mode, uint64_t seed,
    const float* __restrict__ amax_in) {
  constexpr int kPer = InTraits<T>::kPerVec;
  constexpr int kGroupThreads = WPR * 32;
  constexpr int kRowsPerCta = kQuantThreads / kGroupThreads;
  __shared__ float red[kQuantThreads / 32];
  griddep_launch_dependents();  // the GEMM that reads q may start its prologue

  const int group = threadIdx.x / kGroupThreads;
  const int gt = threadIdx.x % kGroupThreads;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int row = blockIdx.x * kRowsPerCta + group;
  const bool live = row < rows;
  const int nvec = cols / kPer;

  const uint4* xrow = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(live ? row : 0) * ldx);
  uint4 v[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = gt + i * kGroupThreads;
    if (live && vi < nvec) v[i] = __ldg(xrow + vi);
  }
  float amax = 0.0f;
  if constexpr (kMode == 2) {
    if (live) amax = __ldg(amax_in + row);
  } else {
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = gt + i * kGroupThreads;
      if (live && vi < nvec) amax = fmaxf(amax, vec_absmax<T>(v[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if constexpr (WPR > 1) {
      if (lane == 0) red[warp] = amax;
      __syncthreads();
      amax = red[group * WPR];
#pragma unroll
      for (int w = 1; w < WPR; ++w) amax = fmaxf(amax, red[group * WPR + w]);
    }
  }
  if (!live) return;
  if constexpr (kMode == 1) {
    if (gt == 0) scales[row] = amax;
    return;
  }
  const float scale = quant_row_scale<T>(amax, scale_mode);
  if (gt == 0) scales[row] = scale;
  const float div = quant_divisor<T>(scale, scale_mode);
  const float recip = __frcp_rn(div);
  const bool fast = scale_mode == kScaleKitchenCuda;
  int8_t* qrow = q + static_cast<int64_t>(row) * ldq;
  const int64_t base_idx = static_cast<int64_t>(row) * cols;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = gt + i * kGroupThreads;
    if constexpr (std::is_same<T, __nv_bfloat16>::value && !kStochastic) {
      if (vi < nvec) reinterpret_cast<uint2*>(qrow)[vi] = quant8_bf16(v[i], div, recip);
      continue;
    }
    if (vi < nvec) {
      const T* e = reinterpret_cast<const T*>(&v[i]);
      uint32_t packed[kPer / 4];
#pragma unroll
      for (int w = 0; w < kPer / 4; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = vi * kPer + w * 4 + j;
          const int qv = quant_elem<T, kStochastic>(InTraits<T>::to_f(e[w * 4 + j]), div, recip,
                                                    base_idx + c, seed, fast);
          word |= (static_cast<uint32_t>(qv) & 0xFFu) << (8 * j);
        }
        packed[w] = word;
      }
      if constexpr (kPer == 8) {
        reinterpret_cast<uint2*>(qrow)[vi] = make_uint2(packed[0], packed[1]);
      } else {
        reinterpret_cast<uint32_t*>(qrow)[vi] = packed[0];
      }
    }
  }
}

// Scalar two-pass fallback: one CTA per row.
template <typename T, bool kStochastic, int kMode>
__global__ void __launch_bounds__(kQuantThreads) quantize_rowwise_scalar_kernel(
    const T* __restrict__ x, int64_t ldx, int8_t* __restrict__ q, int64_t ldq,
    float* __restrict__ scales, int rows, int cols, int scale_mode, uint64_t seed,
    const float* __restrict__ amax_in) {
  __shared__ float red[kQuantThreads / 32];
  const int row = blockIdx.x;
  const T* xr = x + static_cast<int64_t>(row) * ldx;
  float amax = 0.0f;
  if constexpr (kMode == 2) {
    amax = __ldg(amax_in + row);
  } else {
    for (int c = threadIdx.x; c < cols; c += blockDim.x) amax = fmaxf(amax, fabsf(InTraits<T>::to_f(xr[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = red[0];
    for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  }
  if constexpr (kMode == 1) {
    if (threadIdx.x == 0) scales[row] = amax;
    return;
  }
  const float scale = quant_row_scale<T>(amax, scale_mode);
  if (threadIdx.x == 0) scales[row] = scale;
  const float div = quant_divisor<T>(scale, scale_mode);
  const float recip = __frcp_rn(div);
  const bool fast = scale_mode == kScaleKitchenCuda;
  int8_t* qr = q + static_cast<int64_t>(row) * ldq;
  const int64_t base_idx = static_cast<int64_t>(row) * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    qr[c] = static_cast<int8_t>(
        quant_elem<T, kStochastic>(InTraits<T>::to_f(xr[c]), div, recip, base_idx + c, seed, fast));
  }
}

template <typename T>
int launch_quant(const void* x, int64_t ldx, int8_t* q, int64_t ldq, float* scales, int rows,
                 int cols, int scale_mode, int stochastic, uint64_t seed, int mode,
                 const float* amax_in, cudaStream_t stream) {
  constexpr int kPer = InTraits<T>::kPerVec;
  const bool aligned = (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(q) % 16 == 0) && (cols % kPer == 0) &&
                       ((ldx * static_cast<int64_t>(sizeof(T))) % 16 == 0) && (ldq % 8 == 0);
  const int nvec = cols / kPer;
  // Smallest warps-per-row giving each thread at most 4 vectors, then 8, then
  // 16 (large K); 0 selects the scalar path.
  int wpr = 0, maxv = 0;
  if (aligned) {
    for (int mv : {4, 8, 16}) {
      for (int w : {1, 2, 4, 8}) {
        if (nvec <= w * 32 * mv) {
          wpr = w;
          maxv = mv;
          break;
        }
      }
      if (wpr) break;
    }
  }
  auto go = [&](auto kernel, int rows_per_cta) {
    const int grid = (rows + rows_per_cta - 1) / rows_per_cta;
    kernel<<<grid, kQuantThreads, 0, stream>>>(static_cast<const T*>(x), ldx, q, ldq, scales, rows,
                                               cols, scale_mode, seed, amax_in);
  };
  auto pick = [&](auto stoch, auto mode_c) {
    constexpr bool S = decltype(stoch)::value;
    constexpr int MD = decltype(mode_c)::value;
    auto by_w = [&](auto mv_c) {
      constexpr int MV = decltype(mv_c)::value;
      switch (wpr) {
        case 1: go(quantize_rowwise_vec_kernel<T, 1, MV, S, MD>, 8); break;
        case 2: go(quantize_rowwise_vec_kernel<T, 2, MV, S, MD>, 4); break;
        case 4: go(quantize_rowwise_vec_kernel<T, 4, MV, S, MD>, 2); break;
        default: go(quantize_rowwise_vec_kernel<T, 8, MV, S, MD>, 1); break;
      }
    };
    if (wpr == 0) {
      go(quantize_rowwise_scalar_kernel<T, S, MD>, 1);
    } else if (maxv == 4) {
      by_w(std::integral_constant<int, 4>{});
    } else if (maxv == 8) {
      by_w(std::integral_constant<int, 8>{});
    } else {
      by_w(std::integral_constant<int, 16>{});
    }
  };
  using M0 = std::integral_constant<int, 0>;
  using M1 = std::integral_constant<int, 1>;
  using M2 = std::integral_constant<int, 2>;
  if (mode == 1) {
    pick(std::false_type{}, M1{});
  } else if (mode == 2) {
    pick(std::false_type{}, M2{});
  } else if (stochastic) {
    pick(std::true_type{}, M0{});
  } else {
    pick(std::false_type{}, M0{});
  }
  return 0;
}


// ---- modulation (without ConvRot) + quantiser in the row-in-registers layout
// of quantize_rowwise_vec_kernel: a group of WPR warps owns one row of 16-bit
// values, each thread up to MAXV 16-byte vectors of it.  ACT: 5 x (1 + s),
// 6 rms_norm(x, w) (1 + s), 7 layer_norm(x) (1 + s) + shift, 8 rms_norm(x)
// (1 + s) + shift; the per-element arithmetic and its roundings to T are
// those of the ConvRot kernel's modulation step (the reference's ATen
// sequence, inference/src/backend_eager.rs:176-197 and
// inference/src/backend_bindings.rs:329-405, or with `kitchen` its CUDA
// adaln, KSRC backends/cuda/ops/adaln.cu:103-190); only the order in which
// the row statistics are summed differs.
template <typename T, int WPR, int MAXV, int ACT>
__global__ void __launch_bounds__(kQuantThreads) quantize_modulated_vec_kernel(
    const T* __restrict__ x, int64_t ldx, const T* __restrict__ msc, const T* __restrict__ msh,
    const T* __restrict__ nw, int64_t mgroup, float eps, int8_t* __restrict__ q, int64_t ldq,
    float* __restrict__ scales, int rows, int cols, int kitchen) {
  static_assert(sizeof(T) == 2, "16-bit inputs");
  constexpr int kPer = 8;
  constexpr int kGroupThreads = WPR * 32;
  constexpr int kRowsPerCta = kQuantThreads / kGroupThreads;
  __shared__ float red[kQuantThreads / 32];
  griddep_launch_dependents();  // the GEMM that reads q may start its prologue
  const int group = threadIdx.x / kGroupThreads;
  const int gt = threadIdx.x % kGroupThreads;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int row = blockIdx.x * kRowsPerCta + group;
  const bool live = row < rows;
  const int nvec = cols / kPer;
  // sum (or max) over the row's WPR warps; every thread of the CTA calls it
  auto row_reduce = [&](float v, bool is_max) -> float {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, t) : __fadd_rn(v, t);
    }
    __syncthreads();  // red[] may still be read by the previous reduction
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[group * WPR];
#pragma unroll
    for (int w = 1; w < WPR; ++w) {
      r = is_max ? fmaxf(r, red[group * WPR + w]) : __fadd_rn(r, red[group * WPR + w]);
    }
    return r;
  };
  auto elem = [](const uint4& u, int e) -> float {
    return QuantTraits<T>::to_f(reinterpret_cast<const T*>(&u)[e]);
  };

  const uint4* xrow = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(live ? row : 0) * ldx);
  uint4 v[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = gt + i * kGroupThreads;
    v[i] = make_uint4(0, 0, 0, 0);
    if (live && vi < nvec) v[i] = __ldg(xrow + vi);
  }
  // row statistics
  float mean = 0.0f, rstd = 1.0f;
  if constexpr (ACT != 5) {
    float sum = 0.0f, sumsq = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
#pragma unroll
      for (int e = 0; e < kPer; ++e) {
        const float f = elem(v[i], e);  // zero past the row's end
        if constexpr (ACT == 7) sum = __fadd_rn(sum, f);
        sumsq = __fmaf_rn(f, f, sumsq);
      }
    }
    const float kf = static_cast<float>(cols);
    if constexpr (ACT == 7) {
      const float inv_k = 1.0f / kf;
      mean = row_reduce(sum, false) * inv_k;
      if (kitchen) {
        const float s2 = row_reduce(sumsq, false);
        rstd = rsqrtf(fmaxf(s2 * inv_k - mean * mean, 0.0f) + eps);
      } else {
        float dev = 0.0f;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
          const int vi = gt + i * kGroupThreads;
          if (vi < nvec) {
#pragma unroll
            for (int e = 0; e < kPer; ++e) {
              const float d = __fsub_rn(elem(v[i], e), mean);
              dev = __fmaf_rn(d, d, dev);
            }
          }
        }
        rstd = rsqrtf(row_reduce(dev, false) * inv_k + eps);
      }
    } else {
      rstd = rsqrtf(row_reduce(sumsq, false) / kf + eps);
    }
  }
  // modulated values, rounded to T as the reference materialises them, and
  // their absmax
  const int64_t mrow = (static_cast<int64_t>(live ? row : 0) / mgroup) * cols;
  const uint4* srow = reinterpret_cast<const uint4*>(msc + mrow);
  const uint4* hrow = reinterpret_cast<const uint4*>(msh ? msh + mrow : msc);
  float amax = 0.0f;
  // bf16 rows (all modulations but the kitchen-numerics (rms) AdaLN, whose
  // shift is an FMA): the same per-element operations and roundings as the
  // loop below, two elements per f32x2 instruction and per paired bf16
  // conversion
  constexpr bool kPairedAdaLN = std::is_same<T, __nv_bfloat16>::value;
  const bool paired = kPairedAdaLN && (ACT == 5 || ACT == 6 || !kitchen);
  if constexpr (kPairedAdaLN) {
    if (paired) {
      auto rne2 = [](uint64_t p) -> uint32_t {  // two RN bf16 roundings, packed
        const __nv_bfloat162 b = __floats2bfloat162_rn(lo(p), hi(p));
        return *reinterpret_cast<const uint32_t*>(&b);
      };
      auto unpack2 = [](uint32_t w) -> uint64_t {
        return pk(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
      };
      const uint64_t mean2 = pk(mean, mean), rstd2 = pk(rstd, rstd), one2 = pk(1.0f, 1.0f);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = gt + i * kGroupThreads;
        if (live && vi < nvec) {
          const uint4 sv = __ldg(srow + vi);
          uint4 hv = make_uint4(0, 0, 0, 0), nv = make_uint4(0, 0, 0, 0);
          if constexpr (ACT == 7 || ACT == 8) hv = __ldg(hrow + vi);
          if constexpr (ACT == 6) nv = __ldg(reinterpret_cast<const uint4*>(nw) + vi);
          const uint32_t xw[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
          const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
          const uint32_t nwv[4] = {nv.x, nv.y, nv.z, nv.w};
          uint32_t ow[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t one_s = unpack2(rne2(add2(one2, unpack2(sw[k]))));
            if constexpr (ACT == 5) {
              ow[k] = rne2(mul2(unpack2(xw[k]), one_s));
            } else if constexpr (ACT == 6) {
              const uint64_t nrm =
                  unpack2(rne2(mul2(mul2(unpack2(xw[k]), rstd2), unpack2(nwv[k]))));
              ow[k] = rne2(mul2(nrm, one_s));
            } else {
              const uint64_t nrm = mul2(sub2(unpack2(xw[k]), mean2), rstd2);
              const uint64_t t = unpack2(rne2(mul2(unpack2(rne2(nrm)), one_s)));
              ow[k] = rne2(add2(t, unpack2(hw[k])));
            }
          }
          v[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
          amax = fmaxf(amax, vec_absmax<__nv_bfloat16>(v[i]));
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = gt + i * kGroupThreads;
    if (!paired && live && vi < nvec) {
      const uint4 sv = __ldg(srow + vi);
      uint4 hv = make_uint4(0, 0, 0, 0), wv = make_uint4(0, 0, 0, 0);
      if constexpr (ACT == 7 || ACT == 8) hv = __ldg(hrow + vi);
      if constexpr (ACT == 6) wv = __ldg(reinterpret_cast<const uint4*>(nw) + vi);
      T out[kPer];
#pragma unroll
      for (int e = 0; e < kPer; ++e) {
        const float xv = elem(v[i], e);
        const float one_s = QuantTraits<T>::round_t(__fadd_rn(1.0f, elem(sv, e)));
        float y;
        if constexpr (ACT == 5) {
          y = __fmul_rn(xv, one_s);
        } else if constexpr (ACT == 6) {
          const float nrm = QuantTraits<T>::round_t(__fmul_rn(__fmul_rn(xv, rstd), elem(wv, e)));
          y = __fmul_rn(nrm, one_s);
        } else {
          const float nrm = __fmul_rn(__fsub_rn(xv, mean), rstd);
          if (kitchen) {
            y = __fmaf_rn(nrm, __fadd_rn(1.0f, elem(sv, e)), elem(hv, e));
          } else {
            const float t = QuantTraits<T>::round_t(__fmul_rn(QuantTraits<T>::round_t(nrm), one_s));
            y = __fadd_rn(t, elem(hv, e));
          }
        }
        const float yt = QuantTraits<T>::round_t(y);
        amax = fmaxf(amax, fabsf(yt));
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          out[e] = __float2bfloat16_rn(yt);  // exact: yt is a bf16 value
        } else {
          out[e] = __float2half_rn(yt);
        }
      }
      v[i] = *reinterpret_cast<const uint4*>(out);
    }
  }
  amax = row_reduce(amax, true);
  if (!live) return;
  const float scale = quant_row_scale<T>(kitchen ? amax : QuantTraits<T>::round_t(amax), kitchen);
  if (gt == 0) scales[row] = scale;
  const float div = quant_divisor<T>(scale, kitchen);
  const float recip = __frcp_rn(div);
  int8_t* qrow = q + static_cast<int64_t>(row) * ldq;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = gt + i * kGroupThreads;
    if (vi >= nvec) continue;
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      reinterpret_cast<uint2*>(qrow)[vi] = quant8_bf16(v[i], div, recip);
    } else {
      uint32_t packed[2];
#pragma unroll
      for (int w = 0; w < 2; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int qv = quant_code<T>(elem(v[i], w * 4 + j), div, recip, kitchen == kScaleKitchenCuda);
          word |= (static_cast<uint32_t>(qv) & 0xFFu) << (8 * j);
        }
        packed[w] = word;
      }
      reinterpret_cast<uint2*>(qrow)[vi] = make_uint2(packed[0], packed[1]);
    }
  }
}

// Row-loop form of the bf16 modulated quantiser for the modulations whose
// per-element arithmetic runs on packed pairs (5, 6, and 7 / 8 with eager
// numerics).  A CTA is one row group of WPR warps; it walks rows blockIdx.x,
// blockIdx.x + gridDim.x, ..., so a thread always owns the same columns: the
// bf16 values 1 + s, the shift and the norm weight of those columns are kept
// in registers (formed again only when a row of another sample comes) instead
// of being loaded and formed once per row, and the next row's x is loaded
// while the current one is worked.  The row statistics are summed on packed
// fp32 pairs.  Per element the operations and their roundings to bf16 are
// those of quantize_modulated_vec_kernel's paired path (bit-identical for
// modulation 5; for the others only the order in which the row statistics
// are summed differs).  Every CTA runs `iters` iterations, rows past the end
// masked, so its barriers match up.
template <int WPR, int MAXV, int ACT>
__global__ void __launch_bounds__(WPR * 32) quantize_modulated_rows_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ msc,
    const __nv_bfloat16* __restrict__ msh, const __nv_bfloat16* __restrict__ nw, int64_t mgroup,
    float eps, int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scales, int rows, int cols,
    int kitchen, int iters) {
  static_assert(ACT >= 5 && ACT <= 8, "modulations 5-8");
  constexpr int kThreads = WPR * 32;
  __shared__ float red[2][WPR];
  griddep_launch_dependents();  // the GEMM that reads q may start its prologue
  const int gt = threadIdx.x;
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int nvec = cols / 8;
  int phase = 0;
  // sum or max over the CTA; red[] alternates between two halves, so one
  // barrier per reduction suffices (a half is rewritten only after the next
  // reduction's barrier, which every reader of it has passed)
  auto reduce = [&](float v, bool is_max) -> float {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float t = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, t) : __fadd_rn(v, t);
    }
    if constexpr (WPR == 1) {
      return v;
    } else {
      if (lane == 0) red[phase][warp] = v;
      __syncthreads();
      float r = red[phase][0];
#pragma unroll
      for (int w = 1; w < WPR; ++w) r = is_max ? fmaxf(r, red[phase][w]) : __fadd_rn(r, red[phase][w]);
      phase ^= 1;
      return r;
    }
  };
  auto unpack2 = [](uint32_t w) -> uint64_t {
    return pk(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  };
  auto rne2 = [](uint64_t p) -> uint32_t {  // two RN bf16 roundings, packed
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo(p), hi(p));
    return *reinterpret_cast<const uint32_t*>(&b);
  };
  auto words = [](const uint4& u, int k) -> uint32_t {
    return k == 0 ? u.x : k == 1 ? u.y : k == 2 ? u.z : u.w;
  };

  // per-column constants as bf16 words: 1 + s (rounded), the shift, the norm weight
  uint32_t one_s[MAXV][4], shw[MAXV][4], nww[MAXV][4];
  if constexpr (ACT == 6) {
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = gt + i * kThreads;
      const uint4 wv = vi < nvec ? __ldg(reinterpret_cast<const uint4*>(nw) + vi) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int k = 0; k < 4; ++k) nww[i][k] = words(wv, k);
    }
  }
  int64_t cur_sample = -1;

  int row = static_cast<int>(blockIdx.x);
  const int stride = static_cast<int>(gridDim.x);
  uint4 nx[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = gt + i * kThreads;
    nx[i] = make_uint4(0, 0, 0, 0);
    if (row < rows && vi < nvec) nx[i] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ldx) + vi);
  }
  const float kf = static_cast<float>(cols);
  const float inv_k = 1.0f / kf;
  for (int it = 0; it < iters; ++it, row += stride) {
    const bool live = row < rows;
    uint64_t p[MAXV][4];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) p[i][k] = unpack2(words(nx[i], k));
    }
    // the next row's x while this one is worked
    const int nrow = row + stride;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = gt + i * kThreads;
      if (nrow < rows && vi < nvec) {
        nx[i] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(nrow) * ldx) + vi);
      }
    }
    // this row's sample constants (uniform over the CTA)
    if (live) {
      const int64_t smp = row / mgroup;
      if (smp != cur_sample) {
        cur_sample = smp;
        const int64_t mrow = smp * cols;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
          const int vi = gt + i * kThreads;
          uint4 sv = make_uint4(0, 0, 0, 0), hv = make_uint4(0, 0, 0, 0);
          if (vi < nvec) {
            sv = __ldg(reinterpret_cast<const uint4*>(msc + mrow) + vi);
            if constexpr (ACT == 7 || ACT == 8) hv = __ldg(reinterpret_cast<const uint4*>(msh + mrow) + vi);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            one_s[i][k] = rne2(add2(pk(1.0f, 1.0f), unpack2(words(sv, k))));
            if constexpr (ACT == 7 || ACT == 8) shw[i][k] = words(hv, k);
          }
        }
      }
    }
    // row statistics (columns past the row's end hold zeros and are skipped
    // where a zero would count)
    float mean = 0.0f, rstd = 1.0f;
    if constexpr (ACT == 7) {
      uint64_t s2 = pk(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
#pragma unroll
        for (int k = 0; k < 4; ++k) s2 = add2(s2, p[i][k]);
      }
      mean = reduce(__fadd_rn(lo(s2), hi(s2)), false) * inv_k;
      const uint64_t mean2 = pk(mean, mean);
      uint64_t d2 = pk(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = gt + i * kThreads;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          p[i][k] = sub2(p[i][k], mean2);  // x - mean, kept for the modulation
          if (vi < nvec) d2 = fma2(p[i][k], p[i][k], d2);
        }
      }
      rstd = rsqrtf(reduce(__fadd_rn(lo(d2), hi(d2)), false) * inv_k + eps);
    } else if constexpr (ACT == 6 || ACT == 8) {
      uint64_t q2 = pk(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
#pragma unroll
        for (int k = 0; k < 4; ++k) q2 = fma2(p[i][k], p[i][k], q2);
      }
      rstd = rsqrtf(reduce(__fadd_rn(lo(q2), hi(q2)), false) / kf + eps);
    }
    // modulated row (bf16 words) and its absmax, as bf16 bit patterns (for
    // non-negative values the integer order is the value order)
    const uint64_t rstd2 = pk(rstd, rstd);
    uint4 ov[MAXV];
    uint32_t amax_bits = 0;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      uint32_t ow[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint64_t os = unpack2(one_s[i][k]);
        if constexpr (ACT == 5) {
          ow[k] = rne2(mul2(p[i][k], os));
        } else if constexpr (ACT == 6) {
          const uint64_t nrm = unpack2(rne2(mul2(mul2(p[i][k], rstd2), unpack2(nww[i][k]))));
          ow[k] = rne2(mul2(nrm, os));
        } else {
          // 7: p holds x - mean; 8: mean is 0 and x - 0 is x
          const uint64_t t = unpack2(rne2(mul2(unpack2(rne2(mul2(p[i][k], rstd2))), os)));
          ow[k] = rne2(add2(t, unpack2(shw[i][k])));
        }
        amax_bits = __vmaxu2(amax_bits, ow[k] & 0x7FFF7FFFu);
      }
      ov[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    const uint32_t mb = max(amax_bits & 0xFFFFu, amax_bits >> 16);
    const float amax = reduce(__uint_as_float(mb << 16), true);
    if (!live) continue;
    const float scale = quant_row_scale<__nv_bfloat16>(amax, kitchen);
    if (gt == 0) scales[row] = scale;
    const float div = quant_divisor<__nv_bfloat16>(scale, kitchen);
    const float recip = __frcp_rn(div);
    int8_t* qrow = q + static_cast<int64_t>(row) * ldq;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = gt + i * kThreads;
      if (vi < nvec) reinterpret_cast<uint2*>(qrow)[vi] = quant8_bf16(ov[i], div, recip);
    }
  }
}

template <int WPR, int MAXV, int ACT>
int launch_modulated_rows(const void* x, int64_t ldx, const void* msc, const void* msh,
                          const void* nw, int64_t mgroup, float eps, int8_t* q, int64_t ldq,
                          float* scales, int rows, int cols, int kitchen, cudaStream_t stream) {
  auto kern = quantize_modulated_rows_kernel<WPR, MAXV, ACT>;
  static int per_sm = 0;  // resident CTAs per SM of this instantiation
  static int sms = 0;
  if (per_sm == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, WPR * 32, 0) != cudaSuccess ||
        per_sm < 1) {
      per_sm = 1;
      sms = sms > 0 ? sms : 1;
    }
  }
  const int grid = std::max(1, std::min(rows, per_sm * sms));
  const int iters = (rows + grid - 1) / grid;
  kern<<<grid, WPR * 32, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(msc),
      static_cast<const __nv_bfloat16*>(msh), static_cast<const __nv_bfloat16*>(nw), mgroup, eps, q,
      ldq, scales, rows, cols, kitchen, iters);
  return 0;
}

template <typename T, int ACT>
int launch_modulated_t(const void* x, int64_t ldx, const void* msc, const void* msh,
                       const void* nw, int64_t mgroup, float eps, int8_t* q, int64_t ldq,
                       float* scales, int rows, int cols, int kitchen, cudaStream_t stream) {
  const int nvec = cols / 8;
  int wpr = 0;
  for (int w : {1, 2, 4, 8}) {
    if (nvec <= w * 32 * 4) {
      wpr = w;
      break;
    }
  }
  if (!wpr) return -1;  // more than 8192 columns: the ConvRot-layout kernel
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (ACT == 5 || ACT == 6 || !kitchen) {
      int rc;
      if (wpr == 4 && nvec <= 4 * 32 * 3) {
        rc = launch_modulated_rows<4, 3, ACT>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream);
      } else {
        switch (wpr) {
          case 1: rc = launch_modulated_rows<1, 4, ACT>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream); break;
          case 2: rc = launch_modulated_rows<2, 4, ACT>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream); break;
          case 4: rc = launch_modulated_rows<4, 4, ACT>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream); break;
          default: rc = launch_modulated_rows<8, 4, ACT>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream); break;
        }
      }
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) {
        set_error("modulated quantiser launch failed: %s", cudaGetErrorString(e));
        return W8A8_ERR_ACCELERATOR;
      }
      return rc;
    }
  }
  auto go = [&](auto kernel, int rows_per_cta) {
    kernel<<<(rows + rows_per_cta - 1) / rows_per_cta, kQuantThreads, 0, stream>>>(
        static_cast<const T*>(x), ldx, static_cast<const T*>(msc), static_cast<const T*>(msh),
        static_cast<const T*>(nw), mgroup, eps, q, ldq, scales, rows, cols, kitchen);
  };
  switch (wpr) {
    case 1: go(quantize_modulated_vec_kernel<T, 1, 4, ACT>, 8); break;
    case 2: go(quantize_modulated_vec_kernel<T, 2, 4, ACT>, 4); break;
    case 4: go(quantize_modulated_vec_kernel<T, 4, 4, ACT>, 2); break;
    default: go(quantize_modulated_vec_kernel<T, 8, 4, ACT>, 1); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("modulated quantiser launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

template <typename T>
int launch_modulated(int act, const void* x, int64_t ldx, const void* msc, const void* msh,
                     const void* nw, int64_t mgroup, float eps, int8_t* q, int64_t ldq,
                     float* scales, int rows, int cols, int kitchen, cudaStream_t stream) {
  switch (act) {
    case 5: return launch_modulated_t<T, 5>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream);
    case 6: return launch_modulated_t<T, 6>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream);
    case 7: return launch_modulated_t<T, 7>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream);
    case 8: return launch_modulated_t<T, 8>(x, ldx, msc, msh, nw, mgroup, eps, q, ldq, scales, rows, cols, kitchen, stream);
    default: return -1;
  }
}

}  // namespace

int quantize_modulated_vec_launch(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                  int64_t ldx, int act, const void* norm_w, float eps,
                                  const void* mod_scale, const void* mod_shift, int64_t mod_group,
                                  int8_t* q, int64_t ldq, float* scales, int scale_mode,
                                  cudaStream_t stream) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if ((x_dtype != W8A8_BF16 && x_dtype != W8A8_F16) || cols % 8 || ldx % 8 || ldq % 8 ||
      rows > 0x7fffffffLL || !a16(x) || !a16(q) || !a16(mod_scale) ||
      (mod_shift && !a16(mod_shift)) || (norm_w && !a16(norm_w))) {
    return -1;
  }
  const int km = scale_mode;  // nonzero: kitchen scales (W8A8_SCALE_*)
  const int64_t g = mod_group > 0 ? mod_group : 1;
  if (x_dtype == W8A8_BF16) {
    return launch_modulated<__nv_bfloat16>(act, x, ldx, mod_scale, mod_shift, norm_w, g, eps, q, ldq,
                                           scales, static_cast<int>(rows), static_cast<int>(cols),
                                           km, stream);
  }
  return launch_modulated<__half>(act, x, ldx, mod_scale, mod_shift, norm_w, g, eps, q, ldq, scales,
                                  static_cast<int>(rows), static_cast<int>(cols), km, stream);
}

namespace {
}  // namespace

int quantize_rowwise_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                            int8_t* q, int64_t ldq, float* scales, int scale_mode, int stochastic,
                            uint64_t seed, int mode, const float* amax_in, cudaStream_t stream) {
  switch (x_dtype) {
    case W8A8_BF16:
      return launch_quant<__nv_bfloat16>(x, ldx, q, ldq, scales, (int)rows, (int)cols, scale_mode,
                                         stochastic, seed, mode, amax_in, stream);
    case W8A8_F16:
      return launch_quant<__half>(x, ldx, q, ldq, scales, (int)rows, (int)cols, scale_mode,
                                  stochastic, seed, mode, amax_in, stream);
    case W8A8_F32:
      return launch_quant<float>(x, ldx, q, ldq, scales, (int)rows, (int)cols, scale_mode,
                                 stochastic, seed, mode, amax_in, stream);
    default:
      return -1;
  }
}

}  // namespace w8a8
