// Fused input-activation + ConvRot (256-point Hadamard) + row-wise INT8
// quantiser.
//
// Replaces the reference's quantize_int8_rowwise_convrot64 kernel
// (native/comfy-port/kitchen/int8_linear.cu:1197-1314, launched from
// inference/src/convrot.rs:156-209 when cuda_linear.rs:400-417 says the input
// activation fuses) and, with ROT = false, the reference's "activation in ATen,
// then quantise" sequence for an input activation without ConvRot
// (inference/src/int8_linear.rs:37-97 followed by the row quantiser).
//
// Numerics with ROT and kitchen scales (the reference's fused kernel):
//   v   = act(x) in fp32 (GELU-tanh, SwiGLU = silu(gate) * up, RMSNorm =
//         x * rsqrt(mean(x^2) + eps) * w, or SiTU), no rounding
//   v   = H_256 v per 256-group: four radix-4 stages (digit strides 1, 4, 16,
//         64), each output 0.5 * (a +- b +- c +- d) summed left to right with
//         one operand negated (int8_linear.cu:253-261, 881-934)
//   s   = max(min(amax_fp32, finite_max(T)) * (1/127), 1e-30)     (kitchen)
//         max(T(amax_fp32) / 127, 1e-30)                          (eager)
//   q   = clamp(rne(T(T(v) / T(s))), -128, 127)      (int8_linear.cu:53-57)
// With eager scales, and always without ROT, the activation output is rounded
// to T after each op the reference's ATen sequence rounds after (its eager
// route: ATen activation, T-typed Hadamard matmul, row quantiser); the
// rotation itself is the same fp32 butterfly.
//
// Layout: one CTA per row; a team of 16 threads owns two 256-groups of the
// row at a time, each thread element 16 r + j (j < 16) of both, held as
// packed fp32 pairs so every f32x2 add / mul serves the two groups.  Stages 1
// and 4 of the transform run in registers; the team transposes the pairs
// through an XOR-swizzled (bank-conflict-free) shared buffer to element
// r + 16 j for stages 16 and 64.  Codes go back through shared memory as
// bytes so every thread stores 16 contiguous bytes per group.  A thread keeps
// up to two group pairs in registers (K <= 16 teams x 4 x 256), so x is read
// from HBM exactly once.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "quant_common.cuh"
#include "sm100_ptx.cuh"
#include "w8a8_internal.h"

namespace w8a8 {
namespace {

constexpr int kGroup = 256;
constexpr int kTeam = 16;          // threads per group
constexpr int kMaxTeams = 16;      // 256 threads per CTA

// 0-4: the reference's input activations (input_act_codes.h, plus SiTU);
// 5-8: modulations applied before the linear (W8A8_MOD_* + 5).
enum InputAct : int {
  kInNone = 0,
  kInGeluTanh = 1,
  kInSwiGLU = 2,
  kInRmsNorm = 3,
  kInSiTU = 4,
  kInModScale = 5,     // x * (1 + s)
  kInRmsModScale = 6,  // rms_norm(x, w) * (1 + s)
  kInAdaLN = 7,        // layer_norm(x) * (1 + s) + shift
  kInRmsAdaLN = 8,     // rms_norm(x) * (1 + s) + shift
};

// Modulation rows: scale / shift [rows / group, K] in the input dtype; x row
// i takes modulation row i / group.
struct ModArgs {
  const void* scale;
  const void* shift;
  int64_t group;
};

template <typename T>
struct Ld;
template <>
struct Ld<__nv_bfloat16> {
  static __device__ __forceinline__ float at(const void* p, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
  // 16 consecutive elements from a 16-byte aligned address
  static __device__ __forceinline__ void vec16(const void* p, int64_t i, float* f) {
    const uint4* s = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p) + i);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 v = __ldg(s + h);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        f[8 * h + 2 * t] = __uint_as_float(w[t] << 16);
        f[8 * h + 2 * t + 1] = __uint_as_float(w[t] & 0xFFFF0000u);
      }
    }
  }
  static constexpr int kAlign = 8;  // elements per 16 bytes
};
template <>
struct Ld<__half> {
  static __device__ __forceinline__ float at(const void* p, int64_t i) {
    return __half2float(static_cast<const __half*>(p)[i]);
  }
  static __device__ __forceinline__ void vec16(const void* p, int64_t i, float* f) {
    const uint4* s = reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + i);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 v = __ldg(s + h);
      const __half2* hh = reinterpret_cast<const __half2*>(&v);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 g = __half22float2(hh[t]);
        f[8 * h + 2 * t] = g.x;
        f[8 * h + 2 * t + 1] = g.y;
      }
    }
  }
  static constexpr int kAlign = 8;
};
template <>
struct Ld<float> {
  static __device__ __forceinline__ float at(const void* p, int64_t i) {
    return static_cast<const float*>(p)[i];
  }
  static __device__ __forceinline__ void vec16(const void* p, int64_t i, float* f) {
    const float4* s = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float4 v = __ldg(s + h);
      f[4 * h] = v.x;
      f[4 * h + 1] = v.y;
      f[4 * h + 2] = v.z;
      f[4 * h + 3] = v.w;
    }
  }
  static constexpr int kAlign = 4;
};

template <typename T>
__device__ __forceinline__ void load16(const void* p, int64_t i, bool vec, float* f) {
  if (vec) {
    Ld<T>::vec16(p, i, f);
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) f[j] = Ld<T>::at(p, i + j);
  }
}

// Round to T when the ATen sequence would (round), otherwise keep fp32.
template <typename T>
__device__ __forceinline__ float rt(float v, bool round) {
  return round ? QuantTraits<T>::round_t(v) : v;
}

// GELU-tanh: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
// (torch.nn.functional.gelu(approximate="tanh"); int8_linear.cu:1175-1185).
__device__ __forceinline__ float in_gelu_tanh(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

// silu(g) = g / (1 + exp(-g))  (int8_linear.cu:1196-1200)
__device__ __forceinline__ float in_silu(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ float in_sigmoid(float g) { return 1.0f / (1.0f + expf(-g)); }

// The same activations as the reference's Kitchen CUDA kernels compute them
// as built (--use_fast_math, native/comfy-port/CMakeLists.txt:30-36): there
// tanhf is tanh.approx.f32, expf is __expf and a divide is __fdividef (the
// intrinsic forms give bit-identical outputs to that build's).  Used with the
// W8A8_SCALE_KITCHEN_CUDA numerics on the rotated route.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float in_gelu_tanh_fast(float v) {
  const float inner = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanh_fast(inner));
}

__device__ __forceinline__ float in_silu_fast(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ float in_sigmoid_fast(float g) {
  return __fdividef(1.0f, 1.0f + __expf(-g));
}

// Sum of squares of a K-wide row in the order the reference's fused kernel
// forms it (int8_linear.cu:1239-1248 with block_reduce_sum_f32_t, :141-158):
// B threads (its block size for this launch, chosen from the row count and K
// at :1668-1673) each accumulate v*v with FMA over columns t, t + B, ...; a
// shuffle-down tree (offsets 16 .. 1) within each warp; the same tree over
// the warp totals, zero-padded to 32.  This CTA's threads emulate the B
// partial sums in `part` (1024 + 33 floats: the partials, the warp totals
// and the result) and the trees in registers.
template <typename T>
__device__ float sumsq_reference_order(const void* x, int64_t xrow, int K, int rows, float* part) {
  const int B = rows == 1 ? 512
              : K == 256 ? 64
              : K <= 3072 ? 128
              : K <= 6144 ? 256
              : K < 12288 ? 512
              : 1024;
  for (int t = threadIdx.x; t < B; t += blockDim.x) {
    float acc = 0.0f;
    for (int c = t; c < K; c += B) {
      const float v = Ld<T>::at(x, xrow + c);
      acc = __fmaf_rn(v, v, acc);
    }
    part[t] = acc;
  }
  __syncthreads();
  auto tree32 = [](float* a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int i = 0; i < o; ++i) a[i] = __fadd_rn(a[i], a[i + o]);
    }
    return a[0];
  };
  const int warps = B / 32;
  float w[32];
  if (static_cast<int>(threadIdx.x) < warps) {
    for (int i = 0; i < 32; ++i) w[i] = part[32 * threadIdx.x + i];
    part[1024 + threadIdx.x] = tree32(w);  // warp totals after the B partials
  }
  __syncthreads();
  float result = 0.0f;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 32; ++i) w[i] = i < warps ? part[1024 + i] : 0.0f;
    result = tree32(w);
    part[1024 + 32] = result;
  }
  __syncthreads();
  result = part[1024 + 32];
  __syncthreads();
  return result;
}

// Packed pairs (pk / lo / hi / add2 / sub2 / mul2 / fma2, quant_common.cuh):
// element j of two 256-groups of the row in one 64-bit register pair, so
// every f32x2 instruction serves both groups.

// One radix-4 butterfly of the normalised H4 (rows ++ +-, ++-+, +-++, -+++),
// every sum left to right exactly as int8_linear.cu:253-261 orders it;
// (-a) + b is computed as b - a, which rounds identically.  Packed: two
// independent butterflies per call.
__device__ __forceinline__ void h4x2(uint64_t& a, uint64_t& b, uint64_t& c, uint64_t& d) {
  const uint64_t half = pk(0.5f, 0.5f);
  const uint64_t ab = add2(a, b);
  const uint64_t amb = sub2(a, b);
  const uint64_t bma = sub2(b, a);
  const uint64_t y0 = sub2(add2(ab, c), d);
  const uint64_t y1 = add2(sub2(ab, c), d);
  const uint64_t y2 = add2(add2(amb, c), d);
  const uint64_t y3 = add2(add2(bma, c), d);
  a = mul2(half, y0);
  b = mul2(half, y1);
  c = mul2(half, y2);
  d = mul2(half, y3);
}

// Codes of a pair of values (their low bytes are the int8 codes, two's
// complement): clamp(rne(T(T(v) / div)), -128, 127).
template <typename T>
__device__ __forceinline__ void quant_pair(uint64_t p, float div, float recip, uint32_t& c0,
                                           uint32_t& c1, bool fast) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    // paired RN conversions; bf16(x / d) from the product x RN(1/d), which
    // rounds to the same bf16 for bf16 x and d (proof at quant8_bf16); rne by
    // adding 1.5 * 2^23
    (void)div;
    uint32_t b;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b) : "f"(hi(p)), "f"(lo(p)));
    const uint64_t xv = pk(__uint_as_float(b << 16), __uint_as_float(b & 0xFFFF0000u));
    const uint64_t y = mul2(xv, pk(recip, recip));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(b) : "f"(hi(y)), "f"(lo(y)));
    // |quotient| <= 127.75, so only the upper end needs a clamp (-127.75
    // rounds to -128)
    const float q0 = fminf(__uint_as_float(b << 16), 127.0f);
    const float q1 = fminf(__uint_as_float(b & 0xFFFF0000u), 127.0f);
    const uint64_t t = add2(pk(q0, q1), pk(12582912.0f, 12582912.0f));
    c0 = __float_as_uint(lo(t));
    c1 = __float_as_uint(hi(t));
  } else {
    c0 = static_cast<uint32_t>(quant_code<T>(QuantTraits<T>::round_t(lo(p)), div, recip, fast));
    c1 = static_cast<uint32_t>(quant_code<T>(QuantTraits<T>::round_t(hi(p)), div, recip, fast));
  }
}

template <int NW>
__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, t) : __fadd_rn(v, t);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) {
    if (w * 32 < static_cast<int>(blockDim.x)) r = is_max ? fmaxf(r, red[w]) : __fadd_rn(r, red[w]);
  }
  return r;
}

// Shared memory of one team: the FHT transpose buffer (16 threads x 16
// packed pairs, 128 B per thread, chunks XOR-swizzled) and the code bytes of
// its two groups (272 B each: teams of one warp land on different banks).
constexpr int kTransBytes = kTeam * 16 * 8;
constexpr int kCodeStride = kGroup + 16;
constexpr int kTeamBytes = kTransBytes + 2 * kCodeStride;
static_assert(kTeamBytes % 16 == 0, "team buffers must keep 16-byte alignment");

// PPT: group pairs per team kept in registers.  Team t owns group pairs
// (2 (t + i teams), 2 (t + i teams) + 1), i < PPT.
template <typename T, int ACT, bool ROT, int PPT>
__device__ __forceinline__ void act_rot_row(
    const void* __restrict__ x, int64_t ldx, const void* __restrict__ act_w, float act_eps,
    ModArgs mod, int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scales, int K,
    int kitchen_mode, int vec_in, int vec_out) {
  extern __shared__ __align__(16) uint8_t dsm[];
  __shared__ float red[8];
  griddep_launch_dependents();  // the GEMM that reads q may start its prologue
  const int row = blockIdx.x;
  const int team = threadIdx.x / kTeam;
  const int r = threadIdx.x % kTeam;
  const int teams = blockDim.x / kTeam;
  const int G = K / kGroup;
  const int64_t xrow = static_cast<int64_t>(row) * ldx;
  uint8_t* tbuf = dsm + team * kTeamBytes;
  uint8_t* cbuf = tbuf + kTransBytes;
  // The activation is T-rounded at each step the ATen sequence rounds, except
  // for the kitchen numerics of the fused ConvRot kernel (fp32 throughout).
  const bool kRound = !ROT || !kitchen_mode;
  // the Kitchen CUDA build's fast-math activations (rotated route only; the
  // unrotated route stands for ATen operators, which are not built that way)
  const bool fast_act = ROT && kitchen_mode == kScaleKitchenCuda;

  // v[i][h][j]: element 16 r + j of group 2 (team + i teams) + h
  float v[PPT][2][16];
  float sumsq = 0.0f, sum = 0.0f;
  // ---- load (+ elementwise activation)
#pragma unroll
  for (int i = 0; i < PPT; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int g = 2 * (team + i * teams) + h;
      const int col = g * kGroup + kTeam * r;
      float* f = v[i][h];
      if (g < G) {
        if constexpr (ACT == kInSwiGLU || ACT == kInSiTU) {
          float gate[16], up[16];
          load16<T>(x, xrow + col, vec_in, gate);
          load16<T>(x, xrow + K + col, vec_in, up);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if constexpr (ACT == kInSwiGLU) {
              const float sg = fast_act ? in_silu_fast(gate[j]) : in_silu(gate[j]);
              f[j] = rt<T>(rt<T>(sg, kRound) * up[j], kRound);
            } else if (fast_act) {
              // SiTU in the fast-math forms
              const float a = 25.0f * tanh_fast(__fdividef(gate[j], 25.0f));
              const float t4 = 4.0f * tanh_fast(__fdividef(up[j], 4.0f));
              f[j] = a * (t4 * in_sigmoid_fast(up[j]));
            } else {
              // 25 tanh(a / 25) * (4 tanh(b / 4) * sigmoid(b))
              // (inference/src/int8_linear.rs:54-74)
              const float a =
                  rt<T>(25.0f * rt<T>(tanhf(rt<T>(gate[j] / 25.0f, kRound)), kRound), kRound);
              const float t4 =
                  rt<T>(4.0f * rt<T>(tanhf(rt<T>(up[j] / 4.0f, kRound)), kRound), kRound);
              const float gated = rt<T>(t4 * rt<T>(in_sigmoid(up[j]), kRound), kRound);
              f[j] = rt<T>(a * gated, kRound);
            }
          }
        } else {
          load16<T>(x, xrow + col, vec_in, f);
          if constexpr (ACT == kInGeluTanh) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              f[j] = fast_act ? in_gelu_tanh_fast(f[j]) : rt<T>(in_gelu_tanh(f[j]), kRound);
            }
          } else if constexpr (ACT == kInRmsNorm || ACT == kInRmsModScale || ACT == kInRmsAdaLN) {
#pragma unroll
            for (int j = 0; j < 16; ++j) sumsq = __fmaf_rn(f[j], f[j], sumsq);
          } else if constexpr (ACT == kInAdaLN) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              sum = __fadd_rn(sum, f[j]);
              sumsq = __fmaf_rn(f[j], f[j], sumsq);
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] = 0.0f;
      }
    }
  }
  if constexpr (ACT == kInRmsNorm) {
    // x * rsqrt(mean(x^2) + eps) * w  (int8_linear.cu:1239-1267; ATen's
    // rms_norm forms the same fp32 product and rounds it to T once)
    float rstd;
    if constexpr (ROT) {
      if (fast_act) {
        // the reference kernel's summation order and fast-math divide
        __shared__ float part[1024 + 64];
        const float ss = sumsq_reference_order<T>(x, xrow, K, static_cast<int>(gridDim.x), part);
        rstd = rsqrtf(__fdividef(ss, static_cast<float>(K)) + act_eps);
      } else {
        rstd = rsqrtf(block_reduce<8>(sumsq, false, red) / static_cast<float>(K) + act_eps);
      }
    } else {
      rstd = rsqrtf(block_reduce<8>(sumsq, false, red) / static_cast<float>(K) + act_eps);
    }
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int g = 2 * (team + i * teams) + h;
        if (g < G) {
          float w[16];
          load16<T>(act_w, g * kGroup + kTeam * r, vec_in, w);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[i][h][j] = rt<T>(__fmul_rn(__fmul_rn(v[i][h][j], rstd), w[j]), kRound);
          }
        }
      }
    }
  }
  if constexpr (ACT >= kInModScale) {
    // Modulation (the reference materialises its output in T, so the value
    // is always rounded to T before quantising).
    //   kitchen: the reference's CUDA adaln (KSRC backends/cuda/ops/adaln.cu:
    //            103-190): one-pass mean / E[x^2] - mean^2 statistics,
    //            (x - mean) * rstd * (1 + s) + shift in fp32, one rounding;
    //   eager:   its ATen sequence (inference/src/backend_eager.rs:176-197,
    //            inference/src/backend_bindings.rs:329-405): the normalised row
    //            rounded to T, times T(1 + s) rounded, plus shift rounded.
    float mean = 0.0f, rstd = 1.0f;
    if constexpr (ACT == kInRmsModScale || ACT == kInRmsAdaLN) {
      const float ss = block_reduce<8>(sumsq, false, red);
      rstd = rsqrtf(ss / static_cast<float>(K) + act_eps);
    } else if constexpr (ACT == kInAdaLN) {
      const float inv_k = 1.0f / static_cast<float>(K);
      const float s1 = block_reduce<8>(sum, false, red);
      mean = s1 * inv_k;
      if (kitchen_mode) {
        const float s2 = block_reduce<8>(sumsq, false, red);
        rstd = rsqrtf(fmaxf(s2 * inv_k - mean * mean, 0.0f) + act_eps);
      } else {
        // second pass over the registers: sum of squared deviations
        float dev = 0.0f;
#pragma unroll
        for (int i = 0; i < PPT; ++i) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (2 * (team + i * teams) + h < G) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float d = __fsub_rn(v[i][h][j], mean);
                dev = __fmaf_rn(d, d, dev);
              }
            }
          }
        }
        const float s2 = block_reduce<8>(dev, false, red);
        rstd = rsqrtf(s2 * inv_k + act_eps);
      }
    }
    const int64_t mrow = (static_cast<int64_t>(row) / mod.group) * K;
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int g = 2 * (team + i * teams) + h;
        if (g < G) {
          const int col = g * kGroup + kTeam * r;
          float sc[16], sh[16], w[16];
          load16<T>(mod.scale, mrow + col, vec_in, sc);
          if constexpr (ACT == kInAdaLN || ACT == kInRmsAdaLN) load16<T>(mod.shift, mrow + col, vec_in, sh);
          if constexpr (ACT == kInRmsModScale) load16<T>(act_w, col, vec_in, w);
          if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            if (ACT == kInModScale || ACT == kInRmsModScale || !kitchen_mode) {
              // bf16: the same operations and roundings as the scalar loop
              // below, two elements per f32x2 instruction and per paired
              // bf16 conversion
              auto rne2 = [](uint64_t p) -> uint64_t {
                const __nv_bfloat162 b = __floats2bfloat162_rn(lo(p), hi(p));
                const uint32_t w = *reinterpret_cast<const uint32_t*>(&b);
                return pk(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
              };
              const uint64_t one2 = pk(1.0f, 1.0f), mean2 = pk(mean, mean), rstd2 = pk(rstd, rstd);
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                const uint64_t xp = pk(v[i][h][j], v[i][h][j + 1]);
                const uint64_t one_s = rne2(add2(one2, pk(sc[j], sc[j + 1])));
                uint64_t y;
                if constexpr (ACT == kInModScale) {
                  y = mul2(xp, one_s);
                } else if constexpr (ACT == kInRmsModScale) {
                  y = mul2(rne2(mul2(mul2(xp, rstd2), pk(w[j], w[j + 1]))), one_s);
                } else {
                  const uint64_t nrm = mul2(sub2(xp, mean2), rstd2);
                  y = add2(rne2(mul2(rne2(nrm), one_s)), pk(sh[j], sh[j + 1]));
                }
                y = rne2(y);
                v[i][h][j] = lo(y);
                v[i][h][j + 1] = hi(y);
              }
              continue;
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float xv = v[i][h][j];
            float y;
            if constexpr (ACT == kInModScale) {
              y = __fmul_rn(xv, QuantTraits<T>::round_t(__fadd_rn(1.0f, sc[j])));
            } else if constexpr (ACT == kInRmsModScale) {
              const float nrm = QuantTraits<T>::round_t(__fmul_rn(__fmul_rn(xv, rstd), w[j]));
              y = __fmul_rn(nrm, QuantTraits<T>::round_t(__fadd_rn(1.0f, sc[j])));
            } else {
              const float nrm = __fmul_rn(__fsub_rn(xv, mean), rstd);
              if (kitchen_mode) {
                y = __fmaf_rn(nrm, __fadd_rn(1.0f, sc[j]), sh[j]);
              } else {
                const float t = QuantTraits<T>::round_t(__fmul_rn(
                    QuantTraits<T>::round_t(nrm), QuantTraits<T>::round_t(__fadd_rn(1.0f, sc[j]))));
                y = __fadd_rn(t, sh[j]);
              }
            }
            v[i][h][j] = QuantTraits<T>::round_t(y);
          }
        }
      }
    }
  }

  // ---- Hadamard transform per 256-group (both groups of a pair at once)
  if constexpr (ROT) {
#pragma unroll
    for (int i = 0; i < PPT; ++i) {
      uint64_t P[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) P[j] = pk(v[i][0][j], v[i][1][j]);
      // strides 1 and 4 on e = 16 r + j, j = d0 + 4 d1
#pragma unroll
      for (int d1 = 0; d1 < 4; ++d1) h4x2(P[4 * d1], P[4 * d1 + 1], P[4 * d1 + 2], P[4 * d1 + 3]);
#pragma unroll
      for (int d0 = 0; d0 < 4; ++d0) h4x2(P[d0], P[d0 + 4], P[d0 + 8], P[d0 + 12]);
      // transpose to e = r + 16 j: thread r's 16-byte chunk c (pairs 2c,
      // 2c + 1) is stored at chunk c ^ (r & 7) of its 128-byte row
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        *reinterpret_cast<uint4*>(tbuf + 128 * r + 16 * (c ^ (r & 7))) =
            make_uint4(__float_as_uint(lo(P[2 * c])), __float_as_uint(hi(P[2 * c])),
                       __float_as_uint(lo(P[2 * c + 1])), __float_as_uint(hi(P[2 * c + 1])));
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // element r + 16 j was written by thread j as pair r of its row
        P[j] = *reinterpret_cast<const uint64_t*>(tbuf + 128 * j + 16 * ((r >> 1) ^ (j & 7)) +
                                                  8 * (r & 1));
      }
      // strides 16 and 64 on j = d2 + 4 d3
#pragma unroll
      for (int d3 = 0; d3 < 4; ++d3) h4x2(P[4 * d3], P[4 * d3 + 1], P[4 * d3 + 2], P[4 * d3 + 3]);
#pragma unroll
      for (int d2 = 0; d2 < 4; ++d2) h4x2(P[d2], P[d2 + 4], P[d2 + 8], P[d2 + 12]);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[i][0][j] = lo(P[j]);
        v[i][1][j] = hi(P[j]);
      }
    }
  }

  // ---- row scale
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < PPT; ++i) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[i][h][j]));
    }
  }
  amax = block_reduce<8>(amax, true, red);
  // eager: the reference's rotated row is T-typed, so its absmax is T(amax)
  const float s = quant_row_scale<T>(kitchen_mode ? amax : QuantTraits<T>::round_t(amax), kitchen_mode);
  if (threadIdx.x == 0) scales[row] = s;
  const float div = quant_divisor<T>(s, kitchen_mode);
  const float recip = __frcp_rn(div);
  const bool fast_div = kitchen_mode == kScaleKitchenCuda;

  // ---- codes: bytes into the team's code buffer at the element's position,
  // then 16 contiguous bytes per thread and group to global memory
  int8_t* qrow = q + static_cast<int64_t>(row) * ldq;
#pragma unroll
  for (int i = 0; i < PPT; ++i) {
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      uint32_t c0, c1;
      quant_pair<T>(pk(v[i][0][j], v[i][1][j]), div, recip, c0, c1, fast_div);
      const int e = ROT ? r + 16 * j : 16 * r + j;
      cbuf[e] = static_cast<uint8_t>(c0);
      cbuf[kCodeStride + e] = static_cast<uint8_t>(c1);
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int g = 2 * (team + i * teams) + h;
      if (g < G) {
        const uint4 out = *reinterpret_cast<const uint4*>(cbuf + h * kCodeStride + 16 * r);
        const int col = g * kGroup + kTeam * r;
        if (vec_out) {
          *reinterpret_cast<uint4*>(qrow + col) = out;
        } else {
          const uint32_t w[4] = {out.x, out.y, out.z, out.w};
#pragma unroll
          for (int j = 0; j < 16; ++j) qrow[col + j] = static_cast<int8_t>(w[j >> 2] >> (8 * (j & 3)));
        }
      }
    }
  }
}

template <typename T, int ACT, bool ROT, int PPT>
__global__ void __launch_bounds__(kMaxTeams * kTeam) quantize_act_rot_kernel(
    const void* __restrict__ x, int64_t ldx, const void* __restrict__ act_w, float act_eps,
    ModArgs mod, int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scales, int K,
    int kitchen_mode, int vec_in, int vec_out) {
  act_rot_row<T, ACT, ROT, PPT>(x, ldx, act_w, act_eps, mod, q, ldq, scales, K, kitchen_mode,
                                vec_in, vec_out);
}

// The bf16 ConvRot quantiser without an input activation, one group pair per
// team (K <= 8192), capped at 48 registers: it needs no more (no spills), and
// 14 instead of 10 of its small CTAs then fit on an SM (measured on B200:
// 5600 x 3072 in 22.5 us against 24.6 us uncapped).  The other variants
// spill under that cap and keep their natural allocation.
template <typename T, int ACT, bool ROT>
__global__ void __maxnreg__(48) quantize_rot_kernel_r48(
    const void* __restrict__ x, int64_t ldx, const void* __restrict__ act_w, float act_eps,
    ModArgs mod, int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scales, int K,
    int kitchen_mode, int vec_in, int vec_out) {
  act_rot_row<T, ACT, ROT, 1>(x, ldx, act_w, act_eps, mod, q, ldq, scales, K, kitchen_mode, vec_in,
                              vec_out);
}

template <typename T, int ACT, bool ROT>
int launch_act_rot(const void* x, int64_t ldx, const void* act_w, float eps, ModArgs mod,
                   int8_t* q, int64_t ldq, float* scales, int64_t rows, int K, int kitchen_mode,
                   cudaStream_t stream) {
  const int G = K / kGroup;
  const int pairs = (G + 1) / 2;
  const int ppt = (pairs + kMaxTeams - 1) / kMaxTeams;  // 1 or 2 for K <= 16384
  const int teams = (pairs + ppt - 1) / ppt;
  const int threads = (teams * kTeam + 31) / 32 * 32;
  const size_t smem = static_cast<size_t>(threads / kTeam) * kTeamBytes;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec_in = a16(x) && (ldx % Ld<T>::kAlign) == 0 && (act_w == nullptr || a16(act_w)) &&
                     (mod.scale == nullptr || a16(mod.scale)) && (mod.shift == nullptr || a16(mod.shift));
  const int vec_out = a16(q) && (ldq % 16) == 0;
  const dim3 grid(static_cast<unsigned>(rows));
  constexpr bool kCapped = std::is_same<T, __nv_bfloat16>::value && ACT == 0 && ROT;
  if (kCapped && ppt == 1) {
    if constexpr (kCapped) {
      quantize_rot_kernel_r48<T, ACT, ROT><<<grid, threads, smem, stream>>>(
          x, ldx, act_w, eps, mod, q, ldq, scales, K, kitchen_mode, vec_in, vec_out);
    }
  } else if (ppt == 1) {
    quantize_act_rot_kernel<T, ACT, ROT, 1><<<grid, threads, smem, stream>>>(
        x, ldx, act_w, eps, mod, q, ldq, scales, K, kitchen_mode, vec_in, vec_out);
  } else {
    quantize_act_rot_kernel<T, ACT, ROT, 2><<<grid, threads, smem, stream>>>(
        x, ldx, act_w, eps, mod, q, ldq, scales, K, kitchen_mode, vec_in, vec_out);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("ConvRot quantiser launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

template <typename T, bool ROT>
int by_act(int act, const void* x, int64_t ldx, const void* act_w, float eps, ModArgs mod,
           int8_t* q, int64_t ldq, float* scales, int64_t rows, int K, int kitchen_mode,
           cudaStream_t stream) {
#define W8A8_ACT_CASE(A) \
  case A: return launch_act_rot<T, A, ROT>(x, ldx, act_w, eps, mod, q, ldq, scales, rows, K, kitchen_mode, stream)
  switch (act) {
    W8A8_ACT_CASE(kInNone);
    W8A8_ACT_CASE(kInGeluTanh);
    W8A8_ACT_CASE(kInSwiGLU);
    W8A8_ACT_CASE(kInRmsNorm);
    W8A8_ACT_CASE(kInSiTU);
    W8A8_ACT_CASE(kInModScale);
    W8A8_ACT_CASE(kInRmsModScale);
    W8A8_ACT_CASE(kInAdaLN);
    W8A8_ACT_CASE(kInRmsAdaLN);
    default: break;
  }
#undef W8A8_ACT_CASE
  set_error("unknown input activation code %d", act);
  return W8A8_ERR_VALUE;
}

}  // namespace

int quantize_act_rot_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                            int rotate, int act, const void* act_w, float act_eps,
                            const void* mod_scale, const void* mod_shift, int64_t mod_group,
                            int8_t* q, int64_t ldq, float* scales, int scale_mode,
                            cudaStream_t stream) {
  if (rows == 0) return 0;
  const int K = static_cast<int>(cols);
  const int km = scale_mode;  // nonzero: kitchen scales (W8A8_SCALE_*)
  const ModArgs mod{mod_scale, mod_shift, mod_group > 0 ? mod_group : 1};
  switch (x_dtype) {
    case W8A8_BF16:
      return rotate ? by_act<__nv_bfloat16, true>(act, x, ldx, act_w, act_eps, mod, q, ldq, scales, rows, K, km, stream)
                    : by_act<__nv_bfloat16, false>(act, x, ldx, act_w, act_eps, mod, q, ldq, scales, rows, K, km, stream);
    case W8A8_F16:
      return rotate ? by_act<__half, true>(act, x, ldx, act_w, act_eps, mod, q, ldq, scales, rows, K, km, stream)
                    : by_act<__half, false>(act, x, ldx, act_w, act_eps, mod, q, ldq, scales, rows, K, km, stream);
    case W8A8_F32:
      return rotate ? by_act<float, true>(act, x, ldx, act_w, act_eps, mod, q, ldq, scales, rows, K, km, stream)
                    : by_act<float, false>(act, x, ldx, act_w, act_eps, mod, q, ldq, scales, rows, K, km, stream);
    default: break;
  }
  set_error("unsupported input dtype code %d", x_dtype);
  return W8A8_ERR_VALUE;
}

}  // namespace w8a8
