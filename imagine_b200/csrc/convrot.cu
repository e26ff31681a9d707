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
// Numerics with ROT (the reference's fused kernel):
//   v   = act(x) in fp32 (GELU-tanh, SwiGLU = silu(gate) * up, RMSNorm =
//         x * rsqrt(mean(x^2) + eps) * w, or SiTU), no rounding
//   v   = H_256 v per 256-group: four radix-4 stages (digit strides 1, 4, 16,
//         64), each output 0.5 * (a +- b +- c +- d) summed left to right with
//         one operand negated (int8_linear.cu:253-261, 881-934)
//   s   = max(min(amax_fp32, finite_max(T)) * (1/127), 1e-30)     (kitchen)
//         max(T(amax_fp32) / 127, 1e-30)                          (eager)
//   q   = clamp(rne(T(T(v) / T(s))), -128, 127)      (int8_linear.cu:53-57)
// Without ROT the activation output is rounded to T after each op the ATen
// sequence rounds after, then quantised like the plain row quantiser.
//
// Layout: one CTA per row; a team of 16 threads owns one 256-group at a time,
// each thread 16 elements.  Stages 1 and 4 run on 16 contiguous elements in
// registers (e = 16 r + j); the team transposes through a bank-conflict-free
// swizzled shared buffer to e = r + 16 j for stages 16 and 64; the int8 codes
// go back through shared memory as bytes so every thread stores 16 contiguous
// bytes.  A thread keeps GPT groups in registers (K <= 16 teams x GPT x 256),
// so x is read from HBM exactly once.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "quant_common.cuh"
#include "w8a8_internal.h"

namespace w8a8 {
namespace {

constexpr int kGroup = 256;
constexpr int kTeam = 16;          // threads per group
constexpr int kMaxTeams = 16;      // 256 threads per CTA
constexpr int kTeamFloats = kGroup + 16;  // padded: teams of one warp use disjoint banks

enum InputAct : int { kInNone = 0, kInGeluTanh = 1, kInSwiGLU = 2, kInRmsNorm = 3, kInSiTU = 4 };

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

// Round to T when the ATen sequence would (ROUND), otherwise keep fp32.
template <typename T, bool ROUND>
__device__ __forceinline__ float rt(float v) {
  if constexpr (ROUND) {
    return QuantTraits<T>::round_t(v);
  } else {
    return v;
  }
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

// One radix-4 butterfly of the normalised H4 (rows ++ +-, ++-+, +-++, -+++),
// every sum left to right exactly as int8_linear.cu:253-261 orders it;
// (-a) + b is computed as b - a, which rounds identically.
__device__ __forceinline__ void h4(float& a, float& b, float& c, float& d) {
  const float ab = __fadd_rn(a, b);
  const float amb = __fsub_rn(a, b);
  const float bma = __fsub_rn(b, a);
  const float y0 = __fsub_rn(__fadd_rn(ab, c), d);
  const float y1 = __fadd_rn(__fsub_rn(ab, c), d);
  const float y2 = __fadd_rn(__fadd_rn(amb, c), d);
  const float y3 = __fadd_rn(__fadd_rn(bma, c), d);
  a = __fmul_rn(0.5f, y0);
  b = __fmul_rn(0.5f, y1);
  c = __fmul_rn(0.5f, y2);
  d = __fmul_rn(0.5f, y3);
}

// 16 codes (values already T-representable) -> 16 bytes.
template <typename T>
__device__ __forceinline__ uint4 quant16(const float* v, float div, float recip) {
  int q[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) q[j] = quant_code<T>(v[j], div, recip);
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t t;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(t) : "r"(q[4 * i + 3]), "r"(q[4 * i + 2]));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;"
        : "=r"(w[i])
        : "r"(q[4 * i + 1]), "r"(q[4 * i]), "r"(t));
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
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

// GPT: 256-groups per team kept in registers.
template <typename T, int ACT, bool ROT, int GPT>
__global__ void __launch_bounds__(kMaxTeams * kTeam) quantize_act_rot_kernel(
    const void* __restrict__ x, int64_t ldx, const void* __restrict__ act_w, float act_eps,
    int8_t* __restrict__ q, int64_t ldq, float* __restrict__ scales, int K, int kitchen_mode,
    int vec_in, int vec_out) {
  __shared__ __align__(16) float xbuf[kMaxTeams * kTeamFloats];
  __shared__ float red[8];
  const int row = blockIdx.x;
  const int team = threadIdx.x / kTeam;
  const int r = threadIdx.x % kTeam;
  const int teams = blockDim.x / kTeam;
  const int G = K / kGroup;
  const int64_t xrow = static_cast<int64_t>(row) * ldx;
  float* tb = xbuf + team * kTeamFloats;
  // Without ROT the values are T-rounded at each step the ATen sequence rounds.
  constexpr bool kRound = !ROT;

  float v[GPT][16];
  // ---- load (+ elementwise activation)
  float sumsq = 0.0f;
#pragma unroll
  for (int i = 0; i < GPT; ++i) {
    const int g = team + i * teams;
    const int col = g * kGroup + kTeam * r;
    if (g < G) {
      if constexpr (ACT == kInSwiGLU || ACT == kInSiTU) {
        float gate[16], up[16];
        load16<T>(x, xrow + col, vec_in, gate);
        load16<T>(x, xrow + K + col, vec_in, up);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if constexpr (ACT == kInSwiGLU) {
            v[i][j] = rt<T, kRound>(rt<T, kRound>(in_silu(gate[j])) * up[j]);
          } else {
            // 25 tanh(a / 25) * (4 tanh(b / 4) * sigmoid(b))
            // (inference/src/int8_linear.rs:54-74)
            const float a = rt<T, kRound>(25.0f * rt<T, kRound>(tanhf(rt<T, kRound>(gate[j] / 25.0f))));
            const float t4 = rt<T, kRound>(4.0f * rt<T, kRound>(tanhf(rt<T, kRound>(up[j] / 4.0f))));
            const float gated = rt<T, kRound>(t4 * rt<T, kRound>(in_sigmoid(up[j])));
            v[i][j] = rt<T, kRound>(a * gated);
          }
        }
      } else {
        load16<T>(x, xrow + col, vec_in, v[i]);
        if constexpr (ACT == kInGeluTanh) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[i][j] = rt<T, kRound>(in_gelu_tanh(v[i][j]));
        } else if constexpr (ACT == kInRmsNorm) {
#pragma unroll
          for (int j = 0; j < 16; ++j) sumsq = __fmaf_rn(v[i][j], v[i][j], sumsq);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[i][j] = 0.0f;
    }
  }
  if constexpr (ACT == kInRmsNorm) {
    // x * rsqrt(mean(x^2) + eps) * w  (int8_linear.cu:1239-1267; ATen's
    // rms_norm forms the same fp32 product and rounds it to T once)
    const float ss = block_reduce<8>(sumsq, false, red);
    const float rstd = rsqrtf(ss / static_cast<float>(K) + act_eps);
#pragma unroll
    for (int i = 0; i < GPT; ++i) {
      const int g = team + i * teams;
      if (g < G) {
        float w[16];
        load16<T>(act_w, g * kGroup + kTeam * r, vec_in, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[i][j] = rt<T, kRound>(__fmul_rn(__fmul_rn(v[i][j], rstd), w[j]));
      }
    }
  }

  // ---- Hadamard transform per 256-group
  if constexpr (ROT) {
#pragma unroll
    for (int i = 0; i < GPT; ++i) {
      // stride 1 and stride 4 on e = 16 r + j, j = d0 + 4 d1
#pragma unroll
      for (int d1 = 0; d1 < 4; ++d1) h4(v[i][4 * d1], v[i][4 * d1 + 1], v[i][4 * d1 + 2], v[i][4 * d1 + 3]);
#pragma unroll
      for (int d0 = 0; d0 < 4; ++d0) h4(v[i][d0], v[i][d0 + 4], v[i][d0 + 8], v[i][d0 + 12]);
      // transpose to e = r + 16 j: float4 chunk c of thread r is stored at
      // chunk 4 r + (c ^ ((r >> 1) & 3)) of the team's buffer
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int pc = 4 * r + (c ^ ((r >> 1) & 3));
        *reinterpret_cast<float4*>(tb + 4 * pc) =
            make_float4(v[i][4 * c], v[i][4 * c + 1], v[i][4 * c + 2], v[i][4 * c + 3]);
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // element r + 16 j was written by thread j as its chunk r >> 2, word r & 3
        v[i][j] = tb[16 * j + 4 * ((r >> 2) ^ ((j >> 1) & 3)) + (r & 3)];
      }
      // stride 16 and stride 64 on j = d2 + 4 d3
#pragma unroll
      for (int d3 = 0; d3 < 4; ++d3) h4(v[i][4 * d3], v[i][4 * d3 + 1], v[i][4 * d3 + 2], v[i][4 * d3 + 3]);
#pragma unroll
      for (int d2 = 0; d2 < 4; ++d2) h4(v[i][d2], v[i][d2 + 4], v[i][d2 + 8], v[i][d2 + 12]);
    }
  }

  // ---- row scale
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < GPT; ++i) {
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
  }
  amax = block_reduce<8>(amax, true, red);
  // eager: the reference's rotated row is T-typed, so its absmax is T(amax)
  const float s = quant_row_scale<T>(kitchen_mode ? amax : QuantTraits<T>::round_t(amax), kitchen_mode);
  if (threadIdx.x == 0) scales[row] = s;
  const float div = quant_divisor<T>(s);
  const float recip = __frcp_rn(div);

  // ---- codes
  int8_t* qrow = q + static_cast<int64_t>(row) * ldq;
#pragma unroll
  for (int i = 0; i < GPT; ++i) {
    const int g = team + i * teams;
    float t[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) t[j] = QuantTraits<T>::round_t(v[i][j]);
    const uint4 c = quant16<T>(t, div, recip);
    uint4 out = c;
    if constexpr (ROT) {
      // codes are for e = r + 16 j: bounce through shared memory as bytes
      uint8_t* cb = reinterpret_cast<uint8_t*>(tb);
      __syncwarp();
      const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) cb[r + 16 * j] = static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)));
      __syncwarp();
      out = *reinterpret_cast<const uint4*>(cb + 16 * r);
    }
    if (g < G) {
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

template <typename T, int ACT, bool ROT>
int launch_act_rot(const void* x, int64_t ldx, const void* act_w, float eps, int8_t* q,
                   int64_t ldq, float* scales, int64_t rows, int K, int kitchen_mode,
                   cudaStream_t stream) {
  const int G = K / kGroup;
  const int gpt = (G + kMaxTeams - 1) / kMaxTeams;
  const int teams = (G + gpt - 1) / gpt;
  const int threads = (teams * kTeam + 31) / 32 * 32;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec_in = a16(x) && (ldx % Ld<T>::kAlign) == 0 && (act_w == nullptr || a16(act_w));
  const int vec_out = a16(q) && (ldq % 16) == 0;
  const dim3 grid(static_cast<unsigned>(rows));
#define W8A8_LAUNCH_GPT(N)                                                                        \
  quantize_act_rot_kernel<T, ACT, ROT, N><<<grid, threads, 0, stream>>>(                           \
      x, ldx, act_w, eps, q, ldq, scales, K, kitchen_mode, vec_in, vec_out)
  switch (gpt) {
    case 1: W8A8_LAUNCH_GPT(1); break;
    case 2: W8A8_LAUNCH_GPT(2); break;
    case 3: W8A8_LAUNCH_GPT(3); break;
    default: W8A8_LAUNCH_GPT(4); break;
  }
#undef W8A8_LAUNCH_GPT
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("ConvRot quantiser launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

template <typename T, bool ROT>
int by_act(int act, const void* x, int64_t ldx, const void* act_w, float eps, int8_t* q,
           int64_t ldq, float* scales, int64_t rows, int K, int kitchen_mode, cudaStream_t stream) {
  switch (act) {
    case kInNone: return launch_act_rot<T, kInNone, ROT>(x, ldx, act_w, eps, q, ldq, scales, rows, K, kitchen_mode, stream);
    case kInGeluTanh: return launch_act_rot<T, kInGeluTanh, ROT>(x, ldx, act_w, eps, q, ldq, scales, rows, K, kitchen_mode, stream);
    case kInSwiGLU: return launch_act_rot<T, kInSwiGLU, ROT>(x, ldx, act_w, eps, q, ldq, scales, rows, K, kitchen_mode, stream);
    case kInRmsNorm: return launch_act_rot<T, kInRmsNorm, ROT>(x, ldx, act_w, eps, q, ldq, scales, rows, K, kitchen_mode, stream);
    case kInSiTU: return launch_act_rot<T, kInSiTU, ROT>(x, ldx, act_w, eps, q, ldq, scales, rows, K, kitchen_mode, stream);
    default: break;
  }
  set_error("unknown input activation code %d", act);
  return W8A8_ERR_VALUE;
}

}  // namespace

int quantize_act_rot_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                            int rotate, int act, const void* act_w, float act_eps, int8_t* q,
                            int64_t ldq, float* scales, int scale_mode, cudaStream_t stream) {
  if (rows == 0) return 0;
  const int K = static_cast<int>(cols);
  const int km = scale_mode == W8A8_SCALE_KITCHEN ? 1 : 0;
  switch (x_dtype) {
    case W8A8_BF16:
      return rotate ? by_act<__nv_bfloat16, true>(act, x, ldx, act_w, act_eps, q, ldq, scales, rows, K, km, stream)
                    : by_act<__nv_bfloat16, false>(act, x, ldx, act_w, act_eps, q, ldq, scales, rows, K, km, stream);
    case W8A8_F16:
      return rotate ? by_act<__half, true>(act, x, ldx, act_w, act_eps, q, ldq, scales, rows, K, km, stream)
                    : by_act<__half, false>(act, x, ldx, act_w, act_eps, q, ldq, scales, rows, K, km, stream);
    case W8A8_F32:
      return rotate ? by_act<float, true>(act, x, ldx, act_w, act_eps, q, ldq, scales, rows, K, km, stream)
                    : by_act<float, false>(act, x, ldx, act_w, act_eps, q, ldq, scales, rows, K, km, stream);
    default: break;
  }
  set_error("unsupported input dtype code %d", x_dtype);
  return W8A8_ERR_VALUE;
}

}  // namespace w8a8
