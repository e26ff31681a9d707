// One pass per denoising step of the Qwen-Image sampler: the flow (CONST)
// parameterisation of the model outputs, the full-area CFG combine and the
// Euler or ER-SDE update of the latent, fused into one elementwise kernel.
//
// Reference (per element, in ATen's order; every fp32 operation rounds once):
//   denoised_b = x - out_b * sigma                         flow_denoised
//       (inference/src/models/qwen_image21/sampling.rs:165-167, called from
//        denoiser.rs:135 with the model output cast to float)
//   cond = (0 + denoised_c * 1) / (1e-37 + 1), likewise uncond (zeros / 1e-37
//       when the negative branch is skipped)                 full_area_cfg
//       (inference/src/models/qwen_image21/cfg.rs:145-207)
//   denoised = uncond + (cond - uncond) * scale              cfg_combine
//       (sampling.rs:178-180)
//   Euler:  d = (x - denoised) / sigma_hat;  x += d * dt     (sampling.rs:231-277)
//   ER-SDE: x = (r_alpha r) x + (alpha_t (1 - r)) denoised
//           + c3 * derivative + c4 * second + alpha_t * noise * s_noise * dev
//           (inference/src/models/qwen_image21/er_sde.rs:60-134)
// The per-step scalars are computed by the caller with the reference's own
// 0-dim tensor operations and passed as a small device array, so the kernel
// only does the per-element arithmetic, with __f*_rn intrinsics so that no
// operation is contracted into an FMA.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "w8a8_internal.h"

namespace w8a8 {
namespace {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

struct StepArgs {
  float* x;
  const void* oc;
  const void* ou;
  const float* coef;
  float* den;
  float* old_den;
  float* old_der;
  const float* noise;
  int64_t n;
  float scale;
  float s_noise;
  int stage;
  int last;
  int has_noise;
  int denoised_input;
};

// The step's arithmetic for one element.  MODE: 0 denoised only, 1 Euler,
// 2 ER-SDE, 3 Euler churn (x += noise * s_noise * c, before the model runs).
// Inputs: the latent x, the branches' outputs oc / ou (as fp32), the ER-SDE
// state od / odr and the noise nz; outputs the new latent, denoised and the
// new state.
template <int MODE>
__device__ __forceinline__ void step_math(const StepArgs& a, const float* c, float x, float oc,
                                          float ou, float od, float odr, float nz, float& x_out,
                                          float& den, float& od_out, float& odr_out) {
  if constexpr (MODE == 3) {
    x_out = __fadd_rn(x, __fmul_rn(__fmul_rn(nz, a.s_noise), c[0]));
    return;
  } else {
    const float sigma = c[0];
    if (a.denoised_input) {
      den = oc;
    } else {
      // flow_denoised, then full_area_cfg's aggregation (x 1, + 0, / 1: only
      // the sign of a zero can change) and cfg_combine
      const float cond = __fadd_rn(0.0f, __fmul_rn(__fsub_rn(x, __fmul_rn(oc, sigma)), 1.0f));
      float uncond = 0.0f;
      if (a.ou) uncond = __fadd_rn(0.0f, __fmul_rn(__fsub_rn(x, __fmul_rn(ou, sigma)), 1.0f));
      den = __fadd_rn(uncond, __fmul_rn(__fsub_rn(cond, uncond), a.scale));
    }
    if constexpr (MODE == 1) {
      x_out = __fadd_rn(x, __fmul_rn(__fdiv_rn(__fsub_rn(x, den), c[1]), c[2]));
    } else if constexpr (MODE == 2) {
      odr_out = odr;
      if (a.last) {
        x = den;
      } else {
        x = __fadd_rn(__fmul_rn(c[1], x), __fmul_rn(c[2], den));
        if (a.stage >= 2) {
          const float der = __fdiv_rn(__fsub_rn(den, od), c[4]);
          x = __fadd_rn(x, __fmul_rn(c[3], der));
          if (a.stage >= 3) x = __fadd_rn(x, __fmul_rn(c[5], __fdiv_rn(__fsub_rn(der, odr), c[6])));
          odr_out = der;
        }
        if (a.has_noise) x = __fadd_rn(x, __fmul_rn(__fmul_rn(__fmul_rn(c[7], nz), a.s_noise), c[8]));
      }
      od_out = den;
      x_out = x;
    } else {
      x_out = x;
    }
  }
}

// V consecutive elements of a model output as fp32 (V = 4: one 8-byte load
// for 16-bit outputs, one 16-byte load for fp32).
template <typename OutT, int V>
__device__ __forceinline__ void load_out(const void* p, int64_t i, float (&v)[V]) {
  const OutT* q = static_cast<const OutT*>(p) + i;
  if constexpr (V == 4 && sizeof(OutT) == 4) {
    const float4 t = *reinterpret_cast<const float4*>(q);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else if constexpr (V == 4) {
    const uint2 t = *reinterpret_cast<const uint2*>(q);
    const OutT* h = reinterpret_cast<const OutT*>(&t);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = to_f32(h[k]);
  } else {
    v[0] = to_f32(q[0]);
  }
}

template <int V>
__device__ __forceinline__ void load_f(const float* p, int64_t i, float (&v)[V]) {
  if constexpr (V == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p + i);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    v[0] = p[i];
  }
}

template <int V>
__device__ __forceinline__ void store_f(float* p, int64_t i, const float (&v)[V]) {
  if constexpr (V == 4) {
    *reinterpret_cast<float4*>(p + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    p[i] = v[0];
  }
}

// V elements starting at i: vector loads of every operand the mode reads,
// the arithmetic, vector stores of every operand it writes.
template <int MODE, typename OutT, int V>
__device__ __forceinline__ void step_group(const StepArgs& a, const float* c, int64_t i) {
  float x[V], oc[V] = {}, ou[V] = {}, od[V] = {}, odr[V] = {}, nz[V] = {};
  load_f<V>(a.x, i, x);
  if constexpr (MODE != 3) {
    load_out<OutT, V>(a.oc, i, oc);
    if (a.ou) load_out<OutT, V>(a.ou, i, ou);
  }
  if constexpr (MODE == 2) {
    if (!a.last && a.stage >= 2) load_f<V>(a.old_den, i, od);
    if (!a.last && a.stage >= 3) load_f<V>(a.old_der, i, odr);
  }
  if (MODE == 3 || (MODE == 2 && a.has_noise && !a.last)) load_f<V>(a.noise, i, nz);
  float xo[V], den[V], odo[V], odro[V];
#pragma unroll
  for (int k = 0; k < V; ++k) {
    step_math<MODE>(a, c, x[k], oc[k], ou[k], od[k], odr[k], nz[k], xo[k], den[k], odo[k], odro[k]);
  }
  if constexpr (MODE != 0) store_f<V>(a.x, i, xo);
  if constexpr (MODE != 3) {
    if (a.den) store_f<V>(a.den, i, den);
  }
  if constexpr (MODE == 2) {
    store_f<V>(a.old_den, i, odo);
    if (!a.last && a.stage >= 2) store_f<V>(a.old_der, i, odro);
  }
}

// scalars read per mode (the coefficient array's length)
template <int MODE>
constexpr int kCoefs = MODE == 1 ? 3 : (MODE == 2 ? 9 : 1);

// Grid-stride over groups of V elements (V = 4 when every operand is 16-byte
// aligned and n % 4 == 0, else 1).
template <int MODE, typename OutT, int V>
__global__ void __launch_bounds__(256) sampler_step_kernel(StepArgs a) {
  __shared__ float c[16];
  if (threadIdx.x < kCoefs<MODE>) c[threadIdx.x] = a.coef[threadIdx.x];
  __syncthreads();
  const int64_t groups = a.n / V;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < groups;
       g += stride) {
    step_group<MODE, OutT, V>(a, c, g * V);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <int MODE, typename OutT>
int launch_typed(const StepArgs& a, cudaStream_t stream) {
  const bool vec = a.n % 4 == 0 && aligned16(a.x) && aligned16(a.den) && aligned16(a.old_den) &&
                   aligned16(a.old_der) && aligned16(a.noise) &&
                   (reinterpret_cast<uintptr_t>(a.oc) & (4 * sizeof(OutT) - 1)) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.ou) & (4 * sizeof(OutT) - 1)) == 0;
  const int64_t groups = vec ? a.n / 4 : a.n;
  // at most one resident wave (8 CTAs of 256 threads per SM), grid-stride beyond
  const int64_t want = (groups + 255) / 256;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 8;
  const unsigned grid = static_cast<unsigned>(want < cap ? (want > 0 ? want : 1) : cap);
  if (vec) {
    sampler_step_kernel<MODE, OutT, 4><<<grid, 256, 0, stream>>>(a);
  } else {
    sampler_step_kernel<MODE, OutT, 1><<<grid, 256, 0, stream>>>(a);
  }
  return 0;
}

template <int MODE>
int launch_mode(const StepArgs& a, int out_dtype, cudaStream_t stream) {
  switch (out_dtype) {
    case W8A8_BF16: launch_typed<MODE, __nv_bfloat16>(a, stream); break;
    case W8A8_F16: launch_typed<MODE, __half>(a, stream); break;
    default: launch_typed<MODE, float>(a, stream); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("sampler step launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

}  // namespace

int sampler_step_launch(float* x, const void* out_cond, const void* out_uncond, int out_dtype,
                        int64_t n, const float* coef, const w8a8_sampler_step_t& step,
                        float* denoised, float* old_denoised, float* old_derivative,
                        const float* noise, cudaStream_t stream) {
  if (n == 0) return 0;
  StepArgs a{};
  a.x = x;
  a.oc = out_cond;
  a.ou = out_uncond;
  a.coef = coef;
  a.den = denoised;
  a.old_den = old_denoised;
  a.old_der = old_derivative;
  a.noise = noise;
  a.n = n;
  a.scale = step.cfg_scale;
  a.s_noise = step.s_noise;
  a.stage = step.stage;
  a.last = step.last;
  a.has_noise = step.has_noise;
  a.denoised_input = step.denoised_input;
  switch (step.mode) {
    case W8A8_STEP_DENOISED: return launch_mode<0>(a, out_dtype, stream);
    case W8A8_STEP_EULER: return launch_mode<1>(a, out_dtype, stream);
    case W8A8_STEP_ER_SDE: return launch_mode<2>(a, out_dtype, stream);
    default: return launch_mode<3>(a, out_dtype, stream);
  }
}

}  // namespace w8a8
