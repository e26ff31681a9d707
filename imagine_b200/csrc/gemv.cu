// M <= 2 INT8 GEMV (the AdaLN modulation linear, a5) and its fused
// quantise-then-GEMV form, plus the stand-alone int32 -> T dequant.
//
// Replaces the reference's int8_gemv_dequant_kernel / _warp_kernel /
// int8_gemv2_dequant_warp_kernel (native/comfy-port/kitchen/int8_linear.cu:
// 585-708, launcher :1800-1929), Kitchen's int8_linear_m1 (KSRC
// backends/cuda/dlpack_bindings.cpp:3594-3690: quantiser launch + GEMV launch)
// and dequantize_int8_linear(_vec4)_kernel (int8_linear.cu:517-583).
//
// The GEMV is HBM-bound on W (N x K bytes).  Each warp owns kRowsPerWarp rows
// of W and streams them with 16-byte non-allocating loads, dp4a against the
// activation codes held in shared memory, and reduces with shuffles.  The
// fused form quantises x inside every CTA (x is a few KB and L2-resident), so
// quantiser and GEMV are one launch; each warp first asks the TMA unit to
// prefetch its W rows into L2 so that the quantisation latency overlaps the
// first W fetches.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cstdint>

#include "epilogue.cuh"
#include "quant_common.cuh"
#include "w8a8_internal.h"

namespace w8a8 {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kRowsPerWarp = 4;
constexpr int kMaxSmallK = 16384;  // x codes held in shared memory: M * K bytes

template <typename T>
struct In;
template <>
struct In<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float r(float v) { return v; }
  static constexpr float kFinite = 3.4028234663852886e38f;
  static constexpr float kTiny = 1.1754943508222875e-38f;
};
template <>
struct In<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ float r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  static constexpr float kFinite = 3.3895313892515355e38f;
  static constexpr float kTiny = 1.1754943508222875e-38f;
};
template <>
struct In<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ float r(float v) { return __half2float(__float2half_rn(v)); }
  static constexpr float kFinite = 65504.0f;
  static constexpr float kTiny = 6.103515625e-05f;
};

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int w = 1; w < kGemvWarps; ++w) r = fmaxf(r, red[w]);
  return r;
}

// Quantise `rows` rows of x (row stride K) into shared-memory codes with the
// row-wise quantiser's exact numerics.
template <typename T>
__device__ void quantize_rows_to_smem(const T* __restrict__ x, int rows, int K, int scale_mode,
                                      int8_t* sq, float* s_scale, float* red) {
  for (int m = 0; m < rows; ++m) {
    const T* xr = x + static_cast<int64_t>(m) * K;
    float amax = 0.0f;
    for (int c = threadIdx.x; c < K; c += kGemvThreads) amax = fmaxf(amax, fabsf(In<T>::f(xr[c])));
    amax = block_max(amax, red);
    const float scale = quant_row_scale<T>(amax, scale_mode);
    const float div = quant_divisor<T>(scale, scale_mode);
    const float recip = __frcp_rn(div);
    if (threadIdx.x == 0) s_scale[m] = scale;
    for (int c = threadIdx.x; c < K; c += kGemvThreads) {
      const int v = quant_code<T>(In<T>::f(xr[c]), div, recip, scale_mode == kScaleKitchenCuda);
      sq[m * K + c] = static_cast<int8_t>(v);
    }
  }
}

template <int M, typename OutT>
__device__ __forceinline__ void store_out(void* out, int64_t idx, float y) {
  if constexpr (std::is_same<OutT, float>::value) {
    static_cast<float*>(out)[idx] = y;
  } else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
    static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(y);
  } else {
    static_cast<__half*>(out)[idx] = __float2half_rn(y);
  }
}

// One kernel for both the pre-quantised GEMV (InT = int8_t: x are codes, xs
// given) and the fused quantise + GEMV (InT = a float type).
template <int M, typename InT, typename OutT, bool kVec>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(
    const InT* __restrict__ x, const float* __restrict__ xs_in, const int8_t* __restrict__ w,
    EpilogueParams ep, void* __restrict__ out, int N, int K, int scale_mode,
    int8_t* __restrict__ q_out, float* __restrict__ xs_out) {
  extern __shared__ __align__(16) int8_t sq[];  // [M, K] codes
  __shared__ float s_scale[2];
  __shared__ float red[kGemvWarps];
  constexpr bool kFused = !std::is_same<InT, int8_t>::value;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int groups = (N + kRowsPerWarp - 1) / kRowsPerWarp;
  const int first_group = blockIdx.x * kGemvWarps + warp;

  // Warm L2 with this warp's first W rows while x is being prepared.
  if (kFused && kVec && lane < kRowsPerWarp && first_group < groups) {
    const int n = first_group * kRowsPerWarp + lane;
    if (n < N) prefetch_l2_bulk(w + static_cast<int64_t>(n) * K, static_cast<uint32_t>(K));
  }
  if constexpr (kFused) {
    quantize_rows_to_smem<InT>(x, M, K, scale_mode, sq, s_scale, red);
  } else {
    if (kVec) {
      const uint4* src = reinterpret_cast<const uint4*>(x);
      uint4* dst = reinterpret_cast<uint4*>(sq);
      for (int i = threadIdx.x; i < M * K / 16; i += kGemvThreads) dst[i] = __ldg(src + i);
    } else {
      for (int i = threadIdx.x; i < M * K; i += kGemvThreads) sq[i] = x[i];
    }
    if (threadIdx.x < M) s_scale[threadIdx.x] = __ldg(xs_in + threadIdx.x);
  }
  __syncthreads();
  if (kFused && blockIdx.x == 0) {
    if (q_out) {
      for (int i = threadIdx.x; i < M * K; i += kGemvThreads) q_out[i] = sq[i];
    }
    if (xs_out && threadIdx.x < M) xs_out[threadIdx.x] = s_scale[threadIdx.x];
  }

  for (int g = first_group; g < groups; g += gridDim.x * kGemvWarps) {
    const int n0 = g * kRowsPerWarp;
    int acc[M][kRowsPerWarp];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) acc[m][r] = 0;
    if constexpr (kVec) {
      const int kv = K / 16;
#pragma unroll 2
      for (int i = lane; i < kv; i += 32) {
        uint4 wv[kRowsPerWarp];
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const int n = min(n0 + r, N - 1);
          wv[r] = ld_nc_v4(w + static_cast<int64_t>(n) * K + i * 16);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const uint4 xv = reinterpret_cast<const uint4*>(sq + m * K)[i];
#pragma unroll
          for (int r = 0; r < kRowsPerWarp; ++r) {
            int a = acc[m][r];
            a = __dp4a(static_cast<int>(xv.x), static_cast<int>(wv[r].x), a);
            a = __dp4a(static_cast<int>(xv.y), static_cast<int>(wv[r].y), a);
            a = __dp4a(static_cast<int>(xv.z), static_cast<int>(wv[r].z), a);
            a = __dp4a(static_cast<int>(xv.w), static_cast<int>(wv[r].w), a);
            acc[m][r] = a;
          }
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) {
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
          const int n = min(n0 + r, N - 1);
          const int wv = w[static_cast<int64_t>(n) * K + k];
#pragma unroll
          for (int m = 0; m < M; ++m) acc[m][r] += wv * static_cast<int>(sq[m * K + k]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        int a = acc[m][r];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        acc[m][r] = a;
      }
    // lanes 0..M*R-1 each finish one output
    if (lane < M * kRowsPerWarp) {
      const int m = lane / kRowsPerWarp;
      const int r = lane % kRowsPerWarp;
      const int n = n0 + r;
      int a = 0;
#pragma unroll
      for (int mm = 0; mm < M; ++mm)
#pragma unroll
        for (int rr = 0; rr < kRowsPerWarp; ++rr)
          if (mm == m && rr == r) a = acc[mm][rr];
      if (n < N) store_out<M, OutT>(out, static_cast<int64_t>(m) * N + n, epi_value<OutT>(a, m, n, s_scale[m], ep));
    }
  }
}

// Stand-alone dequant: out[m, n] = epilogue(acc[m, n]).
template <typename OutT>
__global__ void __launch_bounds__(256) dequant_kernel(const int32_t* __restrict__ acc,
                                                      const float* __restrict__ xs,
                                                      EpilogueParams ep, void* __restrict__ out,
                                                      int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / N;
    const int n = static_cast<int>(i - m * N);
    store_out<1, OutT>(out, i, epi_value<OutT>(acc[i], static_cast<int>(m), n, __ldg(xs + m), ep));
  }
}

// FP8 e4m3 per-tensor quantiser with the eager numerics
// (inference/src/eager.rs:74-88): t = T(x * T(1/scale)); clamp(t, +-448); e4m3.
template <typename T>
__device__ __forceinline__ uint8_t fp8_one(float xv, float recip_t) {
  float t = In<T>::r(__fmul_rn(xv, recip_t));
  t = fminf(448.0f, fmaxf(-448.0f, t));
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3));
}

template <typename T>
__global__ void __launch_bounds__(256) quantize_fp8_tensor_kernel(const T* __restrict__ x,
                                                                  int64_t numel,
                                                                  const float* __restrict__ scale,
                                                                  uint8_t* __restrict__ out,
                                                                  int vec) {
  const float recip_t = In<T>::r(__fdiv_rn(1.0f, __ldg(scale)));
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  constexpr int kPer = 16 / sizeof(T);
  if (vec) {
    const int64_t nv = numel / kPer;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < nv; i += stride) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(x) + i);
      const T* e = reinterpret_cast<const T*>(&v);
      uint8_t b[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) b[j] = fp8_one<T>(In<T>::f(e[j]), recip_t);
      if constexpr (kPer == 8) {
        uint2 o;
        o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (static_cast<uint32_t>(b[3]) << 24);
        o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (static_cast<uint32_t>(b[7]) << 24);
        reinterpret_cast<uint2*>(out)[i] = o;
      } else {
        reinterpret_cast<uint32_t*>(out)[i] =
            b[0] | (b[1] << 8) | (b[2] << 16) | (static_cast<uint32_t>(b[3]) << 24);
      }
    }
    for (int64_t i = nv * kPer + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < numel; i += stride) {
      out[i] = fp8_one<T>(In<T>::f(x[i]), recip_t);
    }
  } else {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < numel; i += stride) {
      out[i] = fp8_one<T>(In<T>::f(x[i]), recip_t);
    }
  }
}

EpilogueParams params_of(const w8a8_epilogue_t* e, int64_t N) {
  EpilogueParams ep{};
  ep.rscale_rows = e->residual_scale_rows;
  ep.ld_rscale = N;
  ep.ws = e->ws;
  ep.ws_scalar = e->ws_numel == 1 ? 1 : 0;
  ep.bias = e->bias;
  ep.residual = e->residual;
  ep.ldr = e->ldr;
  ep.rscale = e->residual_scale;
  ep.dq_order = e->dequant_order;
  ep.act = e->activation;
  return ep;
}

template <int M, typename InT, typename OutT>
int launch_gemv_t(const InT* x, const float* xs, const int8_t* w, const w8a8_epilogue_t* epi,
                  void* out, int N, int K, int scale_mode, int8_t* q_out, float* xs_out,
                  cudaStream_t stream) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = K % 16 == 0 && a16(w) && (std::is_same<InT, int8_t>::value ? a16(x) : true);
  const int groups = (N + kRowsPerWarp - 1) / kRowsPerWarp;
  const int sms = device_sm_count();
  int grid = (groups + kGemvWarps - 1) / kGemvWarps;
  const int cap = sms * 4;
  if (std::is_same<InT, int8_t>::value == false && grid > cap) grid = cap;  // fused: fewer re-quantisations
  if (grid < 1) grid = 1;
  const size_t smem = static_cast<size_t>(M) * K;
  auto kern = vec ? gemv_kernel<M, InT, OutT, true> : gemv_kernel<M, InT, OutT, false>;
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  }
  kern<<<grid, kGemvThreads, smem, stream>>>(x, xs, w, params_of(epi, N), out, N, K, scale_mode, q_out,
                                             xs_out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("GEMV launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

template <typename InT, typename OutT>
int gemv_m(const InT* x, const float* xs, const int8_t* w, const w8a8_epilogue_t* epi, void* out,
           int M, int N, int K, int scale_mode, int8_t* q_out, float* xs_out, cudaStream_t stream) {
  if (M == 1) return launch_gemv_t<1, InT, OutT>(x, xs, w, epi, out, N, K, scale_mode, q_out, xs_out, stream);
  return launch_gemv_t<2, InT, OutT>(x, xs, w, epi, out, N, K, scale_mode, q_out, xs_out, stream);
}

template <typename InT>
int gemv_out(const InT* x, const float* xs, const int8_t* w, const w8a8_epilogue_t* epi, void* out,
             int out_dtype, int M, int N, int K, int scale_mode, int8_t* q_out, float* xs_out,
             cudaStream_t stream) {
  switch (out_dtype) {
    case W8A8_BF16: return gemv_m<InT, __nv_bfloat16>(x, xs, w, epi, out, M, N, K, scale_mode, q_out, xs_out, stream);
    case W8A8_F16: return gemv_m<InT, __half>(x, xs, w, epi, out, M, N, K, scale_mode, q_out, xs_out, stream);
    case W8A8_F32: return gemv_m<InT, float>(x, xs, w, epi, out, M, N, K, scale_mode, q_out, xs_out, stream);
    default: break;
  }
  set_error("unsupported output dtype code %d", out_dtype);
  return W8A8_ERR_VALUE;
}

}  // namespace

int gemv_launch(const int8_t* q, const int8_t* w, const float* xs, const w8a8_epilogue_t* epi,
                void* out, int out_dtype, int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (N == 0) return 0;
  if (M * K > 2 * kMaxSmallK) {
    set_error("GEMV supports M*K <= %d, got M=%lld K=%lld", 2 * kMaxSmallK, (long long)M, (long long)K);
    return W8A8_ERR_VALUE;
  }
  return gemv_out<int8_t>(q, xs, w, epi, out, out_dtype, (int)M, (int)N, (int)K, 0, nullptr, nullptr, stream);
}

int linear_small_launch(const void* x, int x_dtype, const int8_t* w, const w8a8_epilogue_t* epi,
                        int scale_mode, int8_t* q_out, float* xs_out, void* out, int out_dtype,
                        int64_t M, int64_t N, int64_t K, cudaStream_t stream) {
  if (N == 0) return 0;
  if (M * K > 2 * kMaxSmallK) {
    set_error("fused small linear supports M*K <= %d, got M=%lld K=%lld", 2 * kMaxSmallK, (long long)M, (long long)K);
    return W8A8_ERR_VALUE;
  }
  switch (x_dtype) {
    case W8A8_BF16:
      return gemv_out<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), nullptr, w, epi, out, out_dtype, (int)M, (int)N, (int)K, scale_mode, q_out, xs_out, stream);
    case W8A8_F16:
      return gemv_out<__half>(static_cast<const __half*>(x), nullptr, w, epi, out, out_dtype, (int)M, (int)N, (int)K, scale_mode, q_out, xs_out, stream);
    case W8A8_F32:
      return gemv_out<float>(static_cast<const float*>(x), nullptr, w, epi, out, out_dtype, (int)M, (int)N, (int)K, scale_mode, q_out, xs_out, stream);
    default: break;
  }
  set_error("unsupported input dtype code %d", x_dtype);
  return W8A8_ERR_VALUE;
}

int dequant_launch(const int32_t* acc, const float* xs, const w8a8_epilogue_t* epi, void* out,
                   int out_dtype, int64_t M, int64_t N, cudaStream_t stream) {
  if (M == 0 || N == 0) return 0;
  const EpilogueParams ep = params_of(epi, N);
  const int64_t total = M * N;
  int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, device_sm_count() * 16));
  switch (out_dtype) {
    case W8A8_BF16: dequant_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(acc, xs, ep, out, M, N); break;
    case W8A8_F16: dequant_kernel<__half><<<grid, 256, 0, stream>>>(acc, xs, ep, out, M, N); break;
    case W8A8_F32: dequant_kernel<float><<<grid, 256, 0, stream>>>(acc, xs, ep, out, M, N); break;
    default:
      set_error("unsupported output dtype code %d", out_dtype);
      return W8A8_ERR_VALUE;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("dequant launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

int quantize_fp8_tensor_launch(const void* x, int x_dtype, int64_t numel, const float* scale,
                               uint8_t* out, cudaStream_t stream) {
  if (numel == 0) return 0;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = a16(x) && (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
  int grid = static_cast<int>(std::min<int64_t>((numel / 8 + 255) / 256 + 1, device_sm_count() * 8));
  switch (x_dtype) {
    case W8A8_BF16: quantize_fp8_tensor_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), numel, scale, out, vec); break;
    case W8A8_F16: quantize_fp8_tensor_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(x), numel, scale, out, vec); break;
    case W8A8_F32: quantize_fp8_tensor_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), numel, scale, out, vec); break;
    default:
      set_error("unsupported input dtype code %d", x_dtype);
      return W8A8_ERR_VALUE;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("fp8 quantiser launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

// ---- pre-tiled weights for few-row GEMMs -----------------------------------
// tiles[((nb * KB + kb) * 128 + r) * 128 + c] = W[nb * 128 + r][kb * 128 + c]
// (zero outside N x K): every 128 x 128-byte TMA tile of B is one contiguous
// 16 KB block, so a GEMM streaming W from HBM reads it sequentially.
namespace {
__global__ void __launch_bounds__(256) pack_weight_tiles_kernel(const int8_t* __restrict__ w,
                                                                int64_t ldw, int64_t N, int64_t K,
                                                                int64_t kb_count, int vec,
                                                                int8_t* __restrict__ tiles,
                                                                int64_t chunks) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  const int64_t row = i >> 3;  // tiled row (128 bytes = 8 chunks of 16)
  const int c16 = static_cast<int>(i & 7);
  const int64_t blk = row >> 7;  // (nb * KB + kb)
  const int r = static_cast<int>(row & 127);
  const int64_t nb = blk / kb_count, kb = blk - nb * kb_count;
  const int64_t n = nb * 128 + r;
  const int64_t k0 = kb * 128 + c16 * 16;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (n < N && k0 < K) {
    const int8_t* src = w + n * ldw + k0;
    if (vec && k0 + 16 <= K) {
      v = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
      uint8_t b[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) b[j] = k0 + j < K ? static_cast<uint8_t>(src[j]) : 0;
      v = *reinterpret_cast<const uint4*>(b);
    }
  }
  reinterpret_cast<uint4*>(tiles)[i] = v;
}
}  // namespace

int64_t weight_tiles_bytes(int64_t N, int64_t K) {
  return (N + 127) / 128 * ((K + 127) / 128) * 128 * 128;
}

int pack_weight_tiles_launch(const int8_t* w, int64_t ldw, int64_t N, int64_t K, int8_t* tiles,
                             cudaStream_t stream) {
  const int64_t chunks = weight_tiles_bytes(N, K) / 16;
  if (chunks == 0) return 0;
  const int vec = (reinterpret_cast<uintptr_t>(w) & 15u) == 0 && ldw % 16 == 0;
  const int64_t grid = (chunks + 255) / 256;
  pack_weight_tiles_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(
      w, ldw, N, K, (K + 127) / 128, vec, tiles, chunks);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("weight tile packing launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

}  // namespace w8a8
