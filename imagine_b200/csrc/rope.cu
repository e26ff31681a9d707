// Q/K RMSNorm + interleaved-pair RoPE after the QKV projection.
//
// Replaces the reference's `rms_rope(q, k, freqs_cis, q_scale, k_scale,
// epsilon)` (call site inference/src/models/qwen_image21/dit.rs:486-505; eager
// body inference/src/backend_rope.rs:146-223; Kitchen kernel KSRC
// backends/cuda/ops/rms_rope.cu:38-240, rope_device.cuh:65-97) for the
// interleaved (non-split) rotation over the full head:
//   rrms  = 1 / sqrt(sum(x^2) / D + eps)                    (fp32)
//   n     = T(x * rrms * w)                                 (one rounding)
//   (y0, y1) = (f00 n0 + f01 n1, f10 n0 + f11 n1)           (fp32)
//   out   = T(y)
// for every pair (x[2i], x[2i+1]) of a head, with freqs_cis [.., D/2, 2, 2]
// (f[i][r][c]) fp32 indexed by the token's position.
//
// Layout: one warp per token; lane l holds the EPL contiguous elements
// [EPL l, EPL l + EPL) (EPL = D / 32, even) of each head row, loaded with one
// vector load; the sum of squares is a warp reduction.  The lane's EPL/2 pair
// rotations (float4 each) are read once per token and serve every head of q
// and k; four head rows are in flight per warp.  Memory-bound: q and k are
// read and written once.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "w8a8_internal.h"

namespace w8a8 {
namespace {

constexpr int kRopeWarps = 8;

template <typename T>
struct RT;
template <>
struct RT<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};
template <>
struct RT<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half t(float v) { return __float2half_rn(v); }
};
template <>
struct RT<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float t(float v) { return v; }
};

// EPL consecutive elements of a row (vector load when the row is aligned).
template <typename T, int EPL>
__device__ __forceinline__ void load_row(const T* p, bool vec, float (&v)[EPL]) {
  constexpr int kWords = static_cast<int>(EPL * sizeof(T) / 8);
  if constexpr (kWords > 0 && (EPL * sizeof(T)) % 8 == 0) {
    if (vec) {
      uint2 raw[kWords];
#pragma unroll
      for (int i = 0; i < kWords; ++i) raw[i] = reinterpret_cast<const uint2*>(p)[i];
      const T* e = reinterpret_cast<const T*>(raw);
#pragma unroll
      for (int j = 0; j < EPL; ++j) v[j] = RT<T>::f(e[j]);
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < EPL; ++j) v[j] = RT<T>::f(p[j]);
}

template <typename T, int EPL>
__device__ __forceinline__ void store_row(T* p, bool vec, const float (&v)[EPL]) {
  T e[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) e[j] = RT<T>::t(v[j]);
  constexpr int kWords = static_cast<int>(EPL * sizeof(T) / 8);
  if constexpr (kWords > 0 && (EPL * sizeof(T)) % 8 == 0) {
    if (vec) {
#pragma unroll
      for (int i = 0; i < kWords; ++i) {
        reinterpret_cast<uint2*>(p)[i] = reinterpret_cast<const uint2*>(e)[i];
      }
      return;
    }
  }
#pragma unroll
  for (int j = 0; j < EPL; ++j) p[j] = e[j];
}

// RMSNorm with weight w, then the interleaved rotation, of one head row held
// as EPL values per lane; f holds this lane's EPL/2 pair rotations.
template <typename T, int EPL>
__device__ __forceinline__ void rms_rope_vals(float (&v)[EPL], const float (&wv)[EPL],
                                              const float4 (&f)[EPL / 2], float eps, int D) {
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) ss = __fmaf_rn(v[j], v[j], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  // 1 / sqrt in two IEEE roundings, the form torch's rsqrt takes
  const float rrms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps)));
#pragma unroll
  for (int j = 0; j < EPL; j += 2) {
    const float n0 = RT<T>::f(RT<T>::t(__fmul_rn(__fmul_rn(v[j], rrms), wv[j])));
    const float n1 = RT<T>::f(RT<T>::t(__fmul_rn(__fmul_rn(v[j + 1], rrms), wv[j + 1])));
    const float4 r = f[j / 2];  // (f00, f01, f10, f11)
    v[j] = __fmaf_rn(r.y, n1, __fmul_rn(r.x, n0));
    v[j + 1] = __fmaf_rn(r.w, n1, __fmul_rn(r.z, n0));
  }
}

constexpr int kRopeUnroll = 4;  // head rows in flight per warp

// All heads of one tensor (q or k) of token t, kRopeUnroll rows at a time.
template <typename T, int EPL>
__device__ __forceinline__ void rms_rope_heads(const T* x, T* out, const float (&wv)[EPL],
                                               const float4 (&f)[EPL / 2], float eps, int heads,
                                               int D, int lane, bool vec) {
  for (int h0 = 0; h0 < heads; h0 += kRopeUnroll) {
    float v[kRopeUnroll][EPL];
#pragma unroll
    for (int u = 0; u < kRopeUnroll; ++u) {
      if (h0 + u < heads) load_row<T, EPL>(x + (h0 + u) * D + EPL * lane, vec, v[u]);
    }
#pragma unroll
    for (int u = 0; u < kRopeUnroll; ++u) {
      if (h0 + u < heads) {
        rms_rope_vals<T, EPL>(v[u], wv, f, eps, D);
        store_row<T, EPL>(out + (h0 + u) * D + EPL * lane, vec, v[u]);
      }
    }
  }
}

// One warp per token and tensor: lane l owns elements [EPL l, EPL l + EPL) of every
// head, loads the rotations of its EPL/2 pairs once, then walks the heads of
// q (or, in the next warp, of k).
template <typename T, int EPL>
__global__ void __launch_bounds__(kRopeWarps * 32) rms_rope_kernel(
    const T* __restrict__ q, const T* __restrict__ k, T* __restrict__ q_out, T* __restrict__ k_out,
    int64_t rows, int heads, int D, int64_t ldq, int64_t ldk, int64_t ldqo, int64_t ldko,
    const float* __restrict__ freqs, int64_t freq_rows, const T* __restrict__ q_scale,
    const T* __restrict__ k_scale, float eps, int vec) {
  const int lane = threadIdx.x & 31;
  // warp w: token w / per, q (even w) or k (odd w) when both are given
  const int per = k ? 2 : 1;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * kRopeWarps + (threadIdx.x >> 5);
  const int64_t t = w / per;
  if (t >= rows) return;
  const bool is_k = per == 2 && (w & 1);
  const float4* fr = reinterpret_cast<const float4*>(freqs + (t % freq_rows) * (2 * D));
  float4 f[EPL / 2];
#pragma unroll
  for (int j = 0; j < EPL / 2; ++j) f[j] = __ldg(fr + (EPL * lane) / 2 + j);
  float wv[EPL];
  load_row<T, EPL>((is_k ? k_scale : q_scale) + EPL * lane, vec != 0, wv);
  if (is_k) {
    rms_rope_heads<T, EPL>(k + t * ldk, k_out + t * ldko, wv, f, eps, heads, D, lane, vec != 0);
  } else {
    rms_rope_heads<T, EPL>(q + t * ldq, q_out + t * ldqo, wv, f, eps, heads, D, lane, vec != 0);
  }
}

template <typename T>
int launch_rope(const void* q, const void* k, void* q_out, void* k_out, int64_t rows, int heads,
                int D, int64_t ldq, int64_t ldk, int64_t ldqo, int64_t ldko, const float* freqs,
                int64_t freq_rows, const void* q_scale, const void* k_scale, float eps,
                cudaStream_t stream) {
  auto a8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  const int epl = D / 32;
  const bool row_vec = (ldq * static_cast<int64_t>(sizeof(T))) % 8 == 0 &&
                       (ldqo * static_cast<int64_t>(sizeof(T))) % 8 == 0 &&
                       (!k || ((ldk * static_cast<int64_t>(sizeof(T))) % 8 == 0 &&
                               (ldko * static_cast<int64_t>(sizeof(T))) % 8 == 0));
  const int vec = row_vec && a8(q) && a8(q_out) && a8(q_scale) && (!k || (a8(k) && a8(k_out) && a8(k_scale)));
  const int64_t warps = rows * (k ? 2 : 1);  // one warp per token and tensor
  const dim3 grid(static_cast<unsigned>((warps + kRopeWarps - 1) / kRopeWarps));
  const T* qp = static_cast<const T*>(q);
  const T* kp = static_cast<const T*>(k);
  T* qo = static_cast<T*>(q_out);
  T* ko = static_cast<T*>(k_out);
  const T* qs = static_cast<const T*>(q_scale);
  const T* ks = static_cast<const T*>(k_scale);
#define W8A8_ROPE(E)                                                                          \
  rms_rope_kernel<T, E><<<grid, kRopeWarps * 32, 0, stream>>>(qp, kp, qo, ko, rows, heads, D,  \
                                                             ldq, ldk, ldqo, ldko, freqs,      \
                                                             freq_rows, qs, ks, eps, vec)
  switch (epl) {
    case 2: W8A8_ROPE(2); break;
    case 4: W8A8_ROPE(4); break;
    case 6: W8A8_ROPE(6); break;
    case 8: W8A8_ROPE(8); break;
    default:
      set_error("rms_rope supports head_dim 64, 128, 192 or 256, got %d", D);
      return W8A8_ERR_VALUE;
  }
#undef W8A8_ROPE
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("rms_rope launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

// Row-blocked copy of the rotations for the fused projection epilogue (one
// lane per row there): out[((r / 32) * 64 + p) * 32 + r % 32] = the float4
// (f00, f01, f10, f11) of pair p at token r % freq_rows, for every row r of
// rows_pad (a multiple of 128).  One thread per (row, pair); consecutive
// threads write consecutive rows of one pair, so stores are coalesced.
__global__ void __launch_bounds__(256) rope_freqs_rows_kernel(const float4* __restrict__ freqs,
                                                             int64_t freq_rows, int64_t rows_pad,
                                                             float4* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;  // output float4
  if (i >= rows_pad * 64) return;
  const int64_t lane = i & 31;
  const int64_t p = (i >> 5) & 63;
  const int64_t blk = i >> 11;
  const int64_t r = blk * 32 + lane;
  out[i] = __ldg(freqs + (r % freq_rows) * 64 + p);
}

}  // namespace

int rope_freqs_rows_launch(const float* freqs, int64_t freq_rows, int64_t rows, float* out,
                           cudaStream_t stream) {
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  const int64_t n = rows_pad * 64;
  if (n == 0) return 0;
  rope_freqs_rows_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(freqs), freq_rows, rows_pad, reinterpret_cast<float4*>(out));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("rope_freqs_rows launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

int rms_rope_launch(const void* q, const void* k, void* q_out, void* k_out, int dtype,
                    int64_t rows, int heads, int head_dim, int64_t ldq, int64_t ldk, int64_t ldqo,
                    int64_t ldko, const float* freqs, int64_t freq_rows, const void* q_scale,
                    const void* k_scale, float eps, cudaStream_t stream) {
  if (rows == 0 || heads == 0) return 0;
  switch (dtype) {
    case W8A8_BF16:
      return launch_rope<__nv_bfloat16>(q, k, q_out, k_out, rows, heads, head_dim, ldq, ldk, ldqo,
                                        ldko, freqs, freq_rows, q_scale, k_scale, eps, stream);
    case W8A8_F16:
      return launch_rope<__half>(q, k, q_out, k_out, rows, heads, head_dim, ldq, ldk, ldqo, ldko,
                                 freqs, freq_rows, q_scale, k_scale, eps, stream);
    case W8A8_F32:
      return launch_rope<float>(q, k, q_out, k_out, rows, heads, head_dim, ldq, ldk, ldqo, ldko,
                                freqs, freq_rows, q_scale, k_scale, eps, stream);
    default: break;
  }
  set_error("unsupported dtype code %d", dtype);
  return W8A8_ERR_VALUE;
}

}  // namespace w8a8
