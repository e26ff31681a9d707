// MXFP8 quantiser: 32-element K blocks, e4m3 payload, e8m0 block scales in the
// cuBLAS blocked layout.  Replaces the reference's quantize_mxfp8
// (inference/src/eager.rs:176-225; KSRC backends/cuda/ops/quantize_mxfp8.cu:40-147;
// layout inference/src/block_scales.rs:4-31) with the eager numerics:
//   need = max(amax / 448, 2^-127)            (fp32 IEEE divide)
//   e    = clamp(ceil(log2(need)) + 127, 0, 254), 0 for an all-zero block
//   q    = e4m3(clamp(x / 2^(e-127), -448, 448))   (RNE, zero blocks -> 0)
// ceil(log2(need)) is taken from the bit pattern: the biased exponent, plus
// one when the significand is not exactly a power of two (for fp32
// subnormals: 0 at 2^-127, else 1).  The division by a power of two is exact,
// done as a multiply by 2^(127-e).
//
// One thread per (row, K block) of the padded scale grid
// [ceil(M/128)*128, ceil(K/128)*4]; threads outside the data write a zero
// scale byte (the blocked layout's padding) and nothing else.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cstdint>

#include "w8a8_internal.h"

namespace w8a8 {
namespace {

constexpr int kMxThreads = 256;

template <typename T>
struct MxIn;
template <>
struct MxIn<__nv_bfloat16> {
  static constexpr int kVecs = 4;  // 32 elements = 4 x 16 B
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
};
template <>
struct MxIn<__half> {
  static constexpr int kVecs = 4;
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};
template <>
struct MxIn<float> {
  static constexpr int kVecs = 8;
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};

// Byte offset of scale (row, kb) in the blocked layout with `ncb` 4-wide
// column blocks: block (row/128, kb/4) is 512 contiguous bytes, inside it
// byte (row%32)*16 + ((row%128)/32)*4 + kb%4 (inference/src/block_scales.rs:4-31).
__device__ __forceinline__ int64_t blocked_offset(int row, int kb, int ncb) {
  const int64_t blk = static_cast<int64_t>(row >> 7) * ncb + (kb >> 2);
  return blk * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (kb & 3);
}

__device__ __forceinline__ uint32_t e8m0_of(float need) {
  const uint32_t u = __float_as_uint(need);  // need >= 2^-127 > 0
  const uint32_t exp = u >> 23;
  const uint32_t man = u & 0x7FFFFFu;
  int e;
  if (exp == 0) {
    e = (man == 0x400000u) ? 0 : 1;  // subnormal: exactly 2^-127 -> 0, else ceil -> -126
  } else {
    e = static_cast<int>(exp) + (man != 0 ? 1 : 0);
  }
  return static_cast<uint32_t>(min(254, max(0, e)));
}

template <typename T>
__global__ void __launch_bounds__(kMxThreads) quantize_mxfp8_kernel(
    const T* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
    uint8_t* __restrict__ sf, int rows, int cols, int rows_pad, int ncb) {
  const int kb_pad = ncb * 4;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * kMxThreads + threadIdx.x;
  if (idx >= static_cast<int64_t>(rows_pad) * kb_pad) return;
  const int row = static_cast<int>(idx / kb_pad);
  const int kb = static_cast<int>(idx - static_cast<int64_t>(row) * kb_pad);
  const int nkb = cols / 32;
  if (row >= rows || kb >= nkb) {
    sf[blocked_offset(row, kb, ncb)] = 0;
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * ldx + kb * 32);
  float f[32];
  constexpr int kPer = 32 / MxIn<T>::kVecs;
#pragma unroll
  for (int i = 0; i < MxIn<T>::kVecs; ++i) MxIn<T>::unpack(__ldg(src + i), f + i * kPer);
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(f[j]));
  uint32_t e = 0;
  float mul = 0.0f;  // zero blocks: payload 0
  if (amax != 0.0f) {
    const float need = fmaxf(__fdiv_rn(amax, 448.0f), 0x1.0p-127f);
    e = e8m0_of(need);
    // 2^(127 - e) for e in [0, 254]: an exact power of two (normal for e >= 1,
    // 2^127 for e = 0)
    mul = __uint_as_float(static_cast<uint32_t>(254 - static_cast<int>(e)) << 23);
    if (e == 254) mul = 0x1.0p-127f;
  }
  uint32_t out[8];
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    float v[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] = fminf(448.0f, fmaxf(-448.0f, __fmul_rn(f[j + t], mul)));
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[0], v[1]), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(v[2], v[3]), __NV_SATFINITE, __NV_E4M3);
    out[j / 4] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  uint4* dst = reinterpret_cast<uint4*>(q + static_cast<int64_t>(row) * ldq + kb * 32);
  dst[0] = make_uint4(out[0], out[1], out[2], out[3]);
  dst[1] = make_uint4(out[4], out[5], out[6], out[7]);
  sf[blocked_offset(row, kb, ncb)] = static_cast<uint8_t>(e);
}

template <typename T>
int launch_mx(const void* x, int64_t ldx, uint8_t* q, int64_t ldq, uint8_t* sf, int64_t rows,
              int64_t cols, cudaStream_t stream) {
  const int rows_pad = static_cast<int>((rows + 127) / 128 * 128);
  const int ncb = static_cast<int>((cols / 32 + 3) / 4);
  const int64_t total = static_cast<int64_t>(rows_pad) * ncb * 4;
  const int grid = static_cast<int>((total + kMxThreads - 1) / kMxThreads);
  quantize_mxfp8_kernel<T><<<grid, kMxThreads, 0, stream>>>(
      static_cast<const T*>(x), ldx, q, ldq, sf, static_cast<int>(rows), static_cast<int>(cols),
      rows_pad, ncb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("mxfp8 quantiser launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

}  // namespace

int quantize_mxfp8_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                          uint8_t* q, int64_t ldq, uint8_t* sf, cudaStream_t stream) {
  switch (x_dtype) {
    case W8A8_BF16: return launch_mx<__nv_bfloat16>(x, ldx, q, ldq, sf, rows, cols, stream);
    case W8A8_F16: return launch_mx<__half>(x, ldx, q, ldq, sf, rows, cols, stream);
    case W8A8_F32: return launch_mx<float>(x, ldx, q, ldq, sf, rows, cols, stream);
    default: break;
  }
  set_error("unsupported input dtype code %d", x_dtype);
  return W8A8_ERR_VALUE;
}

}  // namespace w8a8
