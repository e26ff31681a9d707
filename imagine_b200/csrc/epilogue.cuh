// Dequantisation epilogue shared by the tcgen05 GEMM, the GEMV and the
// stand-alone dequant kernel.  The arithmetic of each order is spelled with
// explicit-rounding intrinsics (__fmul_rn/__fmaf_rn/__fadd_rn) so that the
// compiler cannot re-associate or contract it differently from the reference.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace w8a8 {

// Dequant orders found in the reference (see oracle/eager.py):
//   kDqEager        inference/src/int8_linear.rs:244-268
//                   y = T(acc * (xs*ws)); y = T(y + bias)         (two roundings)
//   kDqScaleProduct KSRC backends/triton/quantization.py:861-1018
//                   y = T(fma(acc, xs*ws, bias))                  (one rounding)
//   kDqChained      native/comfy-port/kitchen/int8_linear.cu:669-708 (two-row GEMV)
//                   y = T(fma(acc*xs, ws, bias))                  (one rounding)
//   kDqSeparate     native/comfy-port/kitchen/int8_linear.cu:518-543, 586-667
//                   (stand-alone dequant with a bias, one-row GEMV: the bias
//                   added in a statement of its own, so not contracted)
//                   y = T((acc*xs)*ws + bias)                     (three fp32 roundings)
//                   CUDA-core paths only (dequant_one); the tensor-core GEMM
//                   epilogues take orders 0-2.
enum DequantOrder : int { kDqEager = 0, kDqScaleProduct = 1, kDqChained = 2, kDqSeparate = 3 };
// kActRmsRope: per-head RMSNorm + interleaved RoPE of 128-column heads (the
// QKV projection's epilogue; GEMM with 256-column tiles and bf16 output only)
enum OutputAct : int { kActNone = 0, kActGeluTanh = 1, kActRmsRope = 2 };

// Ranks of a fused column-parallel all-gather (one GPU each, one NVLink domain;
// W8A8_MAX_RANKS of the public header).
constexpr int kMaxRanks = 8;

template <typename T>
struct OutTraits;
template <>
struct OutTraits<float> {
  static __device__ __forceinline__ float round(float v) { return v; }
  static __device__ __forceinline__ float load(const void* p, int64_t i) {
    return static_cast<const float*>(p)[i];
  }
};
template <>
struct OutTraits<__nv_bfloat16> {
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
  static __device__ __forceinline__ float load(const void* p, int64_t i) {
    return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  }
};
template <>
struct OutTraits<__half> {
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ float load(const void* p, int64_t i) {
    return __half2float(static_cast<const __half*>(p)[i]);
  }
};

// GELU with the tanh approximation, evaluated in fp32 on a value already
// rounded to the output dtype (the reference applies gelu to the stored
// tensor).  tanh comes from the hardware approximation instruction.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.0f + tanh_fast(inner));
}

struct EpilogueParams {
  const float* xs;         // [M] per-row activation scales (int8 path)
  const float* ws;         // [N] per-channel weight scales, or [1]
  int ws_scalar;           // 1 if ws has one element
  const float* sa;         // fp8 path: per-tensor activation scale (device scalar)
  const float* sb;         // fp8 path: per-tensor weight scale (device scalar)
  const void* bias;        // [N] in the output dtype, or nullptr
  const void* residual;    // [M, ldr] in the output dtype, or nullptr
  int64_t ldr;             // residual row stride (elements)
  const void* rscale;      // [N] in the output dtype (required with residual), or
                           // [ceil(M / rscale_rows), N] when rscale_rows > 0
  int64_t rscale_rows;     // output rows per rscale row (0: one row for all)
  int64_t ld_rscale;       // rscale row stride (elements): N
  int dq_order;            // DequantOrder
  int act;                 // OutputAct
  int vec_ws;              // 1 if ws is 16-byte aligned (vector loads allowed)
  int vec_bias;            // 1 if bias is 16-byte aligned
  int vec_rscale;          // 1 if rscale is 16-byte aligned
  int vec_resid;           // 1 if residual rows are 16-byte aligned (base and ldr)
  const uint8_t* sfa;      // MXFP8: e8m0 scales of A, blocked layout
  const uint8_t* sfb;      // MXFP8: e8m0 scales of B, blocked layout
  int sf_ncb;              // MXFP8: 4-wide column blocks per scale row = ceil(K / 128)
  int b_tiles_kb;          // B pre-tiled (0: row-major): 128 x 128-byte tiles, this many
                           // K-blocks per 128-row block
  // kActRmsRope: columns [0, rope_cols) are 128-column heads that get
  // RMSNorm (weight rope_w: [128] shared, or [rope_cols] per column when
  // rope_w_percol) and the interleaved rotation of their row (rope_f: the
  // row-blocked float4 rotations, [row / 32][pair][row % 32]); later columns
  // get the plain epilogue.
  const void* rope_w;
  int rope_w_percol;
  const float* rope_f;
  int rope_cols;
  float rope_eps;
  // Column-parallel all-gather fused into the epilogue (n_ranks > 1): every
  // finished 32 x 32 output chunk, as staged (swizzled rows), is also copied
  // whole into slot `chunk` of this rank's region of each peer's receive
  // buffer (peer_recv[r] + (rank * chunks + chunk) * chunk bytes, chunk =
  // (row0 / 32) * chunk_cols + col0 / 32); the last CTA to finish then writes
  // `epoch` into slot `rank` of every peer's flag array (peer_flags[r]).
  // cta_count: this rank's CTA arrival counter.
  int n_ranks;
  int rank;
  uint8_t* peer_recv[kMaxRanks];
  unsigned* peer_flags[kMaxRanks];
  int64_t chunks;      // chunks of one shard: ceil(M / 32) * chunk_cols
  int chunk_cols;      // ceil(N_shard / 32)
  unsigned* cta_count;
  unsigned epoch;
  // Row-parallel reduce-scatter (int32 output, rs_rows > 0): rank p owns
  // output rows [p * rs_rows, (p + 1) * rs_rows); every finished int32
  // partial chunk goes whole, as staged, to its owner's receive buffer at
  // slot (rank * rs_rows / 32 + (row0 - owner * rs_rows) / 32) * chunk_cols +
  // col0 / 32 (this rank's own chunks included), instead of an output store.
  int64_t rs_rows;
};

// Value of one output element before the optional residual, already rounded
// to OutT's precision (returned as float).  `a` is the accumulator as fp32
// (int32 converted with round-to-nearest, or the fp8 path's fp32 sum).
template <typename OutT>
__device__ __forceinline__ float dequant_one(float a, float xs_row, float ws_col, float bias_col,
                                             bool has_bias, int order) {
  float y;
  if (order == kDqEager) {
    y = OutTraits<OutT>::round(__fmul_rn(a, __fmul_rn(xs_row, ws_col)));
    if (has_bias) y = OutTraits<OutT>::round(__fadd_rn(y, bias_col));
  } else if (order == kDqScaleProduct) {
    const float s = __fmul_rn(xs_row, ws_col);
    y = OutTraits<OutT>::round(has_bias ? __fmaf_rn(a, s, bias_col) : __fmul_rn(a, s));
  } else if (order == kDqSeparate) {
    const float t = __fmul_rn(__fmul_rn(a, xs_row), ws_col);
    y = OutTraits<OutT>::round(has_bias ? __fadd_rn(t, bias_col) : t);
  } else {
    const float t = __fmul_rn(a, xs_row);
    y = OutTraits<OutT>::round(has_bias ? __fmaf_rn(t, ws_col, bias_col) : __fmul_rn(t, ws_col));
  }
  return y;
}

// Element offset of output row m's residual-scale row (the per-sample gate).
__device__ __forceinline__ int64_t rscale_row(const EpilogueParams& ep, int64_t m) {
  return ep.rscale_rows > 0 ? (m / ep.rscale_rows) * ep.ld_rscale : 0;
}

template <typename OutT>
__device__ __forceinline__ float finish_one(float y, float resid, float rs, bool has_resid, int act) {
  if (act == kActGeluTanh) y = OutTraits<OutT>::round(gelu_tanh(y));
  if (has_resid) y = OutTraits<OutT>::round(__fmaf_rn(y, rs, resid));
  return y;
}

// The whole epilogue of one element from its int32 accumulator (the CUDA-core
// paths: GEMV, stand-alone dequant, the row-parallel reduce-scatter finish).
template <typename OutT>
__device__ __forceinline__ float epi_value(int32_t acc, int64_t m, int n, float xs,
                                           const EpilogueParams& ep) {
  const bool has_bias = ep.bias != nullptr;
  const float b = has_bias ? OutTraits<OutT>::load(ep.bias, n) : 0.0f;
  const float ws = __ldg(ep.ws + (ep.ws_scalar ? 0 : n));
  float y = dequant_one<OutT>(static_cast<float>(acc), xs, ws, b, has_bias, ep.dq_order);
  const bool has_resid = ep.residual != nullptr;
  const float res = has_resid ? OutTraits<OutT>::load(ep.residual, m * ep.ldr + n) : 0.0f;
  const float rs = has_resid ? OutTraits<OutT>::load(ep.rscale, rscale_row(ep, m) + n) : 0.0f;
  return finish_one<OutT>(y, res, rs, has_resid, ep.act);
}

}  // namespace w8a8
