// Persistent, warp-specialised tcgen05 GEMM for the W8A8 / FP8 linear family.
//
// Replaces the reference's CUTLASS 2.x Sm80 INT8 GEMM with EVT dequant
// epilogue (KSRC backends/cuda/ops/cutlass_gemm_int8.cu:66-420), its cuBLASLt
// int32 GEMM + separate dequant pass (KSRC backends/cuda/ops/cublas_gemm_int8.cu,
// native/comfy-port/kitchen/int8_linear.cu:517-583) and the cuBLASLt
// per-tensor FP8 `_scaled_mm` (inference/native/bridge.cpp:401-413).
//
// Structure (one CTA per SM, 192 threads):
//   warp 4      TMA producer: A[128 x 128B] and B[BN x 128B] K-slices into a
//               kStages-deep shared-memory ring (128B swizzle), one mbarrier
//               pair (full/empty) per stage.
//   warp 5      TMEM owner + MMA issuer: one elected thread issues
//               tcgen05.mma (kind::i8 -> s32, or kind::f8f6f4 -> f32),
//               128 x BN x 32 per instruction, into one of two TMEM
//               accumulators (2 x BN columns), and tcgen05.commit's the stage
//               back to the producer / the accumulator to the epilogue.
//   warps 0-3   epilogue: tcgen05.ld 32 lanes x 32 columns, dequant
//               (three reference orders), bias, GELU-tanh, residual, convert,
//               write a swizzled 32x32 staging tile, TMA store.  The double
//               buffered accumulator lets tile i's epilogue overlap tile i+1's
//               main loop.
// Tiles are visited persistently (tile = blockIdx.x + i * gridDim.x) in
// grouped-M order so concurrently running CTAs share A and B panels in L2.
//
// Every mbarrier wait is bounded (sm100_ptx.cuh); on a timeout the kernel
// records an error in g_w8a8_device_error, every role falls through, and TMEM
// is released.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <type_traits>

#include "epilogue.cuh"
#include "quant_common.cuh"
#include "sm100_ptx.cuh"
#include "w8a8_internal.h"

namespace w8a8 {

__device__ int g_w8a8_device_error;

int read_and_clear_device_error(cudaStream_t stream, int* value) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_w8a8_device_error, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_w8a8_device_error, &zero, sizeof(int), 0,
                                cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  *value = v;
  return 0;
}

namespace {

constexpr int kBM = 128;          // rows per tile (TMEM lanes)
constexpr int kBK = 128;          // K bytes per pipeline stage (one 128B swizzle row)
constexpr int kUmmaK = 32;        // K per tcgen05.mma for 8-bit operand kinds
constexpr int kEpiWarps = 8;   // two per TMEM lane quadrant, splitting the columns
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;
constexpr int kThreads = (kEpiWarps + 2) * 32;
constexpr int kMaxSmem = 232448;  // 227 KB opt-in per CTA on sm_100

template <int BN, typename OutT, int CG = 1, int KIND = 0, bool SPLIT = false>
struct Cfg {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = (BN / CG) * kBK;  // each CTA of a pair holds half of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  // MXFP8: one 512-byte block of e8m0 scales for A and BN/128 for B per
  // stage, the slot rounded up to 1024 bytes so that the staging tiles after
  // the scale slots keep the 1024-byte alignment their TMA swizzle needs
  static constexpr int kSFLoadBytes = KIND == 2 ? 512 * (1 + BN / 128) : 0;  // bytes the TMA brings
  static constexpr int kSFBytes = (kSFLoadBytes + 1023) / 1024 * 1024;          // slot size
  static constexpr int kSFCols = KIND == 2 ? 4 * (1 + BN / 128) : 0;  // TMEM columns per stage
  // one warp's staging tile (split-K stages its int32 partials in 32 x 16
  // halves, which fit the 2-byte outputs' tile)
  static constexpr int kStageD = 32 * 32 * static_cast<int>(sizeof(OutT));
  // per epilogue warp: one store staging tile + the fp32 weight scale and bias
  // of each of its column chunks for the current tile (four: its half of a
  // 256-column tile, or one 128-column head with kActRmsRope)
  static constexpr int kChunksPerWarp = 4;
  static constexpr int kVecBytes = 2 * kChunksPerWarp * 32 * 4;
  static constexpr int kDBytes = kEpiWarps * (kStageD + kVecBytes);
  static_assert(kStageD % 1024 == 0, "staging tiles must keep 1024-byte alignment");
  static constexpr int kBarBytes = 256;
  static constexpr int kFixed = 1024 + kDBytes + kBarBytes;
  static constexpr int kStagesRaw = (kMaxSmem - kFixed) / (kStageBytes + kSFBytes);
  static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
  static constexpr int kSmemBytes = kFixed + kStages * (kStageBytes + kSFBytes);
  // TMEM accumulators: two of BN columns (the epilogue of one tile overlaps
  // the MMAs of the next), except MXFP8 at 256 columns, where two would leave
  // no columns for the scale factors: there three 128-column regions, even
  // tiles in regions 0-1 (columns 0-255), odd tiles in regions 1-2 (columns
  // 128-383), so every tile is one N = 256 MMA per K step.  Each region goes
  // back to the MMA warp as soon as the epilogue has copied it to registers,
  // the shared region 1 first, so the next tile starts once the half of this
  // one in region 1 is drained.
  static constexpr bool kRegions3 = KIND == 2 && BN == 256;
  static constexpr int kAccCols = kRegions3 ? 3 * 128 : 2 * BN;
  static constexpr int kSFCol0 = kAccCols;  // scale factors live after the accumulators
  static constexpr uint32_t kTmemCols =
      (kAccCols + kStages * kSFCols <= 256) ? 256u : 512u;
  static_assert(kAccCols + kStages * kSFCols <= 512, "TMEM budget exceeded");
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kSmemBytes <= kMaxSmem, "shared memory budget exceeded");
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& mb,
                                            int& nb) {
  const int per_group = group_m * num_n;
  const int g = tile / per_group;
  const int first_m = g * group_m;
  const int gsize = min(num_m - first_m, group_m);
  const int r = tile - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// 32 consecutive per-column values starting at col0 as fp32.  Every lane of a
// warp reads the same addresses (broadcast); vector loads when the whole
// chunk is in range and the base is 16-byte aligned.
template <typename T>
__device__ __forceinline__ void load_cols32(const void* p, int col0, int N, bool vec_ok,
                                            float (&v)[32]) {
  if (vec_ok && col0 + 32 <= N) {
    if constexpr (sizeof(T) == 4) {
      const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 t = __ldg(q + i);
        v[4 * i] = t.x;
        v[4 * i + 1] = t.y;
        v[4 * i + 2] = t.z;
        v[4 * i + 3] = t.w;
      }
    } else {
      const uint4* q = reinterpret_cast<const uint4*>(static_cast<const T*>(p) + col0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 t = __ldg(q + i);
        const T* e = reinterpret_cast<const T*>(&t);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * i + j] = OutTraits<T>::load(e, j);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = col0 + j < N ? OutTraits<T>::load(p, col0 + j) : 0.0f;
  }
}

// The residual scales of this lane's row for columns col0..+31: the shared
// [N] row (the same addresses for every lane) or, with a per-sample gate, the
// row of the lane's sample (lanes of one sample read the same addresses).
template <typename T>
__device__ __forceinline__ void load_rscale32(const EpilogueParams& ep, int grow, int M, int col0,
                                              int N, float (&v)[32]) {
  const int64_t off = rscale_row(ep, min(grow, M - 1));
  const bool vec = ep.vec_rscale && (off * static_cast<int64_t>(sizeof(T))) % 16 == 0;
  load_cols32<T>(static_cast<const T*>(ep.rscale) + off, col0, N, vec, v);
}

__device__ __forceinline__ void spin_ns(uint64_t ns) {
  const uint64_t t0 = globaltimer_ns();
  while (globaltimer_ns() - t0 < ns) {
  }
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Output rounding to OutT's precision (value kept as fp32).  bf16 uses the
// exact integer round-to-nearest-even (ALU instead of the XU pipe).
template <typename OutT>
__device__ __forceinline__ float round_out(float v) {
  if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
    return round_bf16_alu(v);
  } else {
    return OutTraits<OutT>::round(v);
  }
}

// One output element of the fused epilogue, with the dequant order (ORDER)
// and the output activation (ACT) fixed at compile time.  Returns the value
// rounded to OutT before the optional residual.
template <typename OutT, int ORDER, int ACT>
__device__ __forceinline__ float epi_elem(float a, float xs_row, float ws_col, float bias_col,
                                          bool has_bias) {
  float y;
  if constexpr (ORDER == kDqEager) {
    y = round_out<OutT>(__fmul_rn(a, __fmul_rn(xs_row, ws_col)));
    if (has_bias) y = round_out<OutT>(__fadd_rn(y, bias_col));
  } else if constexpr (ORDER == kDqScaleProduct) {
    const float sc = __fmul_rn(xs_row, ws_col);
    y = round_out<OutT>(has_bias ? __fmaf_rn(a, sc, bias_col) : __fmul_rn(a, sc));
  } else {
    const float t = __fmul_rn(a, xs_row);
    y = round_out<OutT>(has_bias ? __fmaf_rn(t, ws_col, bias_col) : __fmul_rn(t, ws_col));
  }
  if constexpr (ACT == kActGeluTanh) y = round_out<OutT>(gelu_tanh(y));
  return y;
}

// Two adjacent output elements; for bf16 every rounding step rounds the pair
// with one cvt.rn.bf16x2.f32 (same RNE result as two scalar conversions).
__device__ __forceinline__ void round2_bf16(float& a, float& b) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  const uint32_t u = *reinterpret_cast<const uint32_t*>(&p);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xFFFF0000u);
}

template <typename OutT>
__device__ __forceinline__ void round2_out(float& a, float& b) {
  if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
    round2_bf16(a, b);
  } else {
    a = OutTraits<OutT>::round(a);
    b = OutTraits<OutT>::round(b);
  }
}

template <typename OutT, int ORDER, int ACT>
__device__ __forceinline__ void epi_pair(float a0, float a1, float xs_row, float w0, float w1,
                                         float b0, float b1, bool has_bias, float& y0, float& y1) {
  if constexpr (ORDER == kDqEager) {
    y0 = __fmul_rn(a0, __fmul_rn(xs_row, w0));
    y1 = __fmul_rn(a1, __fmul_rn(xs_row, w1));
    round2_out<OutT>(y0, y1);
    if (has_bias) {
      y0 = __fadd_rn(y0, b0);
      y1 = __fadd_rn(y1, b1);
      round2_out<OutT>(y0, y1);
    }
  } else if constexpr (ORDER == kDqScaleProduct) {
    const float s0 = __fmul_rn(xs_row, w0), s1 = __fmul_rn(xs_row, w1);
    y0 = has_bias ? __fmaf_rn(a0, s0, b0) : __fmul_rn(a0, s0);
    y1 = has_bias ? __fmaf_rn(a1, s1, b1) : __fmul_rn(a1, s1);
    round2_out<OutT>(y0, y1);
  } else {
    const float t0 = __fmul_rn(a0, xs_row), t1 = __fmul_rn(a1, xs_row);
    y0 = has_bias ? __fmaf_rn(t0, w0, b0) : __fmul_rn(t0, w0);
    y1 = has_bias ? __fmaf_rn(t1, w1, b1) : __fmul_rn(t1, w1);
    round2_out<OutT>(y0, y1);
  }
  if constexpr (ACT == kActGeluTanh) {
    y0 = gelu_tanh(y0);
    y1 = gelu_tanh(y1);
    round2_out<OutT>(y0, y1);
  }
}

// ---- bf16 output on packed fp32 pairs: the dequant order's arithmetic and
// the GELU on two adjacent elements per f32x2 instruction (each lane rounds
// as the scalar form does), the final cvt.rn.bf16x2 word being what the
// staging tile stores.
__device__ __forceinline__ uint32_t cvt_bf16x2(uint64_t v) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi(v)), "f"(lo(v)));
  return d;
}

__device__ __forceinline__ uint64_t unpack_bf16x2(uint32_t b) {
  return pk(__uint_as_float(b << 16), __uint_as_float(b & 0xFFFF0000u));
}

template <int ORDER, int ACT>
__device__ __forceinline__ uint32_t epi_pair_bf16x2(float a0, float a1, uint64_t xs2, float w0,
                                                    float w1, float b0, float b1, bool has_bias) {
  const uint64_t a = pk(a0, a1);
  const uint64_t w = pk(w0, w1);
  uint32_t bits;
  if constexpr (ORDER == kDqEager) {
    bits = cvt_bf16x2(mul2(a, mul2(xs2, w)));  // T(acc * (xs * ws))
    if (has_bias) bits = cvt_bf16x2(add2(unpack_bf16x2(bits), pk(b0, b1)));
  } else if constexpr (ORDER == kDqScaleProduct) {
    const uint64_t sc = mul2(xs2, w);
    bits = cvt_bf16x2(has_bias ? fma2(a, sc, pk(b0, b1)) : mul2(a, sc));
  } else {
    const uint64_t t = mul2(a, xs2);
    bits = cvt_bf16x2(has_bias ? fma2(t, w, pk(b0, b1)) : mul2(t, w));
  }
  if constexpr (ACT == kActGeluTanh) {
    // 0.5 x (1 + tanh(k0 (x + k1 x^3))) in gelu_tanh's operation order
    const uint64_t x = unpack_bf16x2(bits);
    const uint64_t p = mul2(mul2(pk(0.044715f, 0.044715f), x), x);
    const uint64_t u = fma2(p, x, x);
    const uint64_t in = mul2(pk(0.7978845608028654f, 0.7978845608028654f), u);
    const uint64_t t = pk(tanh_fast(lo(in)), tanh_fast(hi(in)));
    const uint64_t h = mul2(pk(0.5f, 0.5f), x);
    bits = cvt_bf16x2(mul2(h, add2(pk(1.0f, 1.0f), t)));
  }
  return bits;
}

// How the tiles are divided into units of work.
// Split-K (splits > 1): every tile is cut into `splits` units of consecutive
// K-blocks, run by different CTAs.  Scratch: the int32 partial sums of tile t
// at rows t * 128 .. +127 of a [tiles * 128, BN] array, then one arrival
// counter per (tile, epilogue warp); both all-zero between calls.
// Otherwise tiles from `half_from` on run as two units of 128 columns each:
// the last, partial wave of 256-column tiles spread over twice as many SMs.
struct SplitArgs {
  int32_t* acc;
  unsigned* cnt;
  int splits;
  int half_from;
};

struct Unit {
  int tile;
  int kb_lo, kb_hi;  // K-block range
  int col_off;       // first column within the tile
  int width;         // columns: BN, or 128 for a half-width unit
};

template <int BN>
__device__ __forceinline__ Unit unit_of(int unit, int S, int half_from, int num_kb) {
  Unit u;
  u.col_off = 0;
  u.width = BN;
  u.kb_lo = 0;
  u.kb_hi = num_kb;
  if (S > 1) {
    u.tile = unit / S;
    const int sp = unit - u.tile * S;
    u.kb_lo = sp * num_kb / S;
    u.kb_hi = (sp + 1) * num_kb / S;
  } else if (unit < half_from) {
    u.tile = unit;
  } else {
    const int v = unit - half_from;
    u.tile = half_from + (v >> 1);
    u.col_off = (v & 1) * 128;
    u.width = 128;
  }
  return u;
}

// Dequant epilogue of one 32 x 32 chunk (lane = row) from its raw 32-bit
// accumulators, staged in `st` and TMA-stored to (col0, row0) of the output.
template <int KIND, typename OutT, int ORDER, int ACT>
__device__ __forceinline__ void finish_chunk(const uint32_t (&cur)[32], const float* wsv,
                                             const float* bv, float xs_row, bool has_bias,
                                             bool has_resid, const EpilogueParams& ep, int grow,
                                             int col0, int row0, int M, int N, uint8_t* st,
                                             const CUtensorMap* tmD, int lane) {
  constexpr bool kRaw = std::is_same<OutT, int32_t>::value;
  constexpr bool kBf16 = std::is_same<OutT, __nv_bfloat16>::value;
  float y[32];
  uint32_t packed[16];  // bf16 output: the staged words
  if constexpr (kBf16) {
    const float4* wsq = reinterpret_cast<const float4*>(wsv);
    const float4* bq = reinterpret_cast<const float4*>(bv);
    const uint64_t xs2 = pk(xs_row, xs_row);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      const float4 w4 = wsq[j4];
      const float4 b4 = bq[j4];
      const int j = j4 * 4;
      float a[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        a[t] = (KIND == 0) ? static_cast<float>(static_cast<int32_t>(cur[j + t]))
                           : __uint_as_float(cur[j + t]);
      }
      constexpr int kOrder = KIND == 0 ? ORDER : kDqChained;
      packed[2 * j4] = epi_pair_bf16x2<kOrder, ACT>(a[0], a[1], xs2, w4.x, w4.y, b4.x, b4.y, has_bias);
      packed[2 * j4 + 1] =
          epi_pair_bf16x2<kOrder, ACT>(a[2], a[3], xs2, w4.z, w4.w, b4.z, b4.w, has_bias);
    }
    if (has_resid) {
      float rsv[32];
      load_rscale32<OutT>(ep, grow, M, col0, N, rsv);
      // the lane's 32 residual values as bf16 pairs: four 16-byte loads of
      // its row when the rows are aligned and the chunk is whole, element
      // loads otherwise
      uint32_t rw[16];
      if (ep.vec_resid && grow < M && col0 + 32 <= N) {
        const uint4* src = reinterpret_cast<const uint4*>(
            static_cast<const __nv_bfloat16*>(ep.residual) + static_cast<int64_t>(grow) * ep.ldr +
            col0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = __ldg(src + q);
          rw[4 * q] = v.x;
          rw[4 * q + 1] = v.y;
          rw[4 * q + 2] = v.z;
          rw[4 * q + 3] = v.w;
        }
      } else {
        const uint16_t* rrow = static_cast<const uint16_t*>(ep.residual) +
                               static_cast<int64_t>(min(grow, M - 1)) * ep.ldr;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const uint32_t lo = (grow < M && col0 + j < N) ? rrow[col0 + j] : 0u;
          const uint32_t hi = (grow < M && col0 + j + 1 < N) ? rrow[col0 + j + 1] : 0u;
          rw[j / 2] = lo | (hi << 16);
        }
      }
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const uint32_t bits = packed[j / 2];
        float v0 = __uint_as_float(bits << 16), v1 = __uint_as_float(bits & 0xFFFF0000u);
        const float r0 = __uint_as_float(rw[j / 2] << 16);
        const float r1 = __uint_as_float(rw[j / 2] & 0xFFFF0000u);
        v0 = __fmaf_rn(v0, rsv[j], r0);
        v1 = __fmaf_rn(v1, rsv[j + 1], r1);
        packed[j / 2] = cvt_bf16x2(pk(v0, v1));
      }
    }
  } else if constexpr (!kRaw) {
    const float4* wsq = reinterpret_cast<const float4*>(wsv);
    const float4* bq = reinterpret_cast<const float4*>(bv);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      const float4 w4 = wsq[j4];
      const float4 b4 = bq[j4];
      const int j = j4 * 4;
      float a[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        a[t] = (KIND == 0) ? static_cast<float>(static_cast<int32_t>(cur[j + t]))
                           : __uint_as_float(cur[j + t]);
      }
      epi_pair<OutT, (KIND == 0 ? ORDER : kDqChained), ACT>(
          a[0], a[1], xs_row, w4.x, w4.y, b4.x, b4.y, has_bias, y[j], y[j + 1]);
      epi_pair<OutT, (KIND == 0 ? ORDER : kDqChained), ACT>(
          a[2], a[3], xs_row, w4.z, w4.w, b4.z, b4.w, has_bias, y[j + 2], y[j + 3]);
    }
    if (has_resid) {
      float rsv[32];
      load_rscale32<OutT>(ep, grow, M, col0, N, rsv);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float res = (grow < M && col0 + j < N)
                              ? OutTraits<OutT>::load(ep.residual,
                                                      static_cast<int64_t>(grow) * ep.ldr + col0 + j)
                              : 0.0f;
        y[j] = round_out<OutT>(__fmaf_rn(y[j], rsv[j], res));
      }
    }
  }
  // single staging tile: the previous chunk's store was issued a whole chunk
  // of arithmetic ago
  if (lane == 0) tma_store_wait_read<0>();
  __syncwarp();
  if constexpr (sizeof(OutT) == 4) {
    // 32 x 4-byte values = 8 chunks of 16 B; 128B swizzle: chunk ^= row & 7.
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      uint4 v;
      if constexpr (kRaw) {
        v = make_uint4(cur[cc * 4], cur[cc * 4 + 1], cur[cc * 4 + 2], cur[cc * 4 + 3]);
      } else {
        v = make_uint4(__float_as_uint(y[cc * 4]), __float_as_uint(y[cc * 4 + 1]),
                       __float_as_uint(y[cc * 4 + 2]), __float_as_uint(y[cc * 4 + 3]));
      }
      const int phys = cc ^ (lane & 7);
      *reinterpret_cast<uint4*>(st + lane * 128 + phys * 16) = v;
    }
  } else {
    // 32 x 2-byte values = 4 chunks of 16 B; 64B swizzle: chunk ^= (row >> 1) & 3.
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      uint32_t w4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if constexpr (kBf16) {
          w4[e] = packed[cc * 4 + e];
        } else {
          w4[e] = pack2<OutT>(y[cc * 8 + e * 2], y[cc * 8 + e * 2 + 1]);
        }
      }
      const int phys = cc ^ ((lane >> 1) & 3);
      *reinterpret_cast<uint4*>(st + lane * 64 + phys * 16) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && row0 < M) {
    if (kRaw && ep.rs_rows > 0) {
      // row-parallel reduce-scatter: the int32 partial chunk to its owner
      const int owner = static_cast<int>(row0 / ep.rs_rows);
      const int64_t slot =
          (static_cast<int64_t>(ep.rank) * (ep.rs_rows >> 5) + ((row0 - owner * ep.rs_rows) >> 5)) *
              ep.chunk_cols + (col0 >> 5);
      bulk_store(ep.peer_recv[owner] + slot * (32 * 32 * 4), st, 32 * 32 * 4);
    } else {
      tma_store_2d(tmD, st, col0, row0);
    }
    if constexpr (!kRaw) {
      // fused all-gather: the staged chunk, whole and contiguous, into this
      // rank's region of every peer's receive buffer
      if (ep.n_ranks > 1) {
        constexpr uint32_t kChunkBytes = 32 * 32 * sizeof(OutT);
        const int64_t slot = static_cast<int64_t>(ep.rank) * ep.chunks +
                             static_cast<int64_t>(row0 >> 5) * ep.chunk_cols + (col0 >> 5);
        for (int p = 0; p < ep.n_ranks; ++p) {
          if (p != ep.rank) bulk_store(ep.peer_recv[p] + slot * kChunkBytes, st, kChunkBytes);
        }
      }
    }
    tma_store_commit();
  }
}

// 16 packed bf16 words (a lane's 32 columns) into the 64B-swizzled staging
// tile, then the chunk's TMA store to (col0, row0).
__device__ __forceinline__ void store_chunk_bf16(const uint32_t (&w)[16], uint8_t* st,
                                                 const CUtensorMap* tmD, int col0, int row0, int M,
                                                 int lane) {
  if (lane == 0) tma_store_wait_read<0>();
  __syncwarp();
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    const int phys = cc ^ ((lane >> 1) & 3);
    *reinterpret_cast<uint4*>(st + lane * 64 + phys * 16) =
        make_uint4(w[cc * 4], w[cc * 4 + 1], w[cc * 4 + 2], w[cc * 4 + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && row0 < M) {
    tma_store_2d(tmD, st, col0, row0);
    tma_store_commit();
  }
}

// ---- kActRmsRope: Q/K RMSNorm + interleaved RoPE fused into the projection
// (the stand-alone form is rope.cu; reference call site
// inference/src/models/qwen_image21/dit.rs:486-505, eager body
// inference/src/backend_rope.rs:146-223).  An epilogue warp owns one whole
// 128-column head of its 32 rows, one row per lane, so the row's statistics
// need no cross-lane reduction.  Both passes fetch the head's four raw
// accumulator chunks (from TMEM, or from the split-K scratch) and turn them
// into exactly the bf16 words the plain GEMM would store: pass 1 sums their
// squares, pass 2 normalises, rotates and stores them.  Fetching twice keeps
// the head out of the registers, which the rotation's loads need.
//
// The 32 bf16 words of one chunk from its raw accumulators.
template <int ORDER>
__device__ __forceinline__ void rope_dequant_chunk(const uint32_t (&cur)[32], const float* wsv,
                                                   const float* bv, uint64_t xs2, bool has_bias,
                                                   uint32_t (&w)[16]) {
  const float4* wsq = reinterpret_cast<const float4*>(wsv);
  const float4* bq = reinterpret_cast<const float4*>(bv);
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    const float4 w4 = wsq[j4];
    const float4 b4 = bq[j4];
    const int j = j4 * 4;
    const float a0 = static_cast<float>(static_cast<int32_t>(cur[j]));
    const float a1 = static_cast<float>(static_cast<int32_t>(cur[j + 1]));
    const float a2 = static_cast<float>(static_cast<int32_t>(cur[j + 2]));
    const float a3 = static_cast<float>(static_cast<int32_t>(cur[j + 3]));
    w[2 * j4] = epi_pair_bf16x2<ORDER, kActNone>(a0, a1, xs2, w4.x, w4.y, b4.x, b4.y, has_bias);
    w[2 * j4 + 1] = epi_pair_bf16x2<ORDER, kActNone>(a2, a3, xs2, w4.z, w4.w, b4.z, b4.w, has_bias);
  }
}

// fetch(i, cur, second): chunk i's raw accumulators of this lane's row (the
// second fetch of a chunk may release its storage).  wsv / bv: the head's
// per-column weight scales and bias, [4][32] fp32.
//   rrms = 1 / sqrt(sum(x^2) / 128 + eps); n = bf16(x * rrms * w);
//   (y0, y1) = (f00 n0 + f01 n1, f10 n0 + f11 n1); out = bf16(y)
// with f the token's 2 x 2 rotation of each pair.
template <int ORDER, typename Fetch>
__device__ __forceinline__ void rope_head(Fetch&& fetch, const float* wsv, const float* bv,
                                          float xs_row, bool has_bias, const EpilogueParams& ep,
                                          int grow, int hcol0, int row0, int M, uint8_t* st,
                                          const CUtensorMap* tmD, int lane) {
  const uint64_t xs2 = pk(xs_row, xs_row);
  uint64_t ss2 = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t cur[32], w[16];
    fetch(i, cur, false);
    rope_dequant_chunk<ORDER>(cur, wsv + i * 32, bv + i * 32, xs2, has_bias, w);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint64_t v = unpack_bf16x2(w[j]);
      ss2 = fma2(v, v, ss2);
    }
  }
  const float ss = __fadd_rn(lo(ss2), hi(ss2));
  // 1 / sqrt in two IEEE roundings, the form torch's rsqrt takes
  const float rrms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / 128.0f), ep.rope_eps)));
  const uint64_t rr2 = pk(rrms, rrms);
  // this row's rotations: pair p at fr[p * 32] (row-blocked, 128-row padded,
  // so every row of a tile has them); a warp's 32 rows read 512 contiguous bytes
  const float4* fr = reinterpret_cast<const float4*>(ep.rope_f) +
                     (static_cast<int64_t>(grow >> 5) * 64) * 32 + (grow & 31);
  const uint4* nw4 = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(ep.rope_w) +
                                                    (ep.rope_w_percol ? hcol0 : 0));
  // Groups of 4 pairs (one 16-byte word of 8 norm weights, four rotations);
  // the next group's loads are issued before this group's arithmetic, so
  // their L2 latency overlaps the work instead of adding up over the 64 pairs.
  float4 fc[4], fn[4];
  uint4 wc = __ldg(nw4), wn = wc;
#pragma unroll
  for (int e = 0; e < 4; ++e) fc[e] = __ldg(fr + e * 32);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t cur[32], w[16], out[16];
    fetch(i, cur, true);
    rope_dequant_chunk<ORDER>(cur, wsv + i * 32, bv + i * 32, xs2, has_bias, w);
#pragma unroll
    for (int g4 = 0; g4 < 4; ++g4) {
      const int gi = i * 4 + g4;  // group of the head
      if (gi + 1 < 16) {
        wn = __ldg(nw4 + gi + 1);  // same address for every lane
#pragma unroll
        for (int e = 0; e < 4; ++e) fn[e] = __ldg(fr + (4 * (gi + 1) + e) * 32);
      }
      const uint32_t ww[4] = {wc.x, wc.y, wc.z, wc.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t nb =
            cvt_bf16x2(mul2(mul2(unpack_bf16x2(w[g4 * 4 + e]), rr2), unpack_bf16x2(ww[e])));
        const float n0 = __uint_as_float(nb << 16);
        const float n1 = __uint_as_float(nb & 0xFFFF0000u);
        const float4 f = fc[e];  // (f00, f01, f10, f11)
        out[g4 * 4 + e] =
            cvt_bf16x2(fma2(pk(f.y, f.w), pk(n1, n1), mul2(pk(f.x, f.z), pk(n0, n0))));
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) fc[e] = fn[e];
      wc = wn;
    }
    store_chunk_bf16(out, st, tmD, hcol0 + i * 32, row0, M, lane);
  }
}

// This unit's int32 partial chunk (32 rows x 32 columns, lane = row) +=
// the scratch at (scol, srow): two 32 x 16 TMA reductions through the warp's
// 64B-swizzled staging tile.
__device__ __forceinline__ void splitk_reduce_chunk(const CUtensorMap* tmW, uint8_t* st,
                                                    const uint32_t (&cur)[32], int scol, int srow,
                                                    int lane) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (lane == 0) tma_store_wait_read<0>();
    __syncwarp();
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const int j = h * 16 + cc * 4;
      *reinterpret_cast<uint4*>(st + lane * 64 + ((cc ^ ((lane >> 1) & 3)) * 16)) =
          make_uint4(cur[j], cur[j + 1], cur[j + 2], cur[j + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_reduce_add_2d(tmW, st, scol + h * 16, srow);
      tma_store_commit();
    }
  }
}

// Split-K read-back: the summed int32 chunk at scratch row srow, columns
// scol..+31 (row length BN) into cur, leaving zeros behind for the next call
// (unless !zero: the chunk is read again).  Rows of a tile past M hold zeros
// and are skipped.
template <int BN>
__device__ __forceinline__ void splitk_take_chunk(const SplitArgs& sk, int srow, int scol,
                                                  bool row_in, uint32_t (&cur)[32],
                                                  bool zero = true) {
  if (!row_in) {
#pragma unroll
    for (int j = 0; j < 32; ++j) cur[j] = 0u;
    return;
  }
  int4* s4 = reinterpret_cast<int4*>(sk.acc + static_cast<int64_t>(srow) * BN + scol);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int4 v = __ldcg(s4 + i);
    cur[4 * i] = static_cast<uint32_t>(v.x);
    cur[4 * i + 1] = static_cast<uint32_t>(v.y);
    cur[4 * i + 2] = static_cast<uint32_t>(v.z);
    cur[4 * i + 3] = static_cast<uint32_t>(v.w);
  }
  if (zero) {
#pragma unroll
    for (int i = 0; i < 8; ++i) __stcg(s4 + i, make_int4(0, 0, 0, 0));
  }
}

// CG = 1: one CTA computes a 128 x BN tile.  CG = 2: a cluster of two CTAs
// computes a 256 x BN tile with 2-SM MMAs (the leader, cluster rank 0,
// issues them); each CTA loads its own 128 rows of A and BN/2 rows of B and
// drains its own 128 x BN accumulator.
//
// SPLIT: the K range of every tile is cut into sk.splits units run by
// different CTAs.  Each unit TMA-reduce-adds its int32 partial tile into the
// sk.acc scratch (exact and order-independent); epilogue warp e of each unit
// then counts itself in at sk.cnt[tile * 8 + e], and the last of the splits to
// arrive reads the summed chunks back, applies the epilogue, and returns the
// chunks and its counter to zero.  Results equal the unsplit GEMM's bit for
// bit.
//
// Half-width units (tiles from sk.half_from on, CG = 1, BN = 256, no split-K)
// load 128 rows of B through tmBh and issue N = 128 MMAs into the first 128
// columns of the accumulator.
//
// KIND 2 (MXFP8) with CG = 2 (BN = 128: 256 x 128 pair tiles, each CTA two
// 128-column accumulators plus its scale blocks in TMEM): tmBh and tmW, unused
// by that kind, are the scale-factor maps of A and B.
template <int KIND, int BN, typename OutT, int ORDER, int ACT, int CG, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmD,
                      const __grid_constant__ CUtensorMap tmW, int M, int N, int K, int num_m_tiles,
                      int num_n_tiles, int group_m, EpilogueParams ep, SplitArgs sk) {
  using C = Cfg<BN, OutT, CG, KIND, SPLIT>;
  static_assert(!SPLIT || (CG == 1 && KIND == 0), "split-K is built for the 1-CTA int8 GEMM");
  static_assert(KIND != 2 || CG == 1 || BN == 128, "MXFP8 pairs run 256 x 128 tiles");
  constexpr bool kRaw = std::is_same<OutT, int32_t>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::kStages * C::kABytes;
  uint8_t* sSF = smem + C::kStages * C::kStageBytes;  // MXFP8 scale blocks (KIND 2)
  uint8_t* sD = sSF + C::kStages * C::kSFBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sD + C::kDBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;  // two accumulators, or three regions (kRegions3)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 3);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  volatile int* abortv = abort_flag;

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_tiles = num_m_tiles * num_n_tiles;
  const int num_kb = (K + kBK - 1) / kBK;
  const int S = SPLIT ? sk.splits : 1;  // K splits per tile
  // tiles run as two half-width units (only 1-CTA 256-column tiles)
  const int half_from = (!SPLIT && CG == 1 && BN == 256) ? sk.half_from : num_tiles;
  const int num_units = S > 1 ? num_tiles * S : half_from + 2 * (num_tiles - half_from);
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int first_tile = static_cast<int>(blockIdx.x) / CG;
  const int tile_step = static_cast<int>(gridDim.x) / CG;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&tfull[b], 1);
    for (int b = 0; b < 3; ++b) {
      mbar_init(&tempty[b], kEpiWarps * CG);  // one arrival per epilogue warp of each CTA
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (half_from < num_tiles || (KIND == 2 && CG == 2)) tma_prefetch_desc(&tmBh);
    if constexpr (!kRaw) tma_prefetch_desc(&tmD);
    if constexpr (SPLIT || (KIND == 2 && CG == 2)) tma_prefetch_desc(&tmW);
  }
  if (warp == kMmaWarp) {
    tmem_alloc<C::kTmemCols, CG>(tmem_slot);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // the peer's barriers exist before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above overlapped the tail of the kernel that wrote A and the
  // row scales (launched with programmatic stream serialization); nothing
  // below runs before that kernel has completed.
  griddep_wait();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int unit = first_tile; ok && unit < num_units; unit += tile_step) {
        const Unit u = unit_of<BN>(unit, S, half_from, num_kb);
        int mb, nb;
        tile_coords(u.tile, num_m_tiles, num_n_tiles, group_m, mb, nb);
        const int a_row = mb * kBM * CG + static_cast<int>(rank) * kBM;
        const int b_row = nb * BN + u.col_off + static_cast<int>(rank) * (BN / CG);
        const bool half_unit = u.width < BN;
        for (int kb = u.kb_lo; kb < u.kb_hi; ++kb, ++it) {
          const int s = static_cast<int>(it % C::kStages);
          const uint32_t ph = (it / C::kStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, abortv, &g_w8a8_device_error, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          if constexpr (CG == 1) {
            mbar_arrive_expect_tx(&full[s], C::kABytes + (half_unit ? C::kBBytes / 2 : C::kBBytes) +
                                                C::kSFLoadBytes);
            tma_load_2d(sA + s * C::kABytes, &tmA, &full[s], kb * kBK, a_row);
            if (half_unit) {
              tma_load_2d(sB + s * C::kBBytes, &tmBh, &full[s], kb * kBK, b_row);
            } else if (ep.b_tiles_kb) {
              // pre-tiled B (128-column tiles): tile (nb, kb) is 16 KB contiguous
              tma_load_2d(sB + s * C::kBBytes, &tmB, &full[s], 0, (nb * ep.b_tiles_kb + kb) * 128);
            } else {
              tma_load_2d(sB + s * C::kBBytes, &tmB, &full[s], kb * kBK, b_row);
            }
            if constexpr (KIND == 2) {
              // blocked scale layout: 512-byte block (row/128, kb) at
              // ((row/128) * ncb + kb) * 512; blocks outside the buffers the
              // caller sized from M, N, K are refused (error 5, abort).  A
              // 256-column tile whose second half lies wholly past N (no
              // block of B there) reads the last block again: those columns
              // are computed but never stored.
              uint8_t* sf = sSF + s * C::kSFBytes;
              const int a_blocks = (M + 127) / 128, b_blocks = (N + 127) / 128;
              const bool in = mb < a_blocks && kb < ep.sf_ncb && nb * (BN / 128) < b_blocks;
              if (!in) {
                atomicCAS(&g_w8a8_device_error, 0, kDevBadScaleBlock);
                *abort_flag = 1;
                ok = false;
                break;
              }
              bulk_load(sf, ep.sfa + (static_cast<int64_t>(mb) * ep.sf_ncb + kb) * 512, 512,
                        &full[s]);
#pragma unroll
              for (int j = 0; j < BN / 128; ++j) {
                const int blk = min(nb * (BN / 128) + j, b_blocks - 1);
                bulk_load(sf + 512 * (1 + j),
                          ep.sfb + (static_cast<int64_t>(blk) * ep.sf_ncb + kb) * 512,
                          512, &full[s]);
              }
            }
          } else {
            // both CTAs' bytes are counted on the leader's barrier
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * (C::kStageBytes + C::kSFLoadBytes));
            const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
            tma_load_2d_pair(sA + s * C::kABytes, &tmA, bar, kb * kBK, a_row);
            tma_load_2d_pair(sB + s * C::kBBytes, &tmB, bar, kb * kBK, b_row);
            if constexpr (KIND == 2) {
              // scale blocks as two 256-byte rows of the [blocks * 2, 256]
              // maps (tmBh: A, tmW: B): this CTA's 128-row block of A and
              // the tile's 128-column block of B; blocks past the buffers'
              // ends read as zeros (rows past M / N, never stored)
              uint8_t* sf = sSF + s * C::kSFBytes;
              const int a_blk = mb * CG + static_cast<int>(rank);
              tma_load_2d_pair(sf, &tmBh, bar, 0, (a_blk * ep.sf_ncb + kb) * 2);
              tma_load_2d_pair(sf + 512, &tmW, bar, 0, (nb * ep.sf_ncb + kb) * 2);
            }
          }
        }
      }
      if (!ok) spin_ns(1000000);  // let TMA loads already in flight land (bounded)
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc<KIND == 0 ? 0 : 1>(kBM * CG, BN);
      constexpr uint32_t idesc_half = make_idesc<KIND == 0 ? 0 : 1>(kBM, 128);
      uint32_t it = 0;
      uint32_t tl = 0;
      bool ok = true;
      for (int unit = first_tile; ok && unit < num_units; unit += tile_step, ++tl) {
        const Unit u = unit_of<BN>(unit, S, half_from, num_kb);
        const int kb_lo = u.kb_lo, kb_hi = u.kb_hi;
        const uint32_t id = u.width < BN ? idesc_half : idesc;
        (void)id;
        const uint32_t acc = tl & 1u;
        const uint32_t use = tl >> 1;
        // regions of this tile (kRegions3): region 1 (its tl-th use) and
        // region 0 (even tiles) or 2 (odd tiles), each that region's
        // (tl / 2)-th use; a use needs the previous one drained
        const uint32_t r_other = (tl & 1u) ? 2u : 0u;
        if constexpr (C::kRegions3) {
          if (!mbar_wait(&tempty[1], (tl & 1u) ^ 1u, abortv, &g_w8a8_device_error,
                         kDevTimeoutTmemEmpty) ||
              !mbar_wait(&tempty[r_other], ((tl >> 1) & 1u) ^ 1u, abortv, &g_w8a8_device_error,
                         kDevTimeoutTmemEmpty)) {
            break;
          }
        } else {
          if (!mbar_wait(&tempty[acc], (use & 1u) ^ 1u, abortv, &g_w8a8_device_error,
                         kDevTimeoutTmemEmpty)) {
            break;
          }
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (C::kRegions3 ? 128u * (tl & 1u) : acc * BN);
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const int s = static_cast<int>(it % C::kStages);
          const uint32_t ph = (it / C::kStages) & 1u;
          if (!mbar_wait(&full[s], ph, abortv, &g_w8a8_device_error, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * C::kABytes);
          const uint32_t b0 = smem_u32(sB + s * C::kBBytes);
          if constexpr (KIND == 2) {
            // scale blocks of this stage -> this stage's TMEM slot, then the
            // four K=32 MMAs each pick their K sub-block with sf_id
            const uint32_t sf_tmem = tmem_base + C::kSFCol0 + s * C::kSFCols;
            const uint32_t sf_smem = smem_u32(sSF + s * C::kSFBytes);
            tmem_cp_32x128b_x4<CG>(sf_tmem, smem_desc_sf(sf_smem));
#pragma unroll
            for (int j = 0; j < BN / 128; ++j) {
              tmem_cp_32x128b_x4<CG>(sf_tmem + 4 * (1 + j), smem_desc_sf(sf_smem + 512 * (1 + j)));
            }
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              umma_mx<CG>(d_tmem, smem_desc_k_sw128(a0 + k * kUmmaK),
                          smem_desc_k_sw128(b0 + k * kUmmaK),
                          make_idesc_mx(kBM * CG, BN, static_cast<uint32_t>(k)), sf_tmem,
                          sf_tmem + 4, (kb != kb_lo || k != 0) ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              const uint64_t ad = smem_desc_k_sw128(a0 + k * kUmmaK);
              const uint64_t bd = smem_desc_k_sw128(b0 + k * kUmmaK);
              const uint32_t accumulate = (kb != kb_lo || k != 0) ? 1u : 0u;
              if constexpr (CG == 1) {
                umma_ss<KIND>(d_tmem, ad, bd, id, accumulate);
              } else {
                umma_ss_pair<KIND>(d_tmem, ad, bd, idesc, accumulate);
              }
            }
          }
          if constexpr (CG == 1) {
            umma_commit(&empty[s]);
          } else {
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
          }
        }
        if (ok) {
          if constexpr (CG == 1) {
            umma_commit(&tfull[acc]);
          } else {
            umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Warp e owns TMEM lane quadrant e % 4 (rows 32q..32q+31 of the tile) and
    // the 32-column chunks c with c % 2 == e / 4.
    const int quad = warp & 3;
    const int half = warp >> 2;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    // staging tiles first (each a multiple of 1024 B, as the TMA swizzle
    // needs), then the per-warp vectors
    uint8_t* st = sD + warp * C::kStageD;
    float* s_ws = reinterpret_cast<float*>(sD + kEpiWarps * C::kStageD + warp * C::kVecBytes);
    float* s_bias = s_ws + C::kChunksPerWarp * 32;  // [chunk][32] each
    const bool has_bias = ep.bias != nullptr;
    const bool has_resid = ep.residual != nullptr;
    constexpr bool kRope = ACT == kActRmsRope;
    static_assert(!kRope || (KIND == 0 && CG == 1 && std::is_same<OutT, __nv_bfloat16>::value),
                  "the RMSNorm + RoPE epilogue is built for the 1-CTA int8 GEMM with bf16 output");
    float fp8_scale = 0.0f;
    if constexpr (KIND == 1) fp8_scale = __fmul_rn(__ldg(ep.sa), __ldg(ep.sb));
    (void)fp8_scale;
    uint32_t tl = 0;
    for (int unit = first_tile; unit < num_units; unit += tile_step, ++tl) {
      const Unit u = unit_of<BN>(unit, S, half_from, num_kb);
      const int tile = u.tile;
      int mb, nb;
      tile_coords(tile, num_m_tiles, num_n_tiles, group_m, mb, nb);
      const uint32_t acc = tl & 1u;
      const uint32_t use = tl >> 1;
      const int col_base = nb * BN + u.col_off;
      const int nch = u.width / 32;  // 32-column chunks of this unit
      if constexpr (!kRaw) {
        // Stage this warp's per-column weight scales and bias while the MMA
        // is still running: lane j loads column j of each of the warp's chunks.
        // (The previous tile's readers of these slots are this warp's own
        // lanes, all past their last read.)
        __syncwarp();
#pragma unroll
        for (int i = 0; i < C::kChunksPerWarp; ++i) {
          const int ch = kRope ? 4 * half + i : half + 2 * i;  // chunk of the tile
          const int col = col_base + ch * 32 + lane;
          const bool in = ch < nch && col < N;
          float wv = 1.0f, bvv = 0.0f;
          if constexpr (KIND == 0) wv = in ? __ldg(ep.ws + (ep.ws_scalar ? 0 : col)) : 0.0f;
          if (has_bias && in) bvv = OutTraits<OutT>::load(ep.bias, col);
          s_ws[i * 32 + lane] = wv;
          s_bias[i * 32 + lane] = bvv;
        }
        __syncwarp();
      }
      if (has_resid && !SPLIT) {
        // The residual rows of this unit into L2 while the MMA still runs:
        // the epilogue's residual loads then find them there (measured on
        // 11200 x 3072 -> 3072 with the residual read from HBM in the
        // epilogue: 204 us against 80 us without a residual).  Lane = row of
        // the quadrant; the quadrant's two warps take alternate 128-byte
        // lines of the row.
        const int prow = mb * kBM * CG + static_cast<int>(rank) * kBM + quad * 32 + lane;
        if (prow < M && col_base < N) {
          const int bytes = min(u.width, N - col_base) * static_cast<int>(sizeof(OutT));
          const char* rrow = static_cast<const char*>(ep.residual) +
                             (static_cast<int64_t>(prow) * ep.ldr + col_base) *
                                 static_cast<int64_t>(sizeof(OutT));
          for (int off = half * 128; off < bytes; off += 256) prefetch_l2_line(rrow + off);
        }
      }
      if (!mbar_wait(&tfull[acc], use & 1u, abortv, &g_w8a8_device_error, kDevTimeoutTmemFull)) {
        break;
      }
      tc_fence_after();
      const int row0 = mb * kBM * CG + static_cast<int>(rank) * kBM + quad * 32;
      const int grow = row0 + lane;
      // split-K: this warp's first scratch row; partials are added to the
      // scratch instead of finishing the chunks
      const int srow0 = tile * kBM + quad * 32;
      constexpr bool do_reduce = SPLIT;
      float xs_row = 0.0f;
      if constexpr (KIND == 0 && !kRaw) xs_row = grow < M ? __ldg(ep.xs + grow) : 0.0f;
      if constexpr (KIND == 1) xs_row = fp8_scale;
      if constexpr (KIND == 2) xs_row = 1.0f;  // block scales are applied by the MMA
      if constexpr (kRope) {
        // this warp's head: chunks 4 half .. 4 half + 3 of the tile
        const int hcol0 = col_base + half * 128;
        const bool active = half * 128 < u.width && hcol0 < N;
        const bool roped = active && hcol0 < ep.rope_cols;
        const uint32_t head_tmem = tmem_base + lane_base + acc * BN + half * 128;
        if (active) {
          if (do_reduce) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t cur[32];
              tmem_ld_32x32b_x32(head_tmem + i * 32, cur);
              tmem_ld_wait();
              if (row0 < M) splitk_reduce_chunk(&tmW, st, cur, half * 128 + i * 32, srow0, lane);
            }
          } else if (roped) {
            auto from_tmem = [&](int i, uint32_t (&cur)[32], bool) {
              tmem_ld_32x32b_x32(head_tmem + i * 32, cur);
              tmem_ld_wait();
            };
            rope_head<ORDER>(from_tmem, s_ws, s_bias, xs_row, has_bias, ep, grow, hcol0, row0, M,
                             st, &tmD, lane);
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t cur[32];
              tmem_ld_32x32b_x32(head_tmem + i * 32, cur);
              tmem_ld_wait();
              finish_chunk<KIND, OutT, ORDER, kActNone>(cur, s_ws + i * 32, s_bias + i * 32, xs_row,
                                                        has_bias, has_resid, ep, grow,
                                                        hcol0 + i * 32, row0, M, N, st, &tmD, lane);
            }
          }
        }
        // the accumulator is free: the MMA warp may start the next tile on it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (do_reduce) {
          unsigned last = 0;
          unsigned* cnt = sk.cnt + static_cast<int64_t>(tile) * kEpiWarps + warp;
          if (lane == 0) {
            tma_store_wait_all<0>();
            fence_proxy_async_global();
            __threadfence();
            last = atomicAdd(cnt, 1u) == static_cast<unsigned>(S - 1) ? 1u : 0u;
          }
          last = __shfl_sync(0xffffffffu, last, 0);
          if (last && active) {
            __threadfence();
            auto from_scratch = [&](int i, uint32_t (&cur)[32], bool second) {
              splitk_take_chunk<BN>(sk, srow0 + lane, half * 128 + i * 32, grow < M, cur, second);
            };
            if (roped) {
              rope_head<ORDER>(from_scratch, s_ws, s_bias, xs_row, has_bias, ep, grow, hcol0, row0,
                               M, st, &tmD, lane);
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                uint32_t cur[32];
                from_scratch(i, cur, true);
                finish_chunk<KIND, OutT, ORDER, kActNone>(cur, s_ws + i * 32, s_bias + i * 32,
                                                          xs_row, has_bias, has_resid, ep, grow,
                                                          hcol0 + i * 32, row0, M, N, st, &tmD, lane);
              }
            }
          }
          if (last && lane == 0) *cnt = 0u;
        }
        continue;
      }
      if constexpr (C::kRegions3) {
        // the tile's columns start at TMEM column 0 (even tiles) or 128 (odd
        // tiles); chunks 0-3 and 4-7 are its two 128-column regions.  Per
        // region, region 1 first: this warp's two chunks to registers, the
        // region back to the MMA warp, then their arithmetic
        static_assert(!SPLIT && CG == 1, "the shared-region layout is built for 1-CTA MXFP8");
        const uint32_t col0_tmem = 128u * (tl & 1u);
#pragma unroll
        for (int step = 0; step < 2; ++step) {
          // group of chunks (0: 0-3, 1: 4-7) in region 1 first
          const int grp = ((tl & 1u) ? 0 : 1) ^ step;
          const uint32_t region = (col0_tmem >> 7) + static_cast<uint32_t>(grp);
          uint32_t two[2][32];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int c = half + 2 * (2 * grp + i);
            if (c < nch && col_base + c * 32 < N) {
              tmem_ld_32x32b_x32(tmem_base + lane_base + col0_tmem + c * 32, two[i]);
            }
          }
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[region]);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int ci = 2 * grp + i;
            const int c = half + 2 * ci;
            const int col0 = col_base + c * 32;
            if (c < nch && col0 < N) {
              finish_chunk<KIND, OutT, ORDER, ACT>(two[i], s_ws + ci * 32, s_bias + ci * 32, xs_row,
                                                   has_bias, has_resid, ep, grow, col0, row0, M, N,
                                                   st, &tmD, lane);
            }
          }
        }
        continue;
      }
      // TMEM loads are software-pipelined: chunk c+2's tcgen05.ld is issued
      // as soon as chunk c's registers are free, so its latency overlaps the
      // arithmetic of chunk c.
      uint32_t r[32];
      if (half * 32 < u.width && col_base + half * 32 < N) {
        tmem_ld_32x32b_x32(tmem_base + lane_base + acc * BN + half * 32, r);
      }
      for (int c = half; c < nch; c += 2) {
        const int col0 = col_base + c * 32;
        if (col0 >= N) break;
        const int ci = (c - half) >> 1;  // this warp's chunk index
        tmem_ld_wait();
        uint32_t cur[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) cur[j] = r[j];
        if (c + 2 < nch && col0 + 64 < N) {
          tmem_ld_32x32b_x32(tmem_base + lane_base + acc * BN + (c + 2) * 32, r);
        }
        if (do_reduce) {
          // this unit's int32 partial -> += scratch (TMA reduction)
          if (row0 < M) splitk_reduce_chunk(&tmW, st, cur, c * 32, srow0, lane);
        } else {
          finish_chunk<KIND, OutT, ORDER, ACT>(cur, s_ws + ci * 32, s_bias + ci * 32, xs_row,
                                               has_bias, has_resid, ep, grow, col0, row0, M, N, st,
                                               &tmD, lane);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 1) {
          mbar_arrive(&tempty[acc]);
        } else {
          mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        }
      }
      if (do_reduce) {
        // Count this warp's chunks in; the last split to arrive finishes them.
        unsigned last = 0;
        unsigned* cnt = sk.cnt + static_cast<int64_t>(tile) * kEpiWarps + warp;
        if (lane == 0) {
          tma_store_wait_all<0>();      // this warp's reductions are complete
          fence_proxy_async_global();
          __threadfence();
          last = atomicAdd(cnt, 1u) == static_cast<unsigned>(S - 1) ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          for (int c = half; c < BN / 32; c += 2) {
            const int col0 = col_base + c * 32;
            if (col0 >= N) break;
            const int ci = (c - half) >> 1;
            uint32_t cur[32];
            splitk_take_chunk<BN>(sk, srow0 + lane, c * 32, grow < M, cur);
            finish_chunk<KIND, OutT, ORDER, ACT>(cur, s_ws + ci * 32, s_bias + ci * 32, xs_row,
                                                 has_bias, has_resid, ep, grow, col0, row0, M, N,
                                                 st, &tmD, lane);
          }
          if (lane == 0) *cnt = 0u;
        }
      }
    }
    if (lane == 0) tma_store_wait_all<0>();
    {
      if (ep.n_ranks > 1) {
        // Fused all-gather / reduce-scatter: this CTA's peer copies are
        // complete (each warp's bulk groups waited above) and published, then
        // it counts itself in; the last CTA of the grid writes this call's
        // epoch into slot `rank` of every peer's done flags.
        fence_proxy_async_global();
        __threadfence_system();
        named_bar_sync(1, kEpiWarps * 32);
        if (threadIdx.x == 0) {
          __threadfence_system();
          const unsigned prev = atomicAdd(ep.cta_count, 1u);
          if (prev == gridDim.x - 1) {
            __threadfence_system();
            for (int p = 0; p < ep.n_ranks; ++p) {
              if (p != ep.rank) st_release_sys(ep.peer_flags[p] + kMaxRanks + ep.rank, ep.epoch);
            }
            *ep.cta_count = 0u;  // every CTA of this call has arrived
          }
        }
      }
    }
  }

  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // the peer is done with its TMEM and our barriers
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc<C::kTmemCols, CG>(tmem_base);
  }
}

// ---------------------------------------------------------------- CUDA-core path
// For shapes the TMA path cannot address (K % 16 != 0, unaligned rows, K == 0).
// One thread per output element; the A row is broadcast across the block.
template <int KIND, typename OutT>
__global__ void __launch_bounds__(128) gemm_simt_kernel(const uint8_t* __restrict__ a, int64_t lda,
                                                        const uint8_t* __restrict__ b, int64_t ldb,
                                                        void* __restrict__ out, int64_t ldo, int M,
                                                        int N, int K, EpilogueParams ep) {
  constexpr bool kRaw = std::is_same<OutT, int32_t>::value;
  const int m = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const uint8_t* ar = a + static_cast<int64_t>(m) * lda;
  const uint8_t* br = b + static_cast<int64_t>(n) * ldb;
  float af = 0.0f;
  int32_t ai = 0;
  if constexpr (KIND == 2) {
    // per 32-element block: exact partial dot product times both block scales
    for (int kb = 0; kb < K / 32; ++kb) {
      float part = 0.0f;
      for (int k = kb * 32; k < kb * 32 + 32; ++k) {
        __nv_fp8_e4m3 x, y;
        x.__x = ar[k];
        y.__x = br[k];
        part = __fmaf_rn(static_cast<float>(x), static_cast<float>(y), part);
      }
      const auto sf = [&](const uint8_t* t, int row) {
        const int64_t blk = static_cast<int64_t>(row >> 7) * ep.sf_ncb + (kb >> 2);
        const uint32_t e = t[blk * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (kb & 3)];
        return e == 0 ? 0x1.0p-127f : __uint_as_float(e << 23);
      };
      af = __fmaf_rn(part, __fmul_rn(sf(ep.sfa, m), sf(ep.sfb, n)), af);
    }
  } else {
    for (int k = 0; k < K; ++k) {
      if constexpr (KIND == 0) {
        ai += static_cast<int32_t>(static_cast<int8_t>(ar[k])) *
              static_cast<int32_t>(static_cast<int8_t>(br[k]));
      } else {
        __nv_fp8_e4m3 x, y;
        x.__x = ar[k];
        y.__x = br[k];
        af = __fmaf_rn(static_cast<float>(x), static_cast<float>(y), af);
      }
    }
  }
  const int64_t o = static_cast<int64_t>(m) * ldo + n;
  if constexpr (kRaw) {
    static_cast<int32_t*>(out)[o] = ai;
  } else {
    const bool has_bias = ep.bias != nullptr;
    const float bias = has_bias ? OutTraits<OutT>::load(ep.bias, n) : 0.0f;
    float y;
    if constexpr (KIND == 0) {
      y = dequant_one<OutT>(static_cast<float>(ai), __ldg(ep.xs + m),
                            __ldg(ep.ws + (ep.ws_scalar ? 0 : n)), bias, has_bias, ep.dq_order);
    } else if constexpr (KIND == 1) {
      y = dequant_one<OutT>(af, __fmul_rn(__ldg(ep.sa), __ldg(ep.sb)), 1.0f, bias, has_bias,
                            kDqChained);
    } else {
      y = dequant_one<OutT>(af, 1.0f, 1.0f, bias, has_bias, kDqChained);
    }
    const bool has_resid = ep.residual != nullptr;
    const float res = has_resid ? OutTraits<OutT>::load(ep.residual, static_cast<int64_t>(m) * ep.ldr + n) : 0.0f;
    const float rs = has_resid ? OutTraits<OutT>::load(ep.rscale, rscale_row(ep, m) + n) : 0.0f;
    y = finish_one<OutT>(y, res, rs, has_resid, ep.act);
    if constexpr (std::is_same<OutT, float>::value) {
      static_cast<float*>(out)[o] = y;
    } else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
      static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(y);
    } else {
      static_cast<__half*>(out)[o] = __float2half_rn(y);
    }
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

bool make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* base,
                 uint64_t inner, uint64_t outer, uint64_t row_stride_elems, uint32_t box_inner,
                 uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

EpilogueParams to_params(const GemmArgs& g) {
  EpilogueParams ep{};
  ep.xs = g.xs;
  ep.sa = g.sa;
  ep.sb = g.sb;
  if (g.epi) {
    ep.ws = g.epi->ws;
    ep.ws_scalar = g.epi->ws_numel == 1 ? 1 : 0;
    ep.bias = g.epi->bias;
    ep.residual = g.epi->residual;
    ep.ldr = g.epi->ldr;
    ep.rscale = g.epi->residual_scale;
    ep.rscale_rows = g.epi->residual_scale_rows;
    ep.ld_rscale = g.N;
    ep.dq_order = g.epi->dequant_order;
    ep.act = g.epi->activation;
  }
  ep.sfa = static_cast<const uint8_t*>(g.sfa);
  ep.sfb = static_cast<const uint8_t*>(g.sfb);
  ep.sf_ncb = static_cast<int>((g.K + 127) / 128);
  ep.b_tiles_kb = g.b_tiled ? static_cast<int>((g.K + kBK - 1) / kBK) : 0;
  ep.n_ranks = g.ag_world > 1 ? g.ag_world : 1;
  if (ep.n_ranks > 1) {
    ep.rank = g.ag_rank;
    for (int r = 0; r < g.ag_world; ++r) {
      ep.peer_recv[r] = static_cast<uint8_t*>(g.ag_recv[r]);
      ep.peer_flags[r] = g.ag_flags[r];
    }
    ep.chunk_cols = static_cast<int>((g.N + 31) / 32);
    ep.chunks = (g.M + 31) / 32 * ep.chunk_cols;
    ep.cta_count = g.ag_flags[g.ag_rank] + 2 * kMaxRanks;
    ep.epoch = g.ag_epoch;
    ep.rs_rows = g.rs_rows;
  }
  if (g.rms_rope) {
    ep.act = kActRmsRope;
    ep.rope_w = g.rope_w;
    ep.rope_w_percol = g.rope_w_percol;
    ep.rope_f = g.rope_f;
    ep.rope_cols = static_cast<int>(g.rope_cols);
    ep.rope_eps = g.rope_eps;
  }
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  ep.vec_ws = ep.ws && a16(ep.ws);
  ep.vec_bias = ep.bias && a16(ep.bias);
  ep.vec_rscale = ep.rscale && a16(ep.rscale);
  const int out_bytes = g.out_dtype == W8A8_F32 || g.out_dtype == W8A8_S32 ? 4 : 2;
  ep.vec_resid = ep.residual && a16(ep.residual) && (ep.ldr * out_bytes) % 16 == 0;
  return ep;
}

// mw / sk: the split-K scratch map and pointers (SPLIT only; otherwise the
// output map stands in for the unused map parameter).
template <int KIND, int BN, typename OutT, int ORDER, int ACT, int CG, bool SPLIT = false>
int launch_tc(const GemmArgs& g, const CUtensorMap& ma, const CUtensorMap& mb,
              const CUtensorMap& mbh, const CUtensorMap& md, const CUtensorMap& mw, SplitArgs sk,
              int group_m, int max_ctas, cudaStream_t stream) {
  // The same configuration the kernel lays its shared memory out with: the
  // block-scaled kind adds scale-factor bytes to every stage.
  using C = Cfg<BN, OutT, CG, KIND, SPLIT>;
  auto kern = gemm_sm100_kernel<KIND, BN, OutT, ORDER, ACT, CG, SPLIT>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (e != cudaSuccess) {
      set_error("cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
      return W8A8_ERR_ACCELERATOR;
    }
    attr_set[dev] = true;
  }
  const int num_m = static_cast<int>((g.M + kBM * CG - 1) / (kBM * CG));
  const int num_n = static_cast<int>((g.N + BN - 1) / BN);
  const int tiles = num_m * num_n;
  const int sms = device_sm_count();
  if (!SPLIT) sk.splits = 1;
  if (SPLIT || CG != 1 || BN != 256 || KIND == 2 || sk.half_from > tiles) sk.half_from = tiles;
  const int64_t all_units = sk.splits > 1 ? static_cast<int64_t>(tiles) * sk.splits
                                          : sk.half_from + 2ll * (tiles - sk.half_from);
  int units = static_cast<int>(
      std::min<int64_t>(all_units, (max_ctas > 0 ? max_ctas : sms) / CG));  // CTAs or CTA pairs
  if (units < 1) units = 1;
  const EpilogueParams ep = to_params(g);
  const int Mi = static_cast<int>(g.M), Ni = static_cast<int>(g.N), Ki = static_cast<int>(g.K);
  // Programmatic stream serialization: the grid may launch while the kernel
  // before it (the quantiser, which triggers early) is still running; the
  // kernel waits for it (griddep_wait) before reading anything it wrote.
  cudaLaunchConfig_t lc{};
  lc.gridDim = dim3(static_cast<unsigned>(units * CG));
  lc.blockDim = dim3(kThreads);
  lc.dynamicSmemBytes = C::kSmemBytes;
  lc.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  if constexpr (CG == 2) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    lc.numAttrs = 2;
  }
  const cudaError_t e = cudaLaunchKernelEx(&lc, kern, ma, mb, mbh, md, mw, Mi, Ni, Ki, num_m,
                                           num_n, group_m, ep, sk);
  if (e != cudaSuccess) {
    set_error("tcgen05 GEMM launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

static_assert(kMaxRanks == W8A8_MAX_RANKS && 4 * kMaxRanks <= W8A8_PEER_FLAG_WORDS,
              "flag block layout");

struct PeerFlags {
  unsigned* flags[kMaxRanks];
};

// Flag block of a fused all-gather / reduce-scatter rank (uint32): [0, 8)
// ready slots, one per peer, [8, 16) done slots, [16] the rank's CTA arrival
// counter for the GEMM, [17] the one for the reduce-scatter finish, [24, 32)
// the finish's done slots.
//
// peer_barrier: every rank writes `epoch` into its slot of each peer's ready
// flags, then waits until all peers' slots of its own block hold it (no rank
// writes into another's output before all have finished reading the previous
// call's).  peer_done_wait: waits until every peer's GEMM has written `epoch`
// into the done slots.  Each wait gives up after kSpinLimitNs, records
// kDevTimeoutPeer and returns.
__global__ void __launch_bounds__(32) peer_flags_kernel(unsigned* mine, PeerFlags peers, int rank,
                                                        int world, unsigned epoch, int base,
                                                        int signal) {
  const int p = threadIdx.x;
  if (p >= world || p == rank) return;
  if (signal) st_release_sys(peers.flags[p] + base + rank, epoch);
  const uint64_t t0 = globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys(mine + base + p) - epoch) < 0) {
    if (globaltimer_ns() - t0 > kSpinLimitNs) {
      atomicCAS(&g_w8a8_device_error, 0, kDevTimeoutPeer);
      return;
    }
    __nanosleep(256);
  }
}

// The peers' chunks in this rank's receive buffer (each as its epilogue
// staged it: 32 rows of 32 * ESZ bytes in 16-byte pieces, swizzled like the
// staging tile) into the output at columns p * N_shard: one warp per chunk,
// lanes covering whole rows of it.
template <int ESZ>
__global__ void __launch_bounds__(256) allgather_unpack_kernel(
    const uint8_t* __restrict__ recv, uint8_t* __restrict__ out, int64_t ldo, int M, int N_shard,
    int rank, int world, int64_t chunks, int chunk_cols) {
  constexpr int kRowBytes = 32 * ESZ;
  constexpr int kPieces = kRowBytes / 16;
  constexpr int kRowsPerPass = 32 / kPieces;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (wid >= static_cast<int64_t>(world - 1) * chunks) return;
  int p = static_cast<int>(wid / chunks);
  if (p >= rank) ++p;  // the peers, skipping this rank
  const int64_t c = wid - static_cast<int64_t>(wid / chunks) * chunks;
  const int rb = static_cast<int>(c / chunk_cols);
  const int cb = static_cast<int>(c - static_cast<int64_t>(rb) * chunk_cols);
  const int piece = lane % kPieces;
  const int col = cb * 32 + piece * (16 / ESZ);  // shard column (N_shard % 8 == 0)
  if (col >= N_shard) return;
  const uint8_t* src = recv + (static_cast<int64_t>(p) * chunks + c) * 32 * kRowBytes;
#pragma unroll
  for (int pass = 0; pass < 32 / kRowsPerPass; ++pass) {
    const int r = pass * kRowsPerPass + lane / kPieces;
    const int row = rb * 32 + r;
    if (row >= M) break;
    const int phys = ESZ == 2 ? (piece ^ ((r >> 1) & 3)) : (piece ^ (r & 7));
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src + r * kRowBytes + phys * 16));
    *reinterpret_cast<uint4*>(
        out + (static_cast<int64_t>(row) * ldo + static_cast<int64_t>(p) * N_shard + col) * ESZ) = v;
  }
}

struct PeerBytes {
  uint8_t* p[kMaxRanks];
};

// Row-parallel reduce-scatter finish, one warp per (owned row, 512 columns):
// sum the int32 partial chunks the ranks sent for those columns (each chunk as its epilogue
// staged it: 32 rows of 128 bytes in 16-byte pieces, piece ^= row & 7),
// apply the dequant epilogue, stage 512 columns at a time in shared memory and
// write them as 16-byte pieces to this rank's output and to every peer's
// staging buffer ([M, N], same rows).  Then every CTA publishes and counts
// itself in at flags[rank][17]; the last one writes `epoch` into slot `rank`
// of every peer's finish-done flags [24, 32).
template <typename OutT>
__global__ void __launch_bounds__(256) rs_reduce_kernel(
    const uint8_t* __restrict__ recv, const float* __restrict__ xs, EpilogueParams ep,
    uint8_t* __restrict__ out, int64_t ldo, int M, int N, int64_t rs_rows, int chunk_cols,
    PeerBytes stages, PeerFlags flags, int rank, int world, unsigned epoch) {
  constexpr int kEsz = static_cast<int>(sizeof(OutT));
  constexpr int kSeg = 512;
  __shared__ __align__(16) uint8_t seg[8][kSeg * kEsz];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row_lo = static_cast<int64_t>(rank) * rs_rows;
  const int64_t nrows = (M < row_lo + rs_rows ? M : row_lo + rs_rows) - row_lo;
  const int64_t slot_rows = rs_rows >> 5;
  const int nseg = (N + kSeg - 1) / kSeg;
  // work item = (owned row, 512-column segment), one per warp; a lane's 16
  // columns of every sender are loaded back to back (32 loads in flight for
  // two ranks) before the epilogue runs on them
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * 8 + warp; item < nrows * nseg;
       item += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t lr = item / nseg;
    const int c0 = static_cast<int>(item - lr * nseg) * kSeg;
    const int cend = N < c0 + kSeg ? N : c0 + kSeg;
    const int64_t row = row_lo + lr;
    const int64_t rb = lr >> 5;
    const int r = static_cast<int>(lr & 31);
    const int in_row = r * 128 + ((((lane >> 2) ^ (r & 7)) << 4) | ((lane & 3) << 2));
    int32_t v[kSeg / 32];
#pragma unroll
    for (int i = 0; i < kSeg / 32; ++i) v[i] = 0;
    for (int s = 0; s < world; ++s) {
      // chunk (rb, c0 / 32 + i) of sender s, this lane's element of row r
      const uint8_t* base =
          recv + ((static_cast<int64_t>(s) * slot_rows + rb) * chunk_cols + (c0 >> 5)) * 4096 +
          in_row;
#pragma unroll
      for (int i = 0; i < kSeg / 32; ++i) {
        if (c0 + lane + 32 * i < cend) {
          v[i] += __ldcg(reinterpret_cast<const int32_t*>(base + static_cast<int64_t>(i) * 4096));
        }
      }
    }
    const float xsr = xs[row];
#pragma unroll
    for (int i = 0; i < kSeg / 32; ++i) {
      const int col = c0 + lane + 32 * i;
      if (col < cend) {
        const float y = epi_value<OutT>(v[i], row, col, xsr, ep);
        OutT* dst = reinterpret_cast<OutT*>(&seg[warp][(col - c0) * kEsz]);
        if constexpr (std::is_same<OutT, float>::value) {
          *dst = y;
        } else if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
          *dst = __float2bfloat16_rn(y);
        } else {
          *dst = __float2half_rn(y);
        }
      }
    }
    __syncwarp();
    const int bytes = (cend - c0) * kEsz;  // a multiple of 16 (N % 8 == 0)
    for (int o = lane * 16; o < bytes; o += 32 * 16) {
      const uint4 v4 = *reinterpret_cast<const uint4*>(&seg[warp][o]);
      *reinterpret_cast<uint4*>(out + (row * ldo + c0) * kEsz + o) = v4;
      for (int p = 0; p < world; ++p) {
        if (p != rank) {
          *reinterpret_cast<uint4*>(stages.p[p] + (row * N + c0) * kEsz + o) = v4;
        }
      }
    }
    __syncwarp();
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* cnt = flags.flags[rank] + 2 * kMaxRanks + 1;
    if (atomicAdd(cnt, 1u) == gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < world; ++p) {
        if (p != rank) st_release_sys(flags.flags[p] + 3 * kMaxRanks + rank, epoch);
      }
      *cnt = 0u;  // every CTA of this call has arrived
    }
  }
}

// After every peer's finish-done flag holds `epoch` (each CTA's thread 0
// waits, bounded: on expiry kDevTimeoutPeer and the CTA copies nothing), the
// rows the peers own go from this rank's staging buffer into its output.
template <int ESZ>
__global__ void __launch_bounds__(256) rs_gather_kernel(uint8_t* __restrict__ out, int64_t ldo,
                                                        int M, int N, int64_t rs_rows,
                                                        const uint8_t* __restrict__ stage,
                                                        unsigned* mine, int rank, int world,
                                                        unsigned epoch) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    ready = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < world && ready; ++p) {
      if (p == rank) continue;
      while (static_cast<int>(ld_acquire_sys(mine + 3 * kMaxRanks + p) - epoch) < 0) {
        if (globaltimer_ns() - t0 > kSpinLimitNs) {
          atomicCAS(&g_w8a8_device_error, 0, kDevTimeoutPeer);
          ready = 0;
          break;
        }
        __nanosleep(256);
      }
    }
  }
  __syncthreads();
  if (!ready) return;
  const int64_t pieces = static_cast<int64_t>(N) * ESZ / 16;  // per row
  const int64_t total = static_cast<int64_t>(M) * pieces;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / pieces;
    if (row / rs_rows == rank) continue;  // this rank's rows are in `out` already
    const int64_t pc = i - row * pieces;
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(stage + (row * N * ESZ) + pc * 16));
    *reinterpret_cast<uint4*>(out + row * ldo * ESZ + pc * 16) = v;
  }
}

template <int KIND, typename OutT>
int launch_simt(const GemmArgs& g, cudaStream_t stream) {
  if (g.M == 0 || g.N == 0) return 0;
  dim3 grid(static_cast<unsigned>((g.N + 127) / 128), static_cast<unsigned>(g.M));
  gemm_simt_kernel<KIND, OutT><<<grid, 128, 0, stream>>>(
      static_cast<const uint8_t*>(g.a), g.lda, static_cast<const uint8_t*>(g.b), g.ldb, g.out,
      g.ldo, static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(g.K), to_params(g));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("CUDA-core GEMM launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

template <int KIND, typename OutT>
int dispatch_out(const GemmArgs& g, bool tc_ok, const GemmPlan& plan, cudaStream_t stream) {
  if (!tc_ok) return launch_simt<KIND, OutT>(g, stream);
  const int bn = plan.bn, cg = plan.cg, group_m = plan.group_m, max_ctas = plan.max_ctas;
  const int splits = plan.splits;
  CUtensorMap ma, mb, mbh, md, mw;
  bool ok = make_map_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.a, g.K, g.M, g.lda, kBK, kBM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (g.b_tiled) {
    // [ceil(N/128) * ceil(K/128) * 128 rows, 128 bytes]
    const int64_t rows = (g.N + 127) / 128 * ((g.K + kBK - 1) / kBK) * 128;
    ok = ok && make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.b, kBK, rows, kBK, kBK, 128,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    ok = ok && make_map_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.b, g.K, g.N, g.ldb, kBK,
                           static_cast<uint32_t>(bn / cg), CU_TENSOR_MAP_SWIZZLE_128B);
  }
  CUtensorMapDataType dt;
  if constexpr (std::is_same<OutT, float>::value) dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  else if constexpr (std::is_same<OutT, int32_t>::value) dt = CU_TENSOR_MAP_DATA_TYPE_INT32;
  else if constexpr (std::is_same<OutT, __half>::value) dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  else dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  ok = ok && make_map_2d(&md, dt, static_cast<int>(sizeof(OutT)), g.out, g.N, g.M, g.ldo, 32, 32,
                         sizeof(OutT) == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  SplitArgs sk{nullptr, nullptr, 1, static_cast<int>(plan.half_from)};
  if (plan.half_from < plan.tiles) {
    // half-width units: 128-row boxes of B
    ok = ok && make_map_2d(&mbh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.b, g.K, g.N, g.ldb, kBK, 128,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    mbh = mb;
  }
  if (KIND == 2 && cg == 2) {
    // MXFP8 pairs: the blocked scales (512 bytes per 128-row block and 128
    // K elements) as [blocks * 2, 256] byte maps, one block per 256 x 2 box
    const int64_t ncb = (g.K + 127) / 128;
    const int64_t a_rows = (g.M + 127) / 128 * ncb * 2, b_rows = (g.N + 127) / 128 * ncb * 2;
    ok = ok && make_map_2d(&mbh, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.sfa, 256, a_rows, 256, 256, 2,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
    ok = ok && make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.sfb, 256, b_rows, 256, 256, 2,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
  } else if (splits > 1) {
    // int32 [tiles * 128, bn] partial sums, then the arrival counters;
    // reductions in 32-row x 16-column boxes
    sk.acc = static_cast<int32_t*>(g.workspace);
    sk.cnt = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(g.workspace) +
                                         splitk_acc_bytes(plan.split_tiles, bn));
    sk.splits = splits;
    ok = ok && make_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, g.workspace, bn,
                           plan.split_tiles * kBM, bn, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    mw = md;
  }
  if (!ok) {
    set_error("cuTensorMapEncodeTiled rejected the operands (M=%lld N=%lld K=%lld)",
              static_cast<long long>(g.M), static_cast<long long>(g.N), static_cast<long long>(g.K));
    return W8A8_ERR_RUNTIME;
  }
  auto by_bn = [&](auto order_c, auto act_c) {
    constexpr int O = decltype(order_c)::value;
    constexpr int A = decltype(act_c)::value;
    if constexpr (A == kActRmsRope) {
      // int8 with bf16 output only (checked by gemm_launch); one CTA per tile
      if constexpr (KIND == 0 && std::is_same<OutT, __nv_bfloat16>::value) {
        if (splits > 1) {  // split-K runs 128-column tiles
          return launch_tc<KIND, 128, OutT, O, A, 1, true>(g, ma, mb, mbh, md, mw, sk, group_m,
                                                           max_ctas, stream);
        }
        if (bn == 128) {
          return launch_tc<KIND, 128, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas, stream);
        }
        return launch_tc<KIND, 256, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas, stream);
      } else {
        set_error("the RMSNorm + RoPE epilogue needs int8 operands and bf16 output");
        return W8A8_ERR_VALUE;
      }
    } else if constexpr (KIND == 2) {
      if (cg == 2) {
        return launch_tc<KIND, 128, OutT, O, A, 2>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas,
                                                   stream);
      }
      if (bn == 128) {
        return launch_tc<KIND, 128, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas,
                                                   stream);
      }
      return launch_tc<KIND, 256, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas, stream);
    } else {
      if constexpr (KIND == 0 && !std::is_same<OutT, int32_t>::value) {
        if (splits > 1) {  // split-K runs 128-column tiles
          return launch_tc<KIND, 128, OutT, O, A, 1, true>(g, ma, mb, mbh, md, mw, sk, group_m,
                                                           max_ctas, stream);
        }
      }
      if constexpr (KIND == 0) {
        if (bn == 64) {
          return launch_tc<KIND, 64, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas,
                                                    stream);
        }
      }
      if (bn == 128) {
        return launch_tc<KIND, 128, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas, stream);
      }
      if (cg == 2) {
        return launch_tc<KIND, 256, OutT, O, A, 2>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas, stream);
      }
      return launch_tc<KIND, 256, OutT, O, A, 1>(g, ma, mb, mbh, md, mw, sk, group_m, max_ctas, stream);
    }
  };
  using I0 = std::integral_constant<int, 0>;
  using I1 = std::integral_constant<int, 1>;
  using I2 = std::integral_constant<int, 2>;
  if constexpr (std::is_same<OutT, int32_t>::value) {
    return by_bn(I0{}, I0{});
  } else {
    const int order = (KIND == 0 && g.epi) ? g.epi->dequant_order : kDqChained;
    const int act = g.epi ? g.epi->activation : kActNone;
    if (KIND != 0) {
      return act == kActGeluTanh ? by_bn(I2{}, I1{}) : by_bn(I2{}, I0{});
    }
    if constexpr (std::is_same<OutT, __nv_bfloat16>::value) {
      if (g.rms_rope) {
        switch (order) {
          case 0: return by_bn(I0{}, I2{});
          case 1: return by_bn(I1{}, I2{});
          default: return by_bn(I2{}, I2{});
        }
      }
    }
    switch (order * 2 + (act == kActGeluTanh ? 1 : 0)) {
      case 0: return by_bn(I0{}, I0{});
      case 1: return by_bn(I0{}, I1{});
      case 2: return by_bn(I1{}, I0{});
      case 3: return by_bn(I1{}, I1{});
      case 4: return by_bn(I2{}, I0{});
      default: return by_bn(I2{}, I1{});
    }
  }
}

}  // namespace

int64_t splitk_acc_bytes(int64_t split_tiles, int bn) {
  return split_tiles * kBM * bn * 4;  // a multiple of 256 bytes
}

int64_t splitk_workspace_bytes(int64_t M, int64_t N) {
  const int64_t tiles128 = ((M + kBM - 1) / kBM) * ((N + 127) / 128);
  return splitk_acc_bytes(tiles128, 128) + tiles128 * kEpiWarps * 4;
}

int peer_flags_launch(unsigned* const* flags, int rank, int world, unsigned epoch, int base,
                      int signal, cudaStream_t stream) {
  PeerFlags pf{};
  for (int r = 0; r < world; ++r) pf.flags[r] = flags[r];
  peer_flags_kernel<<<1, 32, 0, stream>>>(flags[rank], pf, rank, world, epoch, base, signal);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("peer flag kernel launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

int rs_reduce_launch(const void* recv, const float* xs, const w8a8_epilogue_t* epi, void* out,
                     int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t rs_rows,
                     void* const* stages, unsigned* const* flags, int rank, int world,
                     unsigned epoch, cudaStream_t stream) {
  GemmArgs g{};
  g.epi = epi;
  g.N = N;
  g.M = M;
  const EpilogueParams ep = to_params(g);
  PeerBytes st{};
  PeerFlags fl{};
  for (int r = 0; r < world; ++r) {
    st.p[r] = static_cast<uint8_t*>(stages[r]);
    fl.flags[r] = flags[r];
  }
  const int64_t own =
      std::max<int64_t>(0, std::min<int64_t>(M, (rank + 1) * rs_rows) - rank * rs_rows);
  const int64_t want = (own * ((N + 511) / 512) + 7) / 8;
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(device_sm_count()) * 8)));
  const auto* rv = static_cast<const uint8_t*>(recv);
  auto* o = static_cast<uint8_t*>(out);
  const int cc = static_cast<int>((N + 31) / 32);
  const int Mi = static_cast<int>(M), Ni = static_cast<int>(N);
  switch (out_dtype) {
    case W8A8_F32:
      rs_reduce_kernel<float><<<grid, 256, 0, stream>>>(rv, xs, ep, o, ldo, Mi, Ni, rs_rows, cc, st,
                                                        fl, rank, world, epoch);
      break;
    case W8A8_F16:
      rs_reduce_kernel<__half><<<grid, 256, 0, stream>>>(rv, xs, ep, o, ldo, Mi, Ni, rs_rows, cc, st,
                                                         fl, rank, world, epoch);
      break;
    default:
      rs_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(rv, xs, ep, o, ldo, Mi, Ni, rs_rows,
                                                                cc, st, fl, rank, world, epoch);
      break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("reduce-scatter finish launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

int rs_gather_launch(void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t rs_rows,
                     const void* stage, unsigned* const* flags, int rank, int world, unsigned epoch,
                     cudaStream_t stream) {
  const int esz = out_dtype == W8A8_F32 ? 4 : 2;
  const int64_t total = M * N * esz / 16;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(
      1, std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(device_sm_count()) * 4)));
  auto* o = static_cast<uint8_t*>(out);
  const auto* sg = static_cast<const uint8_t*>(stage);
  if (esz == 4) {
    rs_gather_kernel<4><<<grid, 256, 0, stream>>>(o, ldo, static_cast<int>(M), static_cast<int>(N),
                                                  rs_rows, sg, flags[rank], rank, world, epoch);
  } else {
    rs_gather_kernel<2><<<grid, 256, 0, stream>>>(o, ldo, static_cast<int>(M), static_cast<int>(N),
                                                  rs_rows, sg, flags[rank], rank, world, epoch);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("reduce-scatter gather launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

int allgather_unpack_launch(const void* recv, void* out, int out_dtype, int64_t ldo, int64_t M,
                            int64_t N_shard, int rank, int world, cudaStream_t stream) {
  const int chunk_cols = static_cast<int>((N_shard + 31) / 32);
  const int64_t chunks = (M + 31) / 32 * chunk_cols;
  const int64_t warps = static_cast<int64_t>(world - 1) * chunks;
  if (warps == 0) return 0;
  const unsigned grid = static_cast<unsigned>((warps + 7) / 8);
  const auto* r = static_cast<const uint8_t*>(recv);
  auto* o = static_cast<uint8_t*>(out);
  if (out_dtype == W8A8_F32) {
    allgather_unpack_kernel<4><<<grid, 256, 0, stream>>>(r, o, ldo, static_cast<int>(M),
                                                         static_cast<int>(N_shard), rank, world,
                                                         chunks, chunk_cols);
  } else {
    allgather_unpack_kernel<2><<<grid, 256, 0, stream>>>(r, o, ldo, static_cast<int>(M),
                                                         static_cast<int>(N_shard), rank, world,
                                                         chunks, chunk_cols);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("all-gather unpack launch failed: %s", cudaGetErrorString(e));
    return W8A8_ERR_ACCELERATOR;
  }
  return 0;
}

int plan_gemm(const GemmArgs& g, bool tc_ok, GemmPlan& p) {
  const int out_bytes = g.out_dtype == W8A8_F32 || g.out_dtype == W8A8_S32 ? 4 : 2;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  int bn = g.cfg && g.cfg->block_n ? g.cfg->block_n : 0;
  if (bn != 0 && bn != 64 && bn != 128 && bn != 256) {
    set_error("block_n must be 64, 128 or 256, got %d", bn);
    return W8A8_ERR_VALUE;
  }
  if (bn == 64 && (g.kind != 0 || g.rms_rope)) {
    set_error("64-column tiles are built for the int8 GEMM without the RoPE epilogue");
    return W8A8_ERR_VALUE;
  }
  const int sms = device_sm_count();
  if (bn == 0) {
    // 256-column tiles when they alone fill every SM; otherwise the 128-column
    // tiles' extra parallelism wins (measured on B200: 256 x 12288 -> 3072
    // runs 27% faster with 128-column tiles, 5600 x 3072 -> 3072 50% slower);
    // and when even 128-column tiles leave half of the SMs idle (few rows),
    // 64-column tiles run on twice as many.
    const long long tiles256 = ((g.M + kBM - 1) / kBM) * ((g.N + 255) / 256);
    const long long tiles128 = ((g.M + kBM - 1) / kBM) * ((g.N + 127) / 128);
    bn = tiles256 >= sms && g.N >= 256 ? 256 : 128;
    if (bn == 128 && 2 * tiles128 <= sms && g.kind == 0 && !g.rms_rope && !g.b_tiled) bn = 64;
  }
  p.group_m = g.cfg && g.cfg->group_m > 0 ? g.cfg->group_m : 8;
  p.max_ctas = g.cfg ? g.cfg->max_ctas : 0;
  int cg = g.cfg && g.cfg->cta_group ? g.cfg->cta_group : 0;
  if (cg != 0 && cg != 1 && cg != 2) {
    set_error("cta_group must be 1 or 2, got %d", cg);
    return W8A8_ERR_VALUE;
  }
  // Default: CTA pairs (each SM loading half of B, six pipeline stages instead
  // of four) for int8 GEMMs with K >= 8192, one CTA per tile otherwise.  On
  // B200 the pair runs 5600 x 12288 -> 3072 in 139 us against 148 us, while at
  // K = 3072 it is 3-4% slower (5600 x 3072 -> 12288 + GELU: 153 us against
  // 148 us): the longer a tile's K loop, the less the per-tile epilogue costs
  // against the pair's cheaper operand stream.
  if (cg == 0) cg = (g.kind == 0 && bn == 256 && g.K >= 8192) ? 2 : 1;
  if (g.b_tiled) {
    // pre-tiled weights: 128-column tiles, one CTA per tile, tcgen05 path only
    if (!(g.kind == 0 && g.K > 0 && g.K % 16 == 0 && g.lda % 16 == 0 && a16(g.a) && a16(g.b) &&
          a16(g.out) && (g.ldo * out_bytes) % 16 == 0)) {
      set_error("pre-tiled weights need K %% 16 == 0 and 16-byte aligned operands");
      return W8A8_ERR_VALUE;
    }
    bn = 128;
    cg = 1;
  }
  if (g.rms_rope) cg = 1;  // heads of 128 columns per epilogue warp half, 1-CTA tiles
  if (bn != 256) cg = 1;   // pairs are built for 256-column tiles
  p.splits = 1;
  p.split_tiles = 0;
  p.workspace_need = 0;
  // Split-K (int8 with a dequant epilogue, scratch given or asked about):
  // explicit split_k > 1, or 128 x 128 tiles that leave SMs idle (few rows)
  // with a K loop long enough to pay for the partials' round trip: every
  // 128-column tile is cut into `splits` K ranges of at least 32 K-blocks
  // (4 KiB of K).  Measured on B200: 256 x 12288 -> 3072 in 30.7 us split in
  // three against 36.9 us whole, but 256 x 6144 -> 3072 in 25.6 us split in
  // three against 22.5-23.5 us whole, 256 x 3072 -> 3072 22.5 against 16.4 us.  Large GEMMs run every tile whole: cutting only the
  // trailing, partial wave of tiles in K measured slower (5600 x 3072 -> 3072:
  // 48 us whole, 114 us with its last 84 tiles cut in five), because the TMA
  // add-reductions of the int32 partials into L2 sustain under 1 TB/s.  (One
  // slot per split with plain stores, summed by the last split, measured
  // slower still for the few-row shapes: 34.8 and 41.0 us.)
  if (g.kind == 0 && g.out_dtype != W8A8_S32 && tc_ok && g.N % 4 == 0 && g.split_k != 1) {
    const int num_kb = static_cast<int>((g.K + kBK - 1) / kBK);
    const int64_t tiles128 = ((g.M + kBM - 1) / kBM) * ((g.N + 127) / 128);
    int full = 1;
    if (g.split_k > 1) {
      full = std::min(g.split_k, num_kb);
    } else {
      const int64_t fill = sms / std::max<int64_t>(1, tiles128);
      full = static_cast<int>(std::min<int64_t>(fill, std::min(8, num_kb / 32)));
    }
    if (full > 1) {
      p.splits = full;
      p.split_tiles = tiles128;
      p.workspace_need = splitk_acc_bytes(tiles128, 128) + tiles128 * kEpiWarps * 4;
      bn = 128;
      cg = 1;
    }
  }
  p.bn = bn;
  p.cg = cg;
  p.tiles = ((g.M + kBM * cg - 1) / (kBM * cg)) * ((g.N + bn - 1) / bn);
  // A partial last wave of 1-CTA 256-column tiles that fills at most half of
  // the persistent CTAs runs as half-width units, twice as many, each half the
  // work (5600 x 3072 -> 12288: 2112 tiles on 148 SMs, the last 40 run as 80
  // units of 128 x 128).  No partial sums: each unit owns its columns.
  p.half_from = p.tiles;
  if (p.splits == 1 && bn == 256 && cg == 1 && !g.b_tiled && g.kind != 2) {
    const int64_t P = std::min<int64_t>(p.tiles, p.max_ctas > 0 ? p.max_ctas : sms);
    const int64_t R = p.tiles % P;
    if (p.tiles > P && R > 0 && 2 * R <= P) p.half_from = p.tiles - R;
  }
  return 0;
}

bool gemm_tc_ok(const GemmArgs& g) {
  const int out_bytes = g.out_dtype == W8A8_F32 || g.out_dtype == W8A8_S32 ? 4 : 2;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return g.K > 0 && g.K % 16 == 0 && g.lda % 16 == 0 && g.ldb % 16 == 0 && a16(g.a) &&
         a16(g.b) && a16(g.out) && (g.ldo * out_bytes) % 16 == 0 && g.M < (1ll << 31) &&
         g.N < (1ll << 31) && g.K < (1ll << 31);
}

int gemm_launch(const GemmArgs& g_in, cudaStream_t stream) {
  GemmArgs g = g_in;  // split_k is cleared below when no scratch is given
  if (g.M == 0 || g.N == 0) return 0;
  const int out_bytes = g.out_dtype == W8A8_F32 || g.out_dtype == W8A8_S32 ? 4 : 2;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool tc_ok = gemm_tc_ok(g);
  if (g.rms_rope) {
    // heads of 128 columns, one per epilogue warp half: the 1-CTA tcgen05 GEMM
    if (!(g.kind == 0 && g.out_dtype == W8A8_BF16 && tc_ok && !g.b_tiled)) {
      set_error("the RMSNorm + RoPE epilogue needs int8 operands, bf16 output, row-major weights, "
                "K %% 16 == 0 and 16-byte aligned operands");
      return W8A8_ERR_VALUE;
    }
    if (g.epi && (g.epi->activation != kActNone || g.epi->residual)) {
      set_error("the RMSNorm + RoPE epilogue takes no output activation or residual");
      return W8A8_ERR_VALUE;
    }
    if (g.rope_cols < 0 || g.rope_cols > g.N || g.rope_cols % 128 != 0 || g.N % 128 != 0) {
      set_error("RoPE columns (%lld) and N (%lld) must be multiples of the 128-column head, "
                "rope columns <= N", static_cast<long long>(g.rope_cols),
                static_cast<long long>(g.N));
      return W8A8_ERR_VALUE;
    }
    if (g.rope_cols > 0 && (!g.rope_w || !g.rope_f ||
                            (reinterpret_cast<uintptr_t>(g.rope_w) & 15u) ||
                            (reinterpret_cast<uintptr_t>(g.rope_f) & 15u))) {
      set_error("RoPE needs a 16-byte aligned norm weight and rotations");
      return W8A8_ERR_VALUE;
    }
  }
  if (g.ag_world > 1 && g.rs_rows > 0) {
    if (!(g.kind == 0 && tc_ok && !g.b_tiled && g.out_dtype == W8A8_S32 &&
          g.ag_world <= kMaxRanks && g.ag_rank >= 0 && g.ag_rank < g.ag_world &&
          g.rs_rows % 32 == 0 && g.N % 4 == 0)) {
      set_error("the fused reduce-scatter needs int8 codes (K %% 16 == 0, 16-byte aligned), "
                "2..%d ranks, row blocks of a multiple of 32 rows and N %% 4 == 0", kMaxRanks);
      return W8A8_ERR_VALUE;
    }
    g.split_k = 1;
    g.workspace = nullptr;
  } else if (g.ag_world > 1) {
    const int esz = out_bytes;
    if (!(g.kind == 0 && tc_ok && !g.rms_rope && !g.b_tiled && g.out_dtype != W8A8_S32 &&
          g.ag_world <= kMaxRanks && g.ag_rank >= 0 && g.ag_rank < g.ag_world &&
          g.N % 8 == 0 && g.ldo % 8 == 0 && esz >= 2 &&
          !(g.epi && g.epi->residual))) {
      set_error("the fused all-gather needs int8 codes, a floating output without residual, "
                "2..%d ranks, K %% 16 == 0, 16-byte aligned operands and N_shard and ldo "
                "multiples of 8", kMaxRanks);
      return W8A8_ERR_VALUE;
    }
    g.split_k = 1;
    g.workspace = nullptr;
  }
  if (!g.workspace) g.split_k = 1;
  GemmPlan plan{};
  if (int rc = plan_gemm(g, tc_ok, plan)) return rc;
  if (plan.splits > 1) {
    if (g.workspace_bytes < plan.workspace_need) {
      set_error("split-K scratch of %lld bytes is smaller than the %lld bytes M=%lld N=%lld need",
                static_cast<long long>(g.workspace_bytes),
                static_cast<long long>(plan.workspace_need), static_cast<long long>(g.M),
                static_cast<long long>(g.N));
      return W8A8_ERR_VALUE;
    } else if (reinterpret_cast<uintptr_t>(g.workspace) & 255u) {
      set_error("split-K scratch must be 256-byte aligned");
      return W8A8_ERR_VALUE;
    }
  }
  if (g.kind == 0) {
    switch (g.out_dtype) {
      case W8A8_BF16: return dispatch_out<0, __nv_bfloat16>(g, tc_ok, plan, stream);
      case W8A8_F16: return dispatch_out<0, __half>(g, tc_ok, plan, stream);
      case W8A8_F32: return dispatch_out<0, float>(g, tc_ok, plan, stream);
      case W8A8_S32: return dispatch_out<0, int32_t>(g, tc_ok, plan, stream);
      default: break;
    }
  } else if (g.kind == 2) {
    const bool mx_ok = tc_ok && g.K % 32 == 0 && a16(g.sfa) && a16(g.sfb);
    // One CTA per tile, 256 columns (one accumulator, the block scales in the
    // TMEM columns the second would take) where 256-column tiles fill the SMs,
    // else 128; CTA pairs (256 x 128 tiles, each SM loading half of B) only
    // when asked for: on B200 they measured 4-8% slower than 1-CTA 128-column
    // tiles (5600 x 3072 -> 3072: 93.3 against 89.1 us; -> 12288: 314 against
    // 292 us; 5600 x 12288 -> 3072: 333 against 306 us).
    GemmPlan mx_plan = plan;
    mx_plan.cg = g.cfg && g.cfg->cta_group ? g.cfg->cta_group : 1;
    mx_plan.bn = mx_plan.cg == 2 ? 128 : plan.bn;
    switch (g.out_dtype) {
      case W8A8_BF16: return dispatch_out<2, __nv_bfloat16>(g, mx_ok, mx_plan, stream);
      case W8A8_F16: return dispatch_out<2, __half>(g, mx_ok, mx_plan, stream);
      case W8A8_F32: return dispatch_out<2, float>(g, mx_ok, mx_plan, stream);
      default: break;
    }
  } else {
    switch (g.out_dtype) {
      case W8A8_BF16: return dispatch_out<1, __nv_bfloat16>(g, tc_ok, plan, stream);
      case W8A8_F16: return dispatch_out<1, __half>(g, tc_ok, plan, stream);
      case W8A8_F32: return dispatch_out<1, float>(g, tc_ok, plan, stream);
      default: break;
    }
  }
  set_error("unsupported output dtype code %d", g.out_dtype);
  return W8A8_ERR_VALUE;
}

}  // namespace w8a8
