// Internal declarations shared by the libw8a8 translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/w8a8.h"

namespace w8a8 {

// Device-side error word (one per device, module-scope __device__ variable).
int read_and_clear_device_error(cudaStream_t stream, int* value);

// mode 0: quantise; 1: row absmax only (into `scales`); 2: quantise with the
// row absmax given in `amax_in`.
int quantize_rowwise_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                            int8_t* q, int64_t ldq, float* scales, int scale_mode, int stochastic,
                            uint64_t seed, int mode, const float* amax_in, cudaStream_t stream);

// Fused input activation (+ 256-point ConvRot when rotate != 0) + row-wise
// INT8 quantiser; act codes W8A8_INPUT_ACT_*.
// act 5-8 are the modulations (W8A8_MOD_* + 5) with scale / shift rows
// [rows / mod_group, cols].
int quantize_act_rot_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                            int rotate, int act, const void* act_w, float act_eps,
                            const void* mod_scale, const void* mod_shift, int64_t mod_group,
                            int8_t* q, int64_t ldq, float* scales, int scale_mode,
                            cudaStream_t stream);

// kind 0: int8 x int8 (s32 accumulate); kind 1: e4m3 x e4m3 (f32 accumulate);
// kind 2: MXFP8 e4m3 x e4m3 with e8m0 block scales (f32 accumulate).
// Returns 0 on success, a W8A8_ERR_* code otherwise (message via set_error).
struct GemmArgs {
  int kind;
  const void* a;
  int64_t lda;  // elements (bytes)
  const void* b;
  int64_t ldb;
  const float* xs;    // int8: [M] row scales
  const float* sa;    // fp8: device scalar
  const float* sb;    // fp8: device scalar
  const w8a8_epilogue_t* epi;  // may be null for raw s32
  void* out;
  int out_dtype;      // W8A8_F32/F16/BF16/S32
  int64_t ldo;
  int64_t M, N, K;
  const w8a8_gemm_config_t* cfg;
  const void* sfa;  // kind 2 (MXFP8): blocked e8m0 scales of a and b
  const void* sfb;
  // split-K (kind 0 with a dequant epilogue): 0 = choose, 1 = off, >1 = splits;
  // used only with a zero-filled scratch of splitk_workspace_bytes(M, N)
  int split_k;
  void* workspace;
  int64_t workspace_bytes;
  // B in the pre-tiled layout of w8a8_pack_weight_tiles (kind 0 only)
  int b_tiled;
  // per-head RMSNorm + RoPE epilogue (kind 0, bf16 output)
  int rms_rope;
  const void* rope_w;
  int rope_w_percol;
  const float* rope_f;  // row-blocked rotations (w8a8_rope_freqs_rows)
  int64_t rope_cols;
  float rope_eps;
  // column-parallel all-gather fused into the epilogue (ag_world > 1); `out`
  // is this rank's output at its shard's first column, ag_recv[r] rank r's
  // receive buffer
  int ag_world;
  int ag_rank;
  void* ag_recv[W8A8_MAX_RANKS];
  unsigned* ag_flags[W8A8_MAX_RANKS];
  unsigned ag_epoch;
  // row-parallel reduce-scatter of the int32 partials (rs_rows > 0, with the
  // ag_* peers and an S32 output): rank r owns rows [r * rs_rows, ...)
  int64_t rs_rows;
};
int gemm_launch(const GemmArgs& args, cudaStream_t stream);
// Fused all-gather flags (gemm_sm100.cu): base 0 with signal = the barrier on
// the ready slots; base W8A8_MAX_RANKS without signal = the wait for the
// peers' GEMMs.
int peer_flags_launch(unsigned* const* flags, int rank, int world, unsigned epoch, int base,
                      int signal, cudaStream_t stream);
// The peers' chunks in this rank's receive buffer into its output [M, ldo]
// (rank r's shard at columns r * N_shard).
int allgather_unpack_launch(const void* recv, void* out, int out_dtype, int64_t ldo, int64_t M,
                            int64_t N_shard, int rank, int world, cudaStream_t stream);
// Row-parallel reduce-scatter finish: sum the owned rows' int32 partials, the
// dequant epilogue, own rows to `out` and to every peer's staging buffer, then
// (last CTA) the done flags at [24, 32).  rs_gather: wait for every peer's
// rows, copy them from this rank's staging buffer into `out`.
int rs_reduce_launch(const void* recv, const float* xs, const w8a8_epilogue_t* epi, void* out,
                     int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t rs_rows,
                     void* const* stages, unsigned* const* flags, int rank, int world,
                     unsigned epoch, cudaStream_t stream);
int rs_gather_launch(void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t rs_rows,
                     const void* stage, unsigned* const* flags, int rank, int world, unsigned epoch,
                     cudaStream_t stream);
// Modulation (act 5..8) + quantiser without ConvRot for 16-bit rows of at
// most 8192 columns in the plain quantiser's layout; -1: not handled here
// (the ConvRot-layout kernel takes the call).
int quantize_modulated_vec_launch(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                  int64_t ldx, int act, const void* norm_w, float eps,
                                  const void* mod_scale, const void* mod_shift, int64_t mod_group,
                                  int8_t* q, int64_t ldq, float* scales, int scale_mode,
                                  cudaStream_t stream);
// The fused sampler step (flow parameterisation, CFG, Euler / ER-SDE update).
int sampler_step_launch(float* x, const void* out_cond, const void* out_uncond, int out_dtype,
                        int64_t n, const float* coef, const w8a8_sampler_step_t& step,
                        float* denoised, float* old_denoised, float* old_derivative,
                        const float* noise, cudaStream_t stream);
// Tile shape and split-K layout gemm_launch uses for a GEMM.
struct GemmPlan {
  int bn, cg, group_m, max_ctas;
  int splits;              // > 1: every tile is cut into this many K ranges
  int64_t split_tiles;     // tiles cut in K
  int64_t workspace_need;  // scratch bytes the split tiles use (0 without splits)
  int64_t tiles;           // output tiles of bn columns
  int64_t half_from;       // tiles from here on run as two 128-column units
};
// tc_ok: the operands suit the tcgen05 path.  Returns 0 or an error code.
int plan_gemm(const GemmArgs& g, bool tc_ok, GemmPlan& plan);
// Whether the operands suit the tcgen05 path (K % 16, 16-byte aligned rows).
bool gemm_tc_ok(const GemmArgs& g);
// Split-K scratch: int32 partial sums [tiles * 128, bn], then one arrival
// counter per (tile, epilogue warp).
int64_t splitk_acc_bytes(int64_t split_tiles, int bn);
int64_t splitk_workspace_bytes(int64_t M, int64_t N);
// Pre-tiled weights: [ceil(N/128)][ceil(K/128)][128 rows][128 bytes], zero
// padded (gemv.cu).
int64_t weight_tiles_bytes(int64_t N, int64_t K);
int pack_weight_tiles_launch(const int8_t* w, int64_t ldw, int64_t N, int64_t K, int8_t* tiles,
                             cudaStream_t stream);
// gemm_launch on the library's fixed split-K scratch (gemm_splitk_static.cu).
int gemm_splitk_static_launch(GemmArgs g, cudaStream_t stream);

int dequant_launch(const int32_t* acc, const float* xs, const w8a8_epilogue_t* epi, void* out,
                   int out_dtype, int64_t M, int64_t N, cudaStream_t stream);

int gemv_launch(const int8_t* q, const int8_t* w, const float* xs, const w8a8_epilogue_t* epi,
                void* out, int out_dtype, int64_t M, int64_t N, int64_t K, cudaStream_t stream);

int linear_small_launch(const void* x, int x_dtype, const int8_t* w, const w8a8_epilogue_t* epi,
                        int scale_mode, int8_t* q_out, float* xs_out, void* out, int out_dtype,
                        int64_t M, int64_t N, int64_t K, cudaStream_t stream);

int quantize_mxfp8_launch(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                          uint8_t* q, int64_t ldq, uint8_t* sf, cudaStream_t stream);

int quantize_fp8_tensor_launch(const void* x, int x_dtype, int64_t numel, const float* scale,
                               uint8_t* out, cudaStream_t stream);

// Q/K RMSNorm + interleaved RoPE (rope.cu); k may be NULL.
// Row-blocked rotations for the fused RMSNorm + RoPE epilogue (rope.cu).
int rope_freqs_rows_launch(const float* freqs, int64_t freq_rows, int64_t rows, float* out,
                           cudaStream_t stream);
int rms_rope_launch(const void* q, const void* k, void* q_out, void* k_out, int dtype,
                    int64_t rows, int heads, int head_dim, int64_t ldq, int64_t ldk, int64_t ldqo,
                    int64_t ldko, const float* freqs, int64_t freq_rows, const void* q_scale,
                    const void* k_scale, float eps, cudaStream_t stream);

// Error reporting (thread-local), implemented in api.cu.
void set_error(const char* fmt, ...);

// Number of SMs on the current device (cached per device).
int device_sm_count();

}  // namespace w8a8
