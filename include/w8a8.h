/*
 * libw8a8 -- B200 (sm_100a) W8A8 / FP8 / MXFP8 linear family, plain C ABI.
 *
 * Drop-in boundary for the reference's Kitchen INT8/FP8 kernels as the Rust
 * inference crate binds them (reference: inference/native/bridge.hpp:29
 * `imagine_kitchen_call`, dispatching to the launchers of
 * native/comfy-port/kitchen/int8_linear.cu and the Kitchen CUDA ops).  Every
 * entry point takes raw device pointers, element counts/strides and a
 * cudaStream_t passed as `void*`; no framework types cross the boundary.
 *
 * Conventions shared by all entry points:
 *  - The caller owns every buffer (inference/src/cuda_linear.rs:603-605, 638,
 *    681 allocate q, scale and out before each call).  The library allocates
 *    no device memory on any call path.
 *  - Work is enqueued asynchronously on `stream` (the caller's current stream,
 *    inference/src/cuda_linear.rs:448) on the calling thread's current device.
 *  - Return codes follow the reference bridge's exception mapping
 *    (inference/native/bridge.cpp `protect`): 0 ok, -1 runtime, -9 out of
 *    memory, -10 accelerator error, -20 ValueError, -21 IndexError.  The
 *    message is in the thread-local w8a8_last_error().
 *  - Row-major tensors; `ld*` arguments are row strides in elements.
 */
#ifndef IMAGINE_B200_W8A8_H
#define IMAGINE_B200_W8A8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (inference/native/bridge.hpp:14-16, bridge.cpp protect) */
#define W8A8_OK 0
#define W8A8_ERR_RUNTIME (-1)
#define W8A8_ERR_OOM (-9)
#define W8A8_ERR_ACCELERATOR (-10)
#define W8A8_ERR_VALUE (-20)
#define W8A8_ERR_INDEX (-21)

/* ---- dtype codes.  0/1/2 are the reference's output codes
 * (inference/src/cuda_linear.rs:488-497). */
#define W8A8_F32 0
#define W8A8_F16 1
#define W8A8_BF16 2
#define W8A8_S32 3
#define W8A8_S8 4
#define W8A8_E4M3 5

/* ---- row-scale semantics of the INT8 quantiser.
 * EAGER:   max(amax / 127, 1e-30), IEEE divide (inference/src/eager.rs:163-166)
 * KITCHEN: max(min(amax, finite_max) * (1/127), 1e-30), the reference's CUDA
 *          and Triton routes (native/comfy-port/kitchen/int8_linear.cu:206-208),
 *          elements divided with an IEEE divide (its Triton route's numerics)
 * KITCHEN_CUDA: KITCHEN scales with the element numerics of the reference's
 *          Kitchen CUDA kernels as that file is built (--use_fast_math,
 *          native/comfy-port/CMakeLists.txt:30-36): an approximate divide
 *          (__fdividef) for f16 / f32 inputs, a divisor that rounds to zero in
 *          the input type kept (a zero f16 row then codes to -128, as there),
 *          and the fast-math forms of the fused quantiser's input activations.
 *          bf16 codes equal KITCHEN's: a quotient of two 8-bit-significand
 *          values is never within 2 fp32 ulp of a bf16 rounding midpoint. */
#define W8A8_SCALE_EAGER 0
#define W8A8_SCALE_KITCHEN 1
#define W8A8_SCALE_KITCHEN_CUDA 2

/* ---- dequant orders of the INT8 linear epilogue.
 * EAGER:         y = T(acc*(xs*ws)); y = T(y + bias)   (inference/src/int8_linear.rs:244-268)
 * SCALE_PRODUCT: y = T(fma(acc, xs*ws, bias))          (KSRC triton/quantization.py:861-1018)
 * CHAINED:       y = T(fma(acc*xs, ws, bias))          (native/.../int8_linear.cu:669-708, two-row GEMV)
 * SEPARATE:      y = T(((acc*xs)*ws) + bias), three fp32 roundings (native/.../
 *                int8_linear.cu:518-543 and 586-667: the stand-alone dequant with a
 *                bias and the one-row GEMV).  Offered by the CUDA-core entry points
 *                only (w8a8_gemv_dequant, w8a8_linear_small, w8a8_dequantize_linear);
 *                the tensor-core GEMMs reject it. */
#define W8A8_DQ_EAGER 0
#define W8A8_DQ_SCALE_PRODUCT 1
#define W8A8_DQ_CHAINED 2
#define W8A8_DQ_SEPARATE 3

/* ---- output activation applied after bias, before the residual */
#define W8A8_ACT_NONE 0
#define W8A8_ACT_GELU_TANH 1

/* Epilogue description shared by the GEMM, GEMV and dequant entry points. */
typedef struct w8a8_epilogue {
  const float* ws;            /* [N] per-output-channel weight scales, or [1] */
  int64_t ws_numel;           /* N or 1 */
  const void* bias;           /* [N] in the output dtype, or NULL */
  const void* residual;       /* [M, ldr] in the output dtype, or NULL */
  int64_t ldr;                /* residual row stride (elements) */
  const void* residual_scale; /* [N] in the output dtype; required with residual */
  int32_t dequant_order;      /* W8A8_DQ_* */
  int32_t activation;         /* W8A8_ACT_* */
  /* 0: residual_scale is one [N] row for every output row.  g > 0:
   * residual_scale is [ceil(M / g), N] and output row m uses row m / g: the
   * model's gated residual, a per-sample gate [B, 1, N] over B samples of g
   * tokens (inference/src/models/qwen_image21/numeric.rs:110-126), which the
   * reference's residual addcmul broadcasts (inference/src/int8_linear.rs:99-111). */
  int64_t residual_scale_rows;
} w8a8_epilogue_t;

/* Optional GEMM launch configuration (what the autotuner selects).  A NULL
 * pointer, or zero fields, select the built-in heuristic. */
typedef struct w8a8_gemm_config {
  int32_t block_n;   /* 128 or 256 output columns per tile */
  int32_t group_m;   /* M tiles per rasterisation group (L2 reuse) */
  int32_t max_ctas;  /* persistent CTAs (0 = one per SM) */
  int32_t cta_group; /* 1: one CTA per 128-row tile; 2: CTA pairs with 2-SM MMAs on
                        256-row tiles (block_n 256 only); 0: heuristic */
} w8a8_gemm_config_t;

/* ---- library state ---------------------------------------------------- */
/* Thread-local message of the last failing call on this thread
 * (inference/native/bridge.hpp:14 imagine_last_error). */
const char* w8a8_last_error(void);
/* cudaError_t of the last accelerator failure on this thread
 * (inference/native/bridge.hpp:15 imagine_last_accelerator_code). */
int w8a8_last_accelerator_code(void);
/* ABI version of this library (major*100 + minor). */
int w8a8_abi_version(void);
/* Reads, then clears, the device-side error word of the current device after
 * synchronising `stream`.  Nonzero means a kernel's bounded wait gave up
 * (1..4: which barrier).  No reference counterpart: the reference's kernels
 * have no device-side waits. */
int w8a8_device_error(void* stream);

/* ---- a1 / a12: per-row INT8 quantiser ------------------------------------
 * Replaces `quantize_int8_rowwise(x, q, scale, stochastic, seed, stream)`
 * (call site inference/src/cuda_linear.rs:605-616; kernel
 * native/comfy-port/kitchen/int8_linear.cu:184-227, launcher :1322-1371).
 * x [rows, cols] (x_dtype F32/F16/BF16, row stride ldx) -> q int8 [rows, cols]
 * (row stride ldq) and scale fp32 [rows].  stochastic != 0 uses the
 * reference CUDA kernel's PCG-hash noise keyed by (row*cols + col + seed). */
int w8a8_quantize_rowwise(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                          int8_t* q, int64_t ldq, float* scale, int scale_mode, int stochastic,
                          uint64_t seed, void* stream);

/* ---- a2 / a6: input activation + ConvRot fused into the quantiser ---------
 * Replaces `quantize_int8_rowwise_convrot64(x, q, s, group, stochastic,
 * act_code, seed, act_w, eps, stream)` (call site inference/src/convrot.rs:
 * 156-209, chosen by inference/src/cuda_linear.rs:400-417, 586-589; kernel
 * native/comfy-port/kitchen/int8_linear.cu:1197-1314).  group 256: the row is
 * activated and rotated by the normalised 256-point Hadamard matrix in fp32,
 * then quantised (the reference kernel's numerics).  group 0: activation
 * only, rounded to the input dtype the way the reference's ATen activation
 * (inference/src/int8_linear.rs:37-97) rounds it, then quantised.  cols is
 * the quantised width K (a multiple of 256, at most 16384); SwiGLU and SiTU
 * read [gate | up] rows 2*K wide.  act_w [K] (input dtype) is required for
 * RMSNorm.  Stochastic rounding is not offered on this path. */
#define W8A8_INPUT_ACT_NONE 0
#define W8A8_INPUT_ACT_GELU_TANH 1
#define W8A8_INPUT_ACT_SWIGLU 2
#define W8A8_INPUT_ACT_RMS_NORM 3
#define W8A8_INPUT_ACT_SITU 4
int w8a8_quantize_rowwise_convrot(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                  int64_t ldx, int group, int input_act, const void* act_w,
                                  float act_eps, int8_t* q, int64_t ldq, float* scale,
                                  int scale_mode, void* stream);

/* ---- a7: modulation fused into the quantiser ------------------------------
 * The step before the QKV and MLP-up projections, applied on the way into the
 * quantiser so the modulated activation never goes to HBM:
 *   MOD_SCALE      x * (1 + s)                    `int8_linear_modulated`
 *   MOD_RMS_SCALE  rms_norm(x, norm_w, eps) * (1 + s)
 *                                                 `int8_linear_rms_modulated`
 *                  (registry ops inference/src/backend_signatures.rs:128-156,
 *                  eager body inference/src/backend_bindings.rs:329-405)
 *   MOD_ADALN      layer_norm(x, eps) * (1 + s) + shift        `adaln`
 *   MOD_RMS_ADALN  rms_norm(x, eps) * (1 + s) + shift          `rms_adaln`
 *                  (inference/src/backend_eager.rs:176-236; KSRC
 *                  backends/cuda/ops/adaln.cu:103-190)
 * then the optional 256-group ConvRot (group 256) and the row quantiser.
 * s and shift are [rows / mod_group, cols] in the input dtype (row i uses
 * modulation row i / mod_group: the per-sample rows of a batch).  The
 * modulated value is rounded to the input dtype, as the reference stores it;
 * scale_mode KITCHEN follows the reference's CUDA adaln arithmetic (one-pass
 * statistics, one rounding), EAGER its ATen sequence.  cols: a multiple of
 * 256 up to 16384. */
#define W8A8_MOD_SCALE 0
#define W8A8_MOD_RMS_SCALE 1
#define W8A8_MOD_ADALN 2
#define W8A8_MOD_RMS_ADALN 3
int w8a8_quantize_rowwise_modulated(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                    int64_t ldx, int mode, const void* norm_w, float eps,
                                    const void* mod_scale, const void* mod_shift,
                                    int64_t mod_group, int group, int8_t* q, int64_t ldq,
                                    float* scale, int scale_mode, void* stream);

/* ---- a8: Q/K RMSNorm + RoPE after the QKV projection ---------------------
 * Replaces `rms_rope(q, k, freqs_cis, q_scale, k_scale, epsilon)` (call site
 * inference/src/models/qwen_image21/dit.rs:486-505; eager body
 * inference/src/backend_rope.rs:146-223; kernel KSRC
 * backends/cuda/ops/rms_rope.cu:38-240) for the interleaved rotation over the
 * whole head: per (token, head) row of D values, n = T(x * rsqrt(mean(x^2) +
 * eps) * scale), then each pair (n[2i], n[2i+1]) -> (f00 n0 + f01 n1,
 * f10 n0 + f11 n1) in fp32, rounded to T.  q / k: [rows, ld] with heads * D
 * values per row (dtype F32/F16/BF16); freqs: fp32 [freq_rows, D/2, 2, 2]
 * (16-byte aligned), row r uses freqs row r % freq_rows; q_scale / k_scale:
 * [D] in the same dtype.  k may be NULL (q only); q_out may equal q.
 * D: 64, 128, 192 or 256. */
int w8a8_rms_rope(const void* q, const void* k, void* q_out, void* k_out, int dtype, int64_t rows,
                  int64_t heads, int64_t head_dim, int64_t ldq, int64_t ldk, int64_t ldqo,
                  int64_t ldko, const float* freqs, int64_t freq_rows, const void* q_scale,
                  const void* k_scale, float eps, void* stream);

/* ---- a8 fused: the Q or K projection with its RMSNorm + RoPE epilogue ------
 * Replaces the pair `project(q)` (w8a8_gemm_dequant, bf16 output) followed by
 * `rms_rope(q, k, freqs_cis, q_scale, k_scale, epsilon)` (call sites
 * inference/src/models/qwen_image21/dit.rs:427-429 and 486-505; eager body
 * inference/src/backend_rope.rs:146-223) for head_dim 128: the projection's
 * output never makes the round trip through HBM that the stand-alone
 * w8a8_rms_rope pays.  out (bf16, stride ldo) = epilogue(q . w^T) as
 * w8a8_gemm_dequant computes it (activation NONE, no residual); then each
 * 128-column head in columns [0, rope_cols) of every row r is normalised and
 * rotated as w8a8_rms_rope does, with norm_w (bf16) [128] shared by every
 * head or, with norm_w_per_column, [rope_cols] (e.g. q_norm for the q heads
 * then k_norm for the k heads of a fused QKV weight).  Columns from rope_cols
 * on (the v heads of a fused QKV weight) are stored as the plain GEMM stores
 * them.  The rotations come row-blocked (freqs_rows, built for these M rows
 * by w8a8_rope_freqs_rows), so that the epilogue, which holds one row per
 * lane, reads them with coalesced loads.  N and rope_cols: multiples of 128;
 * K % 16 == 0, 16-byte aligned operands (the tcgen05 path); norm_w and
 * freqs_rows 16-byte aligned.  split_k, workspace and workspace_bytes as in
 * w8a8_gemm_dequant_splitk (workspace NULL: no split).  Before the norm the
 * values equal the plain GEMM's bit for bit; the row's sum of squares is
 * added in a different order than w8a8_rms_rope's, so an output may differ
 * from GEMM-then-w8a8_rms_rope by one bf16 ulp per rotated pair. */
int w8a8_gemm_dequant_rms_rope(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw,
                               const float* xs, const w8a8_epilogue_t* epi, void* out, int64_t ldo,
                               int64_t M, int64_t N, int64_t K, int64_t rope_cols,
                               const void* norm_w, int norm_w_per_column, const float* freqs_rows,
                               float eps, int split_k, void* workspace, int64_t workspace_bytes,
                               const w8a8_gemm_config_t* cfg, void* stream);

/* Row-blocked rotations for w8a8_gemm_dequant_rms_rope.  freqs: fp32
 * [freq_rows, 64, 2, 2] (16-byte aligned), row r of the GEMM using freqs row
 * r % freq_rows, as in w8a8_rms_rope.  out: w8a8_rope_freqs_rows_bytes(rows)
 * bytes, 16-byte aligned; out[((r / 32) * 64 + p) * 32 + r % 32] is the
 * 16-byte rotation (f00, f01, f10, f11) of pair p for row r, over rows padded
 * to a multiple of 128.  The rotations are the same for every block of a
 * forward pass: build them once per (freqs, rows). */
int64_t w8a8_rope_freqs_rows_bytes(int64_t rows);
int w8a8_rope_freqs_rows(const float* freqs, int64_t freq_rows, int64_t rows, float* out,
                         void* stream);

/* ---- column-parallel linear with the all-gather fused into the GEMM -------
 * No reference counterpart (the reference runs on one GPU).  Ranks of one
 * NVLink domain (one process per GPU) each hold an equal N-shard of the weight
 * ([N_shard, K], with its ws / bias shard in `epi`) and the same activation
 * codes; every rank ends with the whole [M, N] output, rank r's shard at
 * columns r * N_shard.  Instead of a GEMM followed by an all-gather
 * collective, the GEMM's epilogue writes each finished 32 x 32 output chunk to
 * this rank's output and also copies it, whole and contiguous, into this
 * rank's region of every peer's receive buffer over NVLink, so the exchange
 * overlaps the math tile by tile; w8a8_allgather_finish then waits for the
 * peers and places their chunks into the output.
 *   recvs[r]: rank r's receive buffer, w8a8_allgather_recv_bytes(M, N_shard,
 *             out_dtype, world) bytes, 16-byte aligned, mapped into this
 *             process (peer pointers, e.g. symmetric memory);
 *   flags[r]: rank r's flag block of W8A8_PEER_FLAG_WORDS uint32, zeroed once
 *             before first use, likewise mapped;
 *   epoch:    one more on every call (the same on all ranks, never 0).
 * Per call, on every rank, in stream order: w8a8_peer_barrier (no rank writes
 * into another's receive buffer before all are done with the previous
 * call's), the quantiser, w8a8_gemm_dequant_allgather, w8a8_allgather_finish.
 * The GEMM's last CTA to finish signals the peers; the waits are bounded (2 s)
 * and record a device error on timeout.  N_shard and ldo (>= world * N_shard)
 * multiples of 8; K % 16 == 0; 2 to 8 ranks; int8 codes; no residual; one
 * launch per rank with identical shapes. */
#define W8A8_MAX_RANKS 8
#define W8A8_PEER_FLAG_WORDS 32
int64_t w8a8_allgather_recv_bytes(int64_t M, int64_t N_shard, int out_dtype, int world);
int w8a8_peer_barrier(unsigned* const* flags, int rank, int world, unsigned epoch, void* stream);
int w8a8_gemm_dequant_allgather(const int8_t* q, int64_t ldq, const int8_t* w_shard, int64_t ldw,
                                const float* xs, const w8a8_epilogue_t* epi, void* out,
                                int out_dtype, int64_t ldo, int64_t M, int64_t N_shard, int64_t K,
                                void* const* recvs, unsigned* const* flags, int rank, int world,
                                unsigned epoch, const w8a8_gemm_config_t* cfg, void* stream);
int w8a8_allgather_finish(void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N_shard,
                          void* const* recvs, unsigned* const* flags, int rank, int world,
                          unsigned epoch, void* stream);

/* ---- row-parallel (K-sharded) quantisation --------------------------------
 * No reference counterpart: the reference runs on one GPU.  A K-sharded
 * activation needs the absmax of the whole row before any shard can be
 * quantised.  w8a8_row_absmax writes each row's max |x| (fp32 [rows]); after
 * an all-reduce(MAX) across ranks, w8a8_quantize_rowwise_given_absmax
 * quantises the local shard with the scale the full row would get, so every
 * rank's codes equal the single-GPU codes of its columns. */
int w8a8_row_absmax(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                    float* amax, void* stream);
int w8a8_quantize_rowwise_given_absmax(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                       int64_t ldx, const float* amax, int8_t* q, int64_t ldq,
                                       float* scale, int scale_mode, void* stream);

/* ---- a3 / a4 / a6: INT8 GEMM with fused dequant epilogue -----------------
 * Replaces `cutlass_int8_dequant(q, w, xs, ws, bias, out, out_code, stream)`
 * and `cutlass_int8_dequant_residual(...)` (call sites
 * inference/src/cuda_linear.rs:724-764; kernels KSRC
 * backends/cuda/ops/cutlass_gemm_int8.cu:348-420).  Unlike the reference, the
 * call never declines: it returns 0 for every valid shape (tcgen05 path when
 * K % 16 == 0 and rows are 16-byte aligned, else a CUDA-core path).
 * out[m, n] = epilogue(sum_k q[m,k] * w[n,k]) with q int8 [M, K] (stride ldq),
 * w int8 [N, K] (stride ldw), xs fp32 [M]. */
int w8a8_gemm_dequant(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* xs,
                      const w8a8_epilogue_t* epi, void* out, int out_dtype, int64_t ldo, int64_t M,
                      int64_t N, int64_t K, const w8a8_gemm_config_t* cfg, void* stream);

/* Raw int32 accumulators acc[M, N] = q[M,K] . w[N,K]^T.  Replaces
 * `cublas_gemm_int8(q, w, acc_i32, workspace, stream)` (call site
 * inference/src/cuda_linear.rs:769-780; KSRC backends/cuda/ops/cublas_gemm_int8.cu:89-230);
 * needs no workspace. */
/* ---- a3: split-K form of w8a8_gemm_dequant for few-row shapes -----------
 * Same arguments and results as w8a8_gemm_dequant (which it replaces at the
 * same call sites, inference/src/cuda_linear.rs:724-764, when M is small: the
 * 256-token text stream).  When the 128 x 128 output tiles alone would leave
 * SMs idle, the K range is cut into split_k parts (0: chosen from the SM
 * count, 1: off) run by different CTAs; their int32 partial tiles are added
 * into `workspace`, so results are identical bit for bit to the unsplit
 * GEMM.  The caller owns the workspace, as it owns cublas_gemm_int8's
 * (cuda_linear.rs:769-780): at least w8a8_gemm_splitk_workspace_bytes(M, N)
 * bytes (64 KiB per 128 x 128 output tile plus counters), or for split_k = 0
 * w8a8_gemm_auto_workspace_bytes(M, N, K, cfg), 256-byte aligned,
 * zero-filled before the first call; every call leaves it zero-filled again.  Calls sharing a workspace must not overlap on
 * the GPU.  After a nonzero w8a8_device_error the workspace must be cleared. */
int64_t w8a8_gemm_splitk_workspace_bytes(int64_t M, int64_t N);
/* Scratch the automatic policy (split_k = 0) uses for an M x N x K int8 GEMM
 * with a floating output and tile configuration cfg (NULL: defaults) on the
 * current device: w8a8_gemm_splitk_workspace_bytes(M, N) when it splits the
 * few-row shape, 0 when it runs every tile whole (then the workspace may be
 * NULL). */
int64_t w8a8_gemm_auto_workspace_bytes(int64_t M, int64_t N, int64_t K,
                                       const w8a8_gemm_config_t* cfg);
int w8a8_gemm_dequant_splitk(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw,
                             const float* xs, const w8a8_epilogue_t* epi, void* out, int out_dtype,
                             int64_t ldo, int64_t M, int64_t N, int64_t K, int split_k,
                             void* workspace, int64_t workspace_bytes,
                             const w8a8_gemm_config_t* cfg, void* stream);

/* ---- a3: pre-tiled weights for few-row shapes ----------------------------
 * No reference counterpart (the reference streams W row-major).  A GEMM with
 * few rows (the 256-token text stream) reads all of W from HBM once; row-major
 * W arrives as 128-byte pieces of 128 rows 12 KB apart.  w8a8_pack_weight_tiles
 * rewrites an int8 W [N, K] (row stride ldw) once, offline, as 128-row x
 * 128-byte tiles, each 16 KB contiguous, ordered (row block, K block), zero
 * padded to multiples of 128: w8a8_weight_tiles_bytes(N, K) bytes, 16-byte
 * aligned.  w8a8_gemm_dequant_tiled (K a multiple of 16, q rows and out
 * 16-byte aligned) then equals w8a8_gemm_dequant_splitk on the original W bit
 * for bit (workspace NULL: no split). */
int64_t w8a8_weight_tiles_bytes(int64_t N, int64_t K);
int w8a8_pack_weight_tiles(const int8_t* w, int64_t ldw, int64_t N, int64_t K, int8_t* tiles,
                           void* stream);
int w8a8_gemm_dequant_tiled(const int8_t* q, int64_t ldq, const int8_t* tiles, const float* xs,
                            const w8a8_epilogue_t* epi, void* out, int out_dtype, int64_t ldo,
                            int64_t M, int64_t N, int64_t K, int split_k, void* workspace,
                            int64_t workspace_bytes, const w8a8_gemm_config_t* cfg,
                            void* stream);

/* ---- the same split-K GEMM for callers that cannot allocate --------------
 * No counterpart in the reference.  Some callers cannot hand the library a
 * workspace: a plugin host whose enqueue call passes no workspace pointer, a
 * serving loop that has frozen its memory pool after warm-up and may not call
 * cudaMalloc again, or a binding from another language with no device
 * allocator of its own.  This entry point takes the arguments of
 * w8a8_gemm_dequant_splitk minus the workspace, returns the same results, and
 * allocates nothing: its scratch is an array of
 * W8A8_SPLITK_STATIC_SCRATCH_BYTES (8 MiB) built into the library, one per
 * device.  A GEMM that does not split (split_k = 1, or split_k = 0 on a shape
 * the automatic policy runs whole) uses no scratch and runs at any size.  A
 * GEMM that splits and whose scratch (64 KiB per 128 x 128 output tile plus
 * counters, e.g. up to 512 x 3072 or 256 x 6144) does not fit is rejected
 * with W8A8_ERR_VALUE and a message.  The first call on a device, with that
 * device current, looks the array up (cudaGetSymbolAddress) and caches the
 * address; make it before any stream capture, and do not call this entry
 * point again on a device after cudaDeviceReset in the same process (the
 * cached address is stale then).  A splitting call clears the part of the
 * array it uses on `stream` before the GEMM.  All calls share the array:
 * calls that overlap on the GPU (other streams, other threads) race with
 * each other. */
#define W8A8_SPLITK_STATIC_SCRATCH_BYTES (8ll << 20)
int w8a8_gemm_dequant_splitk_static(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw,
                                    const float* xs, const w8a8_epilogue_t* epi, void* out,
                                    int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                                    int split_k, const w8a8_gemm_config_t* cfg, void* stream);

int w8a8_gemm_s32(const int8_t* q, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K,
                  const w8a8_gemm_config_t* cfg, void* stream);

/* Stand-alone dequant of int32 accumulators.  Replaces
 * `dequantize_int8_linear(acc, xs, ws, bias, out, code, stream)` (call site
 * inference/src/cuda_linear.rs:782-795; kernel
 * native/comfy-port/kitchen/int8_linear.cu:517-583, launcher :1721-1798). */
int w8a8_dequantize_linear(const int32_t* acc, const float* xs, const w8a8_epilogue_t* epi,
                           void* out, int out_dtype, int64_t M, int64_t N, void* stream);

/* ---- a5: M <= 2 GEMV ---------------------------------------------------------
 * Replaces `int8_gemv_dequant(q, w, xs, ws, bias, out, out_code, stream,
 * [resid], [rscale])` (call site inference/src/cuda_linear.rs:657-677;
 * kernels native/comfy-port/kitchen/int8_linear.cu:585-708, launcher
 * :1800-1929).  M in {1, 2}; K % 16 == 0 and 16-byte aligned q/w rows use the
 * vector path, anything else a scalar path. */
int w8a8_gemv_dequant(const int8_t* q, const int8_t* w, const float* xs,
                      const w8a8_epilogue_t* epi, void* out, int out_dtype, int64_t M, int64_t N,
                      int64_t K, void* stream);

/* Fused quantise + GEMV for M <= 2 in one launch.  Replaces
 * `int8_linear_m1(x, q, xs, w, ws, bias, out, out_code, convrot=false, ...)`
 * (call site inference/src/cuda_linear.rs:557-583; KSRC
 * backends/cuda/dlpack_bindings.cpp:3594-3690) and extends it to two rows (the
 * AdaLN modulation linear).  q_out [M, K] / xs_out [M] receive the codes and
 * scales (either may be NULL). */
int w8a8_linear_small(const void* x, int x_dtype, const int8_t* w, const w8a8_epilogue_t* epi,
                      int scale_mode, int8_t* q_out, float* xs_out, void* out, int out_dtype,
                      int64_t M, int64_t N, int64_t K, void* stream);

/* ---- a9: FP8 e4m3, per-tensor scales ---------------------------------------
 * Replaces `quantize_per_tensor_fp8(x, scale, out)` (call site
 * inference/src/models/qwen_image21/layers.rs:124-151; kernel KSRC
 * backends/cuda/ops/per_tensor_quantize.cu:39-72) with the eager numerics of
 * inference/src/eager.rs:74-88: out = e4m3(clamp(x * T(1/scale), +-448)).
 * `scale` is a device fp32 scalar. */
int w8a8_quantize_fp8_tensor(const void* x, int x_dtype, int64_t numel, const float* scale,
                             uint8_t* out, void* stream);

/* Per-tensor FP8 GEMM on tcgen05 kind::f8f6f4: out = (a . b^T) * (sa*sb) + bias.
 * Replaces `imagine_fp8_scaled_mm` -> at::_scaled_mm_v2 TensorWise
 * (inference/native/bridge.cpp:401-413).  a e4m3 [M, K], b e4m3 [N, K],
 * sa / sb device fp32 scalars, bias [N] in the output dtype or NULL. */
int w8a8_fp8_gemm(const uint8_t* a, const uint8_t* b, const float* sa, const float* sb,
                  const void* bias, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                  const w8a8_gemm_config_t* cfg, void* stream);

/* ---- a10: MXFP8 (32-element K blocks, e8m0 scales) ------------------------
 * Replaces `quantize_mxfp8(x, pad_32x=false)` (inference/src/eager.rs:176-225;
 * KSRC backends/cuda/ops/quantize_mxfp8.cu:40-147) with the eager numerics.
 * x [rows, cols] (cols % 32 == 0, 16-byte aligned rows) -> payload e4m3
 * [rows, cols] (row stride ldq) and e8m0 scales in the cuBLAS blocked layout
 * of inference/src/block_scales.rs:4-31: a buffer of
 * ceil(rows/128)*128 x ceil(cols/128)*4 bytes, padding written as zeros.
 * A block with 0 < amax <= 448 * 2^-127 gets scale byte 0 and a finite payload
 * (the reference divides by its zero decoding of byte 0). */
int w8a8_quantize_mxfp8(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                        uint8_t* q, int64_t ldq, uint8_t* scales, void* stream);

/* MXFP8 GEMM on tcgen05 kind::mxf8f6f4.block_scale: out = sum over 32-element
 * blocks of (a . b) * 2^(ea-127) * 2^(eb-127) + bias.  Replaces
 * `scaled_mm_mxfp8` -> at::_scaled_mm_v2 BlockWise1x32 with SWIZZLE_32_4_4
 * (inference/src/backend_quant.rs:320-343).  a e4m3 [M, K], b e4m3 [N, K],
 * scales as written by w8a8_quantize_mxfp8, K % 32 == 0. */
int w8a8_mxfp8_gemm(const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                    const uint8_t* b_scales, const void* bias, void* out, int out_dtype, int64_t M,
                    int64_t N, int64_t K, const w8a8_gemm_config_t* cfg, void* stream);

/* ---- row-parallel linear with the reduce-scatter fused into the GEMM ------
 *
 * No reference counterpart (the reference runs on one GPU).  The K-sharded
 * (row-parallel) linear: each of `world` ranks holds codes q [M, K_shard]
 * quantised with the full rows' scales xs (w8a8_row_absmax, a MAX across
 * ranks, w8a8_quantize_rowwise_given_absmax) and W [:, K_shard].  Instead of
 * an int32 GEMM followed by an all-reduce:
 *   w8a8_gemm_s32_reduce_scatter: the GEMM's epilogue copies every finished
 *     32 x 32 int32 partial chunk, whole, into the receive buffer of the rank
 *     that owns those rows (rank r owns rows [r * R, (r + 1) * R), R =
 *     w8a8_reduce_scatter_rows(M, world)), over NVLink while the math runs;
 *     its last CTA then writes `epoch` into every peer's done flags.
 *   w8a8_reduce_scatter_finish: waits for the peers' partials, sums them
 *     (exact int32), applies the epilogue (dequant order, bias, GELU,
 *     residual: `epi` as for w8a8_gemm_dequant) to the owned rows, writes them
 *     to `out` [M, ldo] and to every peer's staging buffer, then waits for the
 *     peers' rows and copies them into `out`.
 * The result equals the single-GPU linear bit for bit.
 *   recvs[r]:  rank r's receive buffer, w8a8_reduce_scatter_recv_bytes(M, N,
 *              world) bytes;  stages[r]: rank r's staging buffer, M * N *
 *              sizeof(out dtype) bytes;  flags[r]: its 32-word flag block
 *              (zeroed once) -- all mapped into this process (CUDA VMM or
 *              symmetric memory), 16-byte aligned.
 * Per call on every rank: w8a8_peer_barrier, the quantiser,
 * w8a8_gemm_s32_reduce_scatter, w8a8_reduce_scatter_finish (same epoch). */
int64_t w8a8_reduce_scatter_rows(int64_t M, int world);
int64_t w8a8_reduce_scatter_recv_bytes(int64_t M, int64_t N, int world);
int w8a8_gemm_s32_reduce_scatter(const int8_t* q, int64_t ldq, const int8_t* w_shard, int64_t ldw,
                                 int64_t M, int64_t N, int64_t K_shard, void* const* recvs,
                                 unsigned* const* flags, int rank, int world, unsigned epoch,
                                 const w8a8_gemm_config_t* cfg, void* stream);
int w8a8_reduce_scatter_finish(const float* xs, const w8a8_epilogue_t* epi, void* out,
                               int out_dtype, int64_t ldo, int64_t M, int64_t N,
                               void* const* recvs, void* const* stages, unsigned* const* flags,
                               int rank, int world, unsigned epoch, void* stream);

/* ---- sampler step: flow parameterisation + CFG combine + Euler / ER-SDE ----
 *
 * One elementwise pass per denoising step over the fp32 latent x [n]:
 *   denoised = cfg_combine(x - out_cond * sigma, x - out_uncond * sigma, scale)
 * (the flow / CONST parameterisation, inference/src/models/qwen_image21/
 * sampling.rs:165-167 and denoiser.rs:135; the full-area aggregation of
 * cfg.rs:145-207, whose x1 / +0 / /(1e-37 + 1) steps only normalise the sign
 * of zeros; cfg_combine sampling.rs:178-180), then the sampler's update of x:
 *   EULER  (sampling.rs:231-277): x += ((x - denoised) / sigma_hat) * dt
 *   ER_SDE (er_sde.rs:60-134): the stage 1-3 update with the multistep state
 *          old_denoised / old_derivative (updated in place) and the noise term
 *   CHURN  (sampling.rs:244-253): x += (noise * s_noise) * coef[0], before the
 *          model runs at sigma_hat
 *   DENOISED: only writes `denoised`.
 * Every fp32 operation rounds once, in ATen's order (no FMA contraction), so
 * with the same per-step scalars the result equals the reference's tensor
 * operations bit for bit.
 *
 * out_cond / out_uncond: the model outputs (f32, f16 or bf16 code in
 * out_dtype), [n] each; out_uncond NULL when the negative branch is skipped
 * (CFG = 1 shortcut, cfg.rs:136-144: uncond reads as zeros).
 * coef: device fp32 array of the step's scalars (1 for DENOISED and CHURN,
 * 3 for EULER, 9 for ER_SDE), computed with the
 * reference's 0-dim tensor operations on the sigmas' device:
 *   [0] the model's sigma (timestep)
 *   EULER:  [1] sigma_hat, [2] dt = sigma_next - sigma_hat
 *   ER_SDE: [1] r_alpha * r, [2] alpha_t * (1 - r), [3] the stage-2
 *           coefficient alpha_t * (dt + integral * noise_scaler(t)),
 *           [4] s - lambda[i-1], [5] the stage-3 coefficient, [6] (s -
 *           lambda[i-2]) / 2, [7] alpha_t, [8] the noise deviation
 *   CHURN:  [0] (sigma_hat^2 - sigma^2)^0.5
 * denoised: optional output [n] (NULL: not written).  noise: [n] fp32 (ER_SDE
 * with has_noise, CHURN). */
#define W8A8_STEP_DENOISED 0
#define W8A8_STEP_EULER 1
#define W8A8_STEP_ER_SDE 2
#define W8A8_STEP_CHURN 3
typedef struct {
  int mode;        /* W8A8_STEP_* */
  int stage;       /* ER_SDE: min(max_stage, i + 1), 1..3 */
  int last;        /* ER_SDE: the next sigma is 0, x becomes denoised */
  int has_noise;   /* ER_SDE: settings.noise > 0 */
  float cfg_scale; /* the CFG scale as fp32 (ATen's mul by a double scalar) */
  float s_noise;   /* ER_SDE / CHURN: settings.noise as fp32 */
  int denoised_input; /* 1: out_cond already is the denoised prediction (an
                         execution whose denoise() returns it, no flow
                         parameterisation or CFG); out_uncond must be NULL */
} w8a8_sampler_step_t;

int w8a8_sampler_step(float* x, const void* out_cond, const void* out_uncond, int out_dtype,
                      int64_t n, const float* coef, const w8a8_sampler_step_t* step,
                      float* denoised, float* old_denoised, float* old_derivative,
                      const float* noise, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IMAGINE_B200_W8A8_H */
