// extern "C" entry points of libw8a8 (declared in include/w8a8.h): argument
// validation, error reporting and dispatch to the kernels.
//
// Error mapping follows the reference bridge (inference/native/bridge.cpp,
// `protect`): invalid arguments -> W8A8_ERR_VALUE (-20), out-of-range indices
// -> W8A8_ERR_INDEX (-21), CUDA failures -> W8A8_ERR_ACCELERATOR (-10) with the
// cudaError_t kept for w8a8_last_accelerator_code().  No call allocates device
// memory and no call synchronises the stream except w8a8_device_error.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "w8a8_internal.h"

namespace w8a8 {
namespace {
thread_local char g_last_error[512] = "";
thread_local int g_last_accel = 0;
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int device_sm_count() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64) {
    if (cache[dev] == 0) {
      int n = 0;
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
  }
  return 148;
}

namespace {

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// Converts a pending CUDA error (if any) into the accelerator code.
int finish(int rc) {
  if (rc == W8A8_ERR_ACCELERATOR) {
    g_last_accel = static_cast<int>(cudaPeekAtLastError());
  }
  if (rc == 0) g_last_error[0] = '\0';
  return rc;
}

bool is_float_dtype(int d) { return d == W8A8_F32 || d == W8A8_F16 || d == W8A8_BF16; }

// cuda_core: the entry point runs the epilogue on CUDA cores (dequant_one),
// which alone offers W8A8_DQ_SEPARATE.
int check_epilogue(const w8a8_epilogue_t* epi, int64_t N, bool need_ws, bool cuda_core = false) {
  if (!epi) return fail(W8A8_ERR_VALUE, "epilogue descriptor is NULL");
  if (need_ws) {
    if (!epi->ws) return fail(W8A8_ERR_VALUE, "weight scale pointer is NULL");
    if (epi->ws_numel != 1 && epi->ws_numel != N) {
      return fail(W8A8_ERR_VALUE,
                  "INT8 weight scale must be scalar or per-output-channel, got %lld for N=%lld",
                  static_cast<long long>(epi->ws_numel), static_cast<long long>(N));
    }
  }
  if (epi->residual && !epi->residual_scale) {
    return fail(W8A8_ERR_VALUE, "int8_linear: residual requires residual_scale");
  }
  if (epi->residual && epi->residual_scale_rows < 0) {
    return fail(W8A8_ERR_VALUE, "residual_scale_rows must be >= 0, got %lld",
                static_cast<long long>(epi->residual_scale_rows));
  }
  if (epi->residual && epi->ldr < N) {
    return fail(W8A8_ERR_VALUE, "residual row stride %lld < N=%lld",
                static_cast<long long>(epi->ldr), static_cast<long long>(N));
  }
  if (epi->dequant_order == W8A8_DQ_SEPARATE && !cuda_core) {
    return fail(W8A8_ERR_VALUE,
                "dequant order SEPARATE is offered by the GEMV, the small linear and the "
                "stand-alone dequant only");
  }
  if (epi->dequant_order < W8A8_DQ_EAGER || epi->dequant_order > W8A8_DQ_SEPARATE) {
    return fail(W8A8_ERR_VALUE, "unknown dequant order %d", epi->dequant_order);
  }
  if (epi->activation != W8A8_ACT_NONE && epi->activation != W8A8_ACT_GELU_TANH) {
    return fail(W8A8_ERR_VALUE, "unknown output activation %d", epi->activation);
  }
  return 0;
}

}  // namespace
}  // namespace w8a8

using namespace w8a8;

extern "C" {

const char* w8a8_last_error(void) { return g_last_error; }

int w8a8_last_accelerator_code(void) { return g_last_accel; }

int w8a8_abi_version(void) { return 103; }

int w8a8_device_error(void* stream) {
  int v = 0;
  const int rc = read_and_clear_device_error(static_cast<cudaStream_t>(stream), &v);
  if (rc != 0) {
    g_last_accel = rc;
    return fail(W8A8_ERR_ACCELERATOR, "reading the device error word failed: %s",
                cudaGetErrorString(static_cast<cudaError_t>(rc)));
  }
  return v;
}

int w8a8_quantize_rowwise(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                          int8_t* q, int64_t ldq, float* scale, int scale_mode, int stochastic,
                          uint64_t seed, void* stream) {
  if (rows < 0 || cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (scale_mode < W8A8_SCALE_EAGER || scale_mode > W8A8_SCALE_KITCHEN_CUDA) {
    return fail(W8A8_ERR_VALUE, "unknown scale mode %d", scale_mode);
  }
  if (rows == 0 || cols == 0) return finish(0);
  if (!x || !q || !scale) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldx < cols || ldq < cols) return fail(W8A8_ERR_VALUE, "row stride smaller than cols");
  if (cols > 0x7fffffffLL || rows > 0x7fffffffLL) {
    return fail(W8A8_ERR_VALUE, "quantize_int8_rowwise only supports rows, K <= INT_MAX");
  }
  return finish(quantize_rowwise_launch(x, x_dtype, rows, cols, ldx, q, ldq, scale, scale_mode,
                                        stochastic, seed, 0, nullptr,
                                        static_cast<cudaStream_t>(stream)));
}

int w8a8_quantize_rowwise_convrot(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                  int64_t ldx, int group, int input_act, const void* act_w,
                                  float act_eps, int8_t* q, int64_t ldq, float* scale,
                                  int scale_mode, void* stream) {
  if (rows < 0 || cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (scale_mode < W8A8_SCALE_EAGER || scale_mode > W8A8_SCALE_KITCHEN_CUDA) {
    return fail(W8A8_ERR_VALUE, "unknown scale mode %d", scale_mode);
  }
  if (group != 0 && group != 256) {
    return fail(W8A8_ERR_VALUE, "fused ConvRot quantiser supports group 256 (or 0: no rotation), got %d",
                group);
  }
  if (input_act < W8A8_INPUT_ACT_NONE || input_act > W8A8_INPUT_ACT_SITU) {
    return fail(W8A8_ERR_VALUE, "unknown input activation code %d", input_act);
  }
  if (cols == 0 || cols % 256 != 0 || cols > 16384) {
    return fail(W8A8_ERR_VALUE, "fused quantiser needs K a multiple of 256 in [256, 16384], got %lld",
                static_cast<long long>(cols));
  }
  const int64_t in_cols =
      (input_act == W8A8_INPUT_ACT_SWIGLU || input_act == W8A8_INPUT_ACT_SITU) ? 2 * cols : cols;
  if (input_act == W8A8_INPUT_ACT_RMS_NORM && !act_w) {
    return fail(W8A8_ERR_VALUE, "input_act 'rms_norm' requires act_weight");
  }
  if (rows == 0) return finish(0);
  if (rows > 0x7fffffffLL) return fail(W8A8_ERR_VALUE, "rows must be <= INT_MAX");
  if (!x || !q || !scale) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldx < in_cols || ldq < cols) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  return finish(quantize_act_rot_launch(x, x_dtype, rows, cols, ldx, group == 256 ? 1 : 0,
                                        input_act, act_w, act_eps, nullptr, nullptr, 1, q, ldq,
                                        scale, scale_mode, static_cast<cudaStream_t>(stream)));
}

int w8a8_quantize_rowwise_modulated(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                    int64_t ldx, int mode, const void* norm_w, float eps,
                                    const void* mod_scale, const void* mod_shift,
                                    int64_t mod_group, int group, int8_t* q, int64_t ldq,
                                    float* scale, int scale_mode, void* stream) {
  if (rows < 0 || cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (scale_mode < W8A8_SCALE_EAGER || scale_mode > W8A8_SCALE_KITCHEN_CUDA) {
    return fail(W8A8_ERR_VALUE, "unknown scale mode %d", scale_mode);
  }
  if (mode < W8A8_MOD_SCALE || mode > W8A8_MOD_RMS_ADALN) {
    return fail(W8A8_ERR_VALUE, "unknown modulation mode %d", mode);
  }
  if (group != 0 && group != 256) {
    return fail(W8A8_ERR_VALUE, "fused ConvRot quantiser supports group 256 (or 0: no rotation), got %d",
                group);
  }
  if (cols == 0 || cols % 256 != 0 || cols > 16384) {
    return fail(W8A8_ERR_VALUE, "fused quantiser needs K a multiple of 256 in [256, 16384], got %lld",
                static_cast<long long>(cols));
  }
  if (mod_group < 1) return fail(W8A8_ERR_VALUE, "modulation group must be >= 1");
  if (!mod_scale) return fail(W8A8_ERR_VALUE, "modulation scale pointer is NULL");
  if ((mode == W8A8_MOD_ADALN || mode == W8A8_MOD_RMS_ADALN) && !mod_shift) {
    return fail(W8A8_ERR_VALUE, "modulation shift pointer is NULL");
  }
  if (mode == W8A8_MOD_RMS_SCALE && !norm_w) return fail(W8A8_ERR_VALUE, "norm weight pointer is NULL");
  if (rows == 0) return finish(0);
  if (rows > 0x7fffffffLL) return fail(W8A8_ERR_VALUE, "rows must be <= INT_MAX");
  if (!x || !q || !scale) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldx < cols || ldq < cols) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  if (group != 256) {
    // no rotation: the plain quantiser's row-in-registers layout when it fits
    const int rc = quantize_modulated_vec_launch(x, x_dtype, rows, cols, ldx, mode + 5, norm_w, eps,
                                                 mod_scale, mod_shift, mod_group, q, ldq, scale,
                                                 scale_mode, static_cast<cudaStream_t>(stream));
    if (rc != -1) return finish(rc);
  }
  return finish(quantize_act_rot_launch(x, x_dtype, rows, cols, ldx, group == 256 ? 1 : 0, mode + 5,
                                        norm_w, eps, mod_scale, mod_shift, mod_group, q, ldq, scale,
                                        scale_mode, static_cast<cudaStream_t>(stream)));
}

int w8a8_rms_rope(const void* q, const void* k, void* q_out, void* k_out, int dtype, int64_t rows,
                  int64_t heads, int64_t head_dim, int64_t ldq, int64_t ldk, int64_t ldqo,
                  int64_t ldko, const float* freqs, int64_t freq_rows, const void* q_scale,
                  const void* k_scale, float eps, void* stream) {
  if (rows < 0 || heads < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(dtype)) return fail(W8A8_ERR_VALUE, "dtype code %d is not floating", dtype);
  if (head_dim != 64 && head_dim != 128 && head_dim != 192 && head_dim != 256) {
    return fail(W8A8_ERR_VALUE, "rms_rope supports head_dim 64, 128, 192 or 256, got %lld",
                static_cast<long long>(head_dim));
  }
  if (rows == 0 || heads == 0) return finish(0);
  if (rows * heads > (1ll << 40) || heads > 0x7fffffffLL) return fail(W8A8_ERR_VALUE, "shape too large");
  if (!q || !q_out || !freqs || !q_scale) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (k && (!k_out || !k_scale)) return fail(W8A8_ERR_VALUE, "k needs k_out and k_scale");
  if (freq_rows < 1) return fail(W8A8_ERR_VALUE, "freqs must have at least one row");
  if (ldq < heads * head_dim || ldqo < heads * head_dim ||
      (k && (ldk < heads * head_dim || ldko < heads * head_dim))) {
    return fail(W8A8_ERR_VALUE, "row stride smaller than heads * head_dim");
  }
  if (reinterpret_cast<uintptr_t>(freqs) & 15u) return fail(W8A8_ERR_VALUE, "freqs must be 16-byte aligned");
  return finish(rms_rope_launch(q, k, q_out, k_out, dtype, rows, static_cast<int>(heads),
                                static_cast<int>(head_dim), ldq, ldk, ldqo, ldko, freqs, freq_rows,
                                q_scale, k_scale, eps, static_cast<cudaStream_t>(stream)));
}

int w8a8_gemm_dequant_rms_rope(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw,
                               const float* xs, const w8a8_epilogue_t* epi, void* out, int64_t ldo,
                               int64_t M, int64_t N, int64_t K, int64_t rope_cols,
                               const void* norm_w, int norm_w_per_column, const float* freqs_rows,
                               float eps, int split_k, void* workspace, int64_t workspace_bytes,
                               const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0 || rope_cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (split_k < 0) return fail(W8A8_ERR_VALUE, "split_k must be >= 0, got %d", split_k);
  if (int rc = check_epilogue(epi, N, true)) return rc;
  if (epi->activation != W8A8_ACT_NONE || epi->residual) {
    return fail(W8A8_ERR_VALUE, "the RMSNorm + RoPE epilogue takes no output activation or residual");
  }
  if (N % 128 != 0 || rope_cols % 128 != 0 || rope_cols > N) {
    return fail(W8A8_ERR_VALUE,
                "N (%lld) and rope_cols (%lld) must be multiples of 128 with rope_cols <= N",
                static_cast<long long>(N), static_cast<long long>(rope_cols));
  }
  if (M == 0 || N == 0) return finish(0);
  if (!q || !w || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (rope_cols > 0 && (!norm_w || !freqs_rows)) {
    return fail(W8A8_ERR_VALUE, "NULL norm weight or rotations");
  }
  if (ldq < K || ldw < K || ldo < N) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  if (split_k > 1 && !workspace) return fail(W8A8_ERR_VALUE, "split-K needs a scratch buffer");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = w;
  g.ldb = ldw;
  g.xs = xs;
  g.epi = epi;
  g.out = out;
  g.out_dtype = W8A8_BF16;
  g.ldo = ldo;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  g.split_k = workspace ? split_k : 1;
  g.workspace = workspace;
  g.workspace_bytes = workspace_bytes;
  g.rms_rope = 1;
  g.rope_w = norm_w;
  g.rope_w_percol = norm_w_per_column ? 1 : 0;
  g.rope_f = freqs_rows;
  g.rope_cols = rope_cols;
  g.rope_eps = eps;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int64_t w8a8_rope_freqs_rows_bytes(int64_t rows) {
  if (rows < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  return (rows + 127) / 128 * 128 * 64 * 16;
}

int w8a8_rope_freqs_rows(const float* freqs, int64_t freq_rows, int64_t rows, float* out,
                         void* stream) {
  if (rows < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (rows == 0) return finish(0);
  if (!freqs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (freq_rows < 1) return fail(W8A8_ERR_VALUE, "freqs must have at least one row");
  if ((reinterpret_cast<uintptr_t>(freqs) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u)) {
    return fail(W8A8_ERR_VALUE, "freqs and out must be 16-byte aligned");
  }
  return finish(rope_freqs_rows_launch(freqs, freq_rows, rows, out, static_cast<cudaStream_t>(stream)));
}

namespace {
int check_peers(unsigned* const* flags, int rank, int world) {
  if (world < 2 || world > W8A8_MAX_RANKS) {
    return fail(W8A8_ERR_VALUE, "world must be 2..%d, got %d", W8A8_MAX_RANKS, world);
  }
  if (rank < 0 || rank >= world) return fail(W8A8_ERR_VALUE, "rank %d outside 0..%d", rank, world - 1);
  if (!flags) return fail(W8A8_ERR_VALUE, "NULL flag pointer array");
  for (int r = 0; r < world; ++r) {
    if (!flags[r] || (reinterpret_cast<uintptr_t>(flags[r]) & 3u)) {
      return fail(W8A8_ERR_VALUE, "flag block of rank %d is NULL or misaligned", r);
    }
  }
  return 0;
}
}  // namespace

int w8a8_peer_barrier(unsigned* const* flags, int rank, int world, unsigned epoch, void* stream) {
  if (int rc = check_peers(flags, rank, world)) return rc;
  if (epoch == 0) return fail(W8A8_ERR_VALUE, "epoch must be nonzero");
  return finish(peer_flags_launch(flags, rank, world, epoch, 0, 1, static_cast<cudaStream_t>(stream)));
}

int64_t w8a8_allgather_recv_bytes(int64_t M, int64_t N_shard, int out_dtype, int world) {
  if (M < 0 || N_shard < 0 || world < 1) return fail(W8A8_ERR_VALUE, "negative shape");
  const int64_t esz = out_dtype == W8A8_F32 ? 4 : 2;
  return static_cast<int64_t>(world) * ((M + 31) / 32) * ((N_shard + 31) / 32) * 32 * 32 * esz;
}

int w8a8_gemm_dequant_allgather(const int8_t* q, int64_t ldq, const int8_t* w_shard, int64_t ldw,
                                const float* xs, const w8a8_epilogue_t* epi, void* out,
                                int out_dtype, int64_t ldo, int64_t M, int64_t N_shard, int64_t K,
                                void* const* recvs, unsigned* const* flags, int rank, int world,
                                unsigned epoch, const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N_shard < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N_shard, true)) return rc;
  if (int rc = check_peers(flags, rank, world)) return rc;
  if (epoch == 0) return fail(W8A8_ERR_VALUE, "epoch must be nonzero");
  if (!recvs) return fail(W8A8_ERR_VALUE, "NULL receive buffer array");
  for (int r = 0; r < world; ++r) {
    if (!recvs[r] || (reinterpret_cast<uintptr_t>(recvs[r]) & 15u)) {
      return fail(W8A8_ERR_VALUE, "receive buffer of rank %d is NULL or not 16-byte aligned", r);
    }
  }
  if (ldo < world * N_shard) return fail(W8A8_ERR_VALUE, "ldo smaller than world * N_shard");
  if (M == 0 || N_shard == 0) return finish(0);
  if (!q || !w_shard || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldq < K || ldw < K) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  const int esz = out_dtype == W8A8_F32 ? 4 : 2;
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = w_shard;
  g.ldb = ldw;
  g.xs = xs;
  g.epi = epi;
  g.out = static_cast<uint8_t*>(out) + static_cast<int64_t>(rank) * N_shard * esz;
  g.out_dtype = out_dtype;
  g.ldo = ldo;
  g.M = M;
  g.N = N_shard;
  g.K = K;
  g.cfg = cfg;
  g.split_k = 1;
  g.ag_world = world;
  g.ag_rank = rank;
  for (int r = 0; r < world; ++r) {
    g.ag_recv[r] = recvs[r];
    g.ag_flags[r] = flags[r];
  }
  g.ag_epoch = epoch;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int w8a8_allgather_finish(void* out, int out_dtype, int64_t ldo, int64_t M, int64_t N_shard,
                          void* const* recvs, unsigned* const* flags, int rank, int world,
                          unsigned epoch, void* stream) {
  if (M < 0 || N_shard < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_peers(flags, rank, world)) return rc;
  if (epoch == 0) return fail(W8A8_ERR_VALUE, "epoch must be nonzero");
  if (!recvs || !recvs[rank] || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldo < world * N_shard || N_shard % 8 || ldo % 8) {
    return fail(W8A8_ERR_VALUE, "ldo must be >= world * N_shard, both multiples of 8");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = peer_flags_launch(flags, rank, world, epoch, W8A8_MAX_RANKS, 0, st)) return finish(rc);
  return finish(allgather_unpack_launch(recvs[rank], out, out_dtype, ldo, M, N_shard, rank, world, st));
}

int64_t w8a8_reduce_scatter_rows(int64_t M, int world) {
  if (M < 0 || world < 1) return fail(W8A8_ERR_VALUE, "negative shape or no ranks");
  const int64_t per = (M + world - 1) / world;
  return std::max<int64_t>(32, (per + 31) / 32 * 32);
}

int64_t w8a8_reduce_scatter_recv_bytes(int64_t M, int64_t N, int world) {
  const int64_t rows = w8a8_reduce_scatter_rows(M, world);
  if (rows < 0 || N < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  return static_cast<int64_t>(world) * (rows / 32) * ((N + 31) / 32) * 32 * 32 * 4;
}

int w8a8_gemm_s32_reduce_scatter(const int8_t* q, int64_t ldq, const int8_t* w_shard, int64_t ldw,
                                 int64_t M, int64_t N, int64_t K_shard, void* const* recvs,
                                 unsigned* const* flags, int rank, int world, unsigned epoch,
                                 const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K_shard < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (int rc = check_peers(flags, rank, world)) return rc;
  if (epoch == 0) return fail(W8A8_ERR_VALUE, "epoch must be nonzero");
  if (!recvs) return fail(W8A8_ERR_VALUE, "NULL receive buffer array");
  for (int r = 0; r < world; ++r) {
    if (!recvs[r] || (reinterpret_cast<uintptr_t>(recvs[r]) & 15u)) {
      return fail(W8A8_ERR_VALUE, "receive buffer of rank %d is NULL or not 16-byte aligned", r);
    }
  }
  if (N % 4) return fail(W8A8_ERR_VALUE, "N must be a multiple of 4");
  if (M == 0 || N == 0) return finish(0);
  if (!q || !w_shard) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldq < K_shard || ldw < K_shard) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = w_shard;
  g.ldb = ldw;
  g.out = recvs[rank];  // no [M, N] output: the chunks go to their owners
  g.out_dtype = W8A8_S32;
  g.ldo = N;
  g.M = M;
  g.N = N;
  g.K = K_shard;
  g.cfg = cfg;
  g.split_k = 1;
  g.ag_world = world;
  g.ag_rank = rank;
  for (int r = 0; r < world; ++r) {
    g.ag_recv[r] = recvs[r];
    g.ag_flags[r] = flags[r];
  }
  g.ag_epoch = epoch;
  g.rs_rows = w8a8_reduce_scatter_rows(M, world);
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int w8a8_reduce_scatter_finish(const float* xs, const w8a8_epilogue_t* epi, void* out,
                               int out_dtype, int64_t ldo, int64_t M, int64_t N,
                               void* const* recvs, void* const* stages, unsigned* const* flags,
                               int rank, int world, unsigned epoch, void* stream) {
  if (M < 0 || N < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true)) return rc;
  if (int rc = check_peers(flags, rank, world)) return rc;
  if (epoch == 0) return fail(W8A8_ERR_VALUE, "epoch must be nonzero");
  if (!recvs || !stages || !recvs[rank]) return fail(W8A8_ERR_VALUE, "NULL buffer array");
  for (int r = 0; r < world; ++r) {
    if (!stages[r] || (reinterpret_cast<uintptr_t>(stages[r]) & 15u)) {
      return fail(W8A8_ERR_VALUE, "staging buffer of rank %d is NULL or not 16-byte aligned", r);
    }
  }
  if (N % 8 || ldo % 8 || ldo < N) {
    return fail(W8A8_ERR_VALUE, "N and ldo must be multiples of 8 with ldo >= N");
  }
  if (M > 0 && N > 0 && (!xs || !out || (reinterpret_cast<uintptr_t>(out) & 15u))) {
    return fail(W8A8_ERR_VALUE, "NULL row scales or a NULL / misaligned output");
  }
  const int64_t rows = w8a8_reduce_scatter_rows(M, world);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // every peer's partial chunks have landed (the GEMMs' done flags)
  if (int rc = peer_flags_launch(flags, rank, world, epoch, W8A8_MAX_RANKS, 0, st)) return finish(rc);
  if (int rc = rs_reduce_launch(recvs[rank], xs, epi, out, out_dtype, ldo, M, N, rows, stages, flags,
                                rank, world, epoch, st)) {
    return finish(rc);
  }
  return finish(rs_gather_launch(out, out_dtype, ldo, M, N, rows, stages[rank], flags, rank, world,
                                 epoch, st));
}

int w8a8_sampler_step(float* x, const void* out_cond, const void* out_uncond, int out_dtype,
                      int64_t n, const float* coef, const w8a8_sampler_step_t* step,
                      float* denoised, float* old_denoised, float* old_derivative,
                      const float* noise, void* stream) {
  if (n < 0) return fail(W8A8_ERR_VALUE, "negative size");
  if (!step) return fail(W8A8_ERR_VALUE, "NULL step description");
  if (step->mode < W8A8_STEP_DENOISED || step->mode > W8A8_STEP_CHURN) {
    return fail(W8A8_ERR_VALUE, "unknown sampler step mode %d", step->mode);
  }
  if (!is_float_dtype(out_dtype)) {
    return fail(W8A8_ERR_VALUE, "model output dtype code %d is not floating", out_dtype);
  }
  if (n == 0) return finish(0);
  if (!x || !coef) return fail(W8A8_ERR_VALUE, "NULL latent or coefficient pointer");
  const int mode = step->mode;
  if (mode != W8A8_STEP_CHURN && !out_cond) return fail(W8A8_ERR_VALUE, "NULL model output");
  if (mode == W8A8_STEP_DENOISED && !denoised) return fail(W8A8_ERR_VALUE, "NULL denoised output");
  if (mode == W8A8_STEP_ER_SDE) {
    if (step->stage < 1 || step->stage > 3) {
      return fail(W8A8_ERR_VALUE, "ER-SDE stage must be 1..3, got %d", step->stage);
    }
    if (!old_denoised) return fail(W8A8_ERR_VALUE, "ER-SDE needs the old_denoised buffer");
    if (!step->last && step->stage >= 2 && !old_derivative) {
      return fail(W8A8_ERR_VALUE, "ER-SDE stage >= 2 needs the old_derivative buffer");
    }
    if (!step->last && step->has_noise && !noise) return fail(W8A8_ERR_VALUE, "NULL noise");
  }
  if (mode == W8A8_STEP_CHURN && !noise) return fail(W8A8_ERR_VALUE, "NULL noise");
  if (step->denoised_input && out_uncond) {
    return fail(W8A8_ERR_VALUE, "a denoised model output has no unconditional branch");
  }
  return finish(sampler_step_launch(x, out_cond, out_uncond, out_dtype, n, coef, *step, denoised,
                                    old_denoised, old_derivative, noise,
                                    static_cast<cudaStream_t>(stream)));
}

int w8a8_row_absmax(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                    float* amax, void* stream) {
  if (rows < 0 || cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (rows == 0) return finish(0);
  if (!amax || (cols > 0 && !x)) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldx < cols) return fail(W8A8_ERR_VALUE, "row stride smaller than cols");
  if (cols > 0x7fffffffLL || rows > 0x7fffffffLL) return fail(W8A8_ERR_VALUE, "rows, K <= INT_MAX");
  if (cols == 0) {
    cudaError_t e = cudaMemsetAsync(amax, 0, rows * sizeof(float), static_cast<cudaStream_t>(stream));
    return finish(e == cudaSuccess ? 0 : W8A8_ERR_ACCELERATOR);
  }
  return finish(quantize_rowwise_launch(x, x_dtype, rows, cols, ldx, nullptr, cols, amax, 0, 0, 0,
                                        1, nullptr, static_cast<cudaStream_t>(stream)));
}

int w8a8_quantize_rowwise_given_absmax(const void* x, int x_dtype, int64_t rows, int64_t cols,
                                       int64_t ldx, const float* amax, int8_t* q, int64_t ldq,
                                       float* scale, int scale_mode, void* stream) {
  if (rows < 0 || cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (scale_mode < W8A8_SCALE_EAGER || scale_mode > W8A8_SCALE_KITCHEN_CUDA) {
    return fail(W8A8_ERR_VALUE, "unknown scale mode %d", scale_mode);
  }
  if (rows == 0 || cols == 0) return finish(0);
  if (!x || !q || !scale || !amax) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldx < cols || ldq < cols) return fail(W8A8_ERR_VALUE, "row stride smaller than cols");
  if (cols > 0x7fffffffLL || rows > 0x7fffffffLL) return fail(W8A8_ERR_VALUE, "rows, K <= INT_MAX");
  return finish(quantize_rowwise_launch(x, x_dtype, rows, cols, ldx, q, ldq, scale, scale_mode, 0, 0,
                                        2, amax, static_cast<cudaStream_t>(stream)));
}

int w8a8_gemm_dequant(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* xs,
                      const w8a8_epilogue_t* epi, void* out, int out_dtype, int64_t ldo, int64_t M,
                      int64_t N, int64_t K, const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true)) return rc;
  if (M == 0 || N == 0) return finish(0);
  if ((K > 0 && (!q || !w)) || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldq < K || ldw < K || ldo < N) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = w;
  g.ldb = ldw;
  g.xs = xs;
  g.epi = epi;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = ldo;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int64_t w8a8_gemm_splitk_workspace_bytes(int64_t M, int64_t N) {
  if (M < 0 || N < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  return splitk_workspace_bytes(M, N);
}

int64_t w8a8_gemm_auto_workspace_bytes(int64_t M, int64_t N, int64_t K,
                                       const w8a8_gemm_config_t* cfg) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (M == 0 || N == 0) return 0;
  GemmArgs g{};
  g.kind = 0;
  g.out_dtype = W8A8_BF16;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  g.split_k = 0;
  GemmPlan plan{};
  const bool tc_ok = K > 0 && K % 16 == 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31);
  if (int rc = plan_gemm(g, tc_ok, plan)) return fail(rc, "%s", w8a8_last_error());
  return plan.workspace_need;
}

int w8a8_gemm_dequant_splitk(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw,
                             const float* xs, const w8a8_epilogue_t* epi, void* out, int out_dtype,
                             int64_t ldo, int64_t M, int64_t N, int64_t K, int split_k,
                             void* workspace, int64_t workspace_bytes,
                             const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (split_k < 0) return fail(W8A8_ERR_VALUE, "split_k must be >= 0, got %d", split_k);
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true)) return rc;
  if (M == 0 || N == 0) return finish(0);
  if ((K > 0 && (!q || !w)) || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldq < K || ldw < K || ldo < N) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  if (split_k != 1 && !workspace) return fail(W8A8_ERR_VALUE, "split-K needs a scratch buffer");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = w;
  g.ldb = ldw;
  g.xs = xs;
  g.epi = epi;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = ldo;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  g.split_k = split_k;
  g.workspace = workspace;
  g.workspace_bytes = workspace_bytes;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int w8a8_gemm_dequant_splitk_static(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw,
                                    const float* xs, const w8a8_epilogue_t* epi, void* out,
                                    int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                                    int split_k, const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (split_k < 0) return fail(W8A8_ERR_VALUE, "split_k must be >= 0, got %d", split_k);
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true)) return rc;
  if (M == 0 || N == 0) return finish(0);
  if ((K > 0 && (!q || !w)) || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldq < K || ldw < K || ldo < N) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = w;
  g.ldb = ldw;
  g.xs = xs;
  g.epi = epi;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = ldo;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  g.split_k = split_k;
  return finish(gemm_splitk_static_launch(g, static_cast<cudaStream_t>(stream)));
}

int64_t w8a8_weight_tiles_bytes(int64_t N, int64_t K) {
  if (N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  return weight_tiles_bytes(N, K);
}

int w8a8_pack_weight_tiles(const int8_t* w, int64_t ldw, int64_t N, int64_t K, int8_t* tiles,
                           void* stream) {
  if (N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (N == 0 || K == 0) return finish(0);
  if (!w || !tiles) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldw < K) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  if (reinterpret_cast<uintptr_t>(tiles) & 15u) return fail(W8A8_ERR_VALUE, "tiles must be 16-byte aligned");
  return finish(pack_weight_tiles_launch(w, ldw, N, K, tiles, static_cast<cudaStream_t>(stream)));
}

int w8a8_gemm_dequant_tiled(const int8_t* q, int64_t ldq, const int8_t* tiles, const float* xs,
                            const w8a8_epilogue_t* epi, void* out, int out_dtype, int64_t ldo,
                            int64_t M, int64_t N, int64_t K, int split_k, void* workspace,
                            int64_t workspace_bytes, const w8a8_gemm_config_t* cfg,
                            void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (split_k < 0) return fail(W8A8_ERR_VALUE, "split_k must be >= 0, got %d", split_k);
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true)) return rc;
  if (M == 0 || N == 0) return finish(0);
  if (!q || !tiles || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldq < K || ldo < N) return fail(W8A8_ERR_VALUE, "row stride smaller than the row");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = ldq;
  g.b = tiles;
  g.ldb = 128;
  g.xs = xs;
  g.epi = epi;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = ldo;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  g.split_k = workspace ? split_k : 1;
  g.workspace = workspace;
  g.workspace_bytes = workspace_bytes;
  g.b_tiled = 1;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int w8a8_gemm_s32(const int8_t* q, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K,
                  const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (M == 0 || N == 0) return finish(0);
  if ((K > 0 && (!q || !w)) || !acc) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  GemmArgs g{};
  g.kind = 0;
  g.a = q;
  g.lda = K;
  g.b = w;
  g.ldb = K;
  g.out = acc;
  g.out_dtype = W8A8_S32;
  g.ldo = N;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int w8a8_dequantize_linear(const int32_t* acc, const float* xs, const w8a8_epilogue_t* epi,
                           void* out, int out_dtype, int64_t M, int64_t N, void* stream) {
  if (M < 0 || N < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true, true)) return rc;
  if (M == 0 || N == 0) return finish(0);
  if (!acc || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  return finish(dequant_launch(acc, xs, epi, out, out_dtype, M, N, static_cast<cudaStream_t>(stream)));
}

int w8a8_gemv_dequant(const int8_t* q, const int8_t* w, const float* xs,
                      const w8a8_epilogue_t* epi, void* out, int out_dtype, int64_t M, int64_t N,
                      int64_t K, void* stream) {
  if (M != 1 && M != 2) return fail(W8A8_ERR_VALUE, "GEMV supports M in {1, 2}, got %lld", static_cast<long long>(M));
  if (N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (int rc = check_epilogue(epi, N, true, true)) return rc;
  if (N == 0) return finish(0);
  if (!q || !w || !xs || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  return finish(gemv_launch(q, w, xs, epi, out, out_dtype, M, N, K, static_cast<cudaStream_t>(stream)));
}

int w8a8_linear_small(const void* x, int x_dtype, const int8_t* w, const w8a8_epilogue_t* epi,
                      int scale_mode, int8_t* q_out, float* xs_out, void* out, int out_dtype,
                      int64_t M, int64_t N, int64_t K, void* stream) {
  if (M != 1 && M != 2) return fail(W8A8_ERR_VALUE, "small linear supports M in {1, 2}, got %lld", static_cast<long long>(M));
  if (N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (scale_mode < W8A8_SCALE_EAGER || scale_mode > W8A8_SCALE_KITCHEN_CUDA) {
    return fail(W8A8_ERR_VALUE, "unknown scale mode %d", scale_mode);
  }
  if (int rc = check_epilogue(epi, N, true, true)) return rc;
  if (N == 0) return finish(0);
  if (!x || !w || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  return finish(linear_small_launch(x, x_dtype, w, epi, scale_mode, q_out, xs_out, out, out_dtype,
                                    M, N, K, static_cast<cudaStream_t>(stream)));
}

int w8a8_quantize_fp8_tensor(const void* x, int x_dtype, int64_t numel, const float* scale,
                             uint8_t* out, void* stream) {
  if (numel < 0) return fail(W8A8_ERR_VALUE, "negative size");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (numel == 0) return finish(0);
  if (!x || !scale || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  return finish(quantize_fp8_tensor_launch(x, x_dtype, numel, scale, out, static_cast<cudaStream_t>(stream)));
}

int w8a8_fp8_gemm(const uint8_t* a, const uint8_t* b, const float* sa, const float* sb,
                  const void* bias, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                  const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (M == 0 || N == 0) return finish(0);
  if ((K > 0 && (!a || !b)) || !sa || !sb || !out) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  w8a8_epilogue_t epi{};
  epi.ws_numel = 1;
  epi.bias = bias;
  epi.dequant_order = W8A8_DQ_CHAINED;
  GemmArgs g{};
  g.kind = 1;
  g.a = a;
  g.lda = K;
  g.b = b;
  g.ldb = K;
  g.sa = sa;
  g.sb = sb;
  g.epi = &epi;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = N;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

int w8a8_quantize_mxfp8(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx,
                        uint8_t* q, int64_t ldq, uint8_t* scales, void* stream) {
  if (rows < 0 || cols < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(x_dtype)) return fail(W8A8_ERR_VALUE, "input dtype code %d is not floating", x_dtype);
  if (cols % 32 != 0) return fail(W8A8_ERR_VALUE, "K dimension must be divisible by 32");
  if (rows == 0 || cols == 0) return finish(0);
  if (!x || !q || !scales) return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  if (ldx < cols || ldq < cols) return fail(W8A8_ERR_VALUE, "row stride smaller than cols");
  const int elem = x_dtype == W8A8_F32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) % 16 != 0 ||
      (ldx * elem) % 16 != 0 || ldq % 16 != 0) {
    return fail(W8A8_ERR_VALUE, "mxfp8 quantiser needs 16-byte aligned rows");
  }
  if (cols > 0x7fffffffLL || rows > 0x7fffffffLL) return fail(W8A8_ERR_VALUE, "rows, K <= INT_MAX");
  return finish(quantize_mxfp8_launch(x, x_dtype, rows, cols, ldx, q, ldq, scales,
                                      static_cast<cudaStream_t>(stream)));
}

int w8a8_mxfp8_gemm(const uint8_t* a, const uint8_t* a_scales, const uint8_t* b,
                    const uint8_t* b_scales, const void* bias, void* out, int out_dtype, int64_t M,
                    int64_t N, int64_t K, const w8a8_gemm_config_t* cfg, void* stream) {
  if (M < 0 || N < 0 || K < 0) return fail(W8A8_ERR_VALUE, "negative shape");
  if (!is_float_dtype(out_dtype)) return fail(W8A8_ERR_VALUE, "output dtype code %d is not floating", out_dtype);
  if (K % 32 != 0) return fail(W8A8_ERR_VALUE, "K dimension must be divisible by 32");
  if (M == 0 || N == 0) return finish(0);
  if ((K > 0 && (!a || !b || !a_scales || !b_scales)) || !out) {
    return fail(W8A8_ERR_VALUE, "NULL tensor pointer");
  }
  w8a8_epilogue_t epi{};
  epi.ws_numel = 1;
  epi.bias = bias;
  epi.dequant_order = W8A8_DQ_CHAINED;
  GemmArgs g{};
  g.kind = 2;
  g.a = a;
  g.lda = K;
  g.b = b;
  g.ldb = K;
  g.epi = &epi;
  g.out = out;
  g.out_dtype = out_dtype;
  g.ldo = N;
  g.M = M;
  g.N = N;
  g.K = K;
  g.cfg = cfg;
  g.sfa = a_scales;
  g.sfb = b_scales;
  return finish(gemm_launch(g, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
