/*
 * Scalar C restatement of the reference's eager W8A8 path -- TEST
 * INFRASTRUCTURE ONLY (an independent cross-check of oracle/eager.py; the
 * product library never links it).
 *
 * bf16 values travel as their uint16 bit patterns.  Each function names the
 * reference lines it restates (paths relative to the reference repository).
 * Build: make -C oracle   ->  oracle/_build/libref_w8a8.so
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static float bf16_to_f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* round-to-nearest-even fp32 -> bf16 (finite inputs) */
static uint16_t f_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float round_bf16(float f) { return bf16_to_f(f_to_bf16(f)); }

/* inference/src/eager.rs:159-171 (quantize_int8_rowwise, seed <= 0):
 * scale = max(amax / 127, 1e-30) in fp32; q = clamp(rne(bf16(x / bf16(scale)))) */
void ref_quantize_rowwise_bf16(const uint16_t* x, int64_t rows, int64_t cols, int8_t* q,
                               float* scale) {
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * cols;
    float amax = 0.0f;
    for (int64_t c = 0; c < cols; ++c) {
      float v = fabsf(bf16_to_f(xr[c]));
      if (v > amax) amax = v;
    }
    float s = amax / 127.0f;
    if (s < 1e-30f) s = 1e-30f;
    scale[r] = s;
    float d = round_bf16(s);
    if (d == 0.0f) d = 1.17549435e-38f; /* finfo(bfloat16).tiny, eager.rs:94-109 */
    for (int64_t c = 0; c < cols; ++c) {
      float t = round_bf16(bf16_to_f(xr[c]) / d);
      t = rintf(t);
      if (t < -128.0f) t = -128.0f;
      if (t > 127.0f) t = 127.0f;
      q[r * cols + c] = (int8_t)t;
    }
  }
}

/* inference/src/int8_linear.rs:134-168: exact int32 accumulate of a . w^T */
void ref_int8_gemm(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                   int32_t* acc) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      int64_t s = 0;
      for (int64_t t = 0; t < k; ++t) s += (int64_t)a[i * k + t] * (int64_t)w[j * k + t];
      acc[i * n + j] = (int32_t)s;
    }
}

/* inference/src/int8_linear.rs:244-268 (bf16 out): y = bf16(acc * (xs * ws));
 * y = bf16(y + bias) */
void ref_dequant_eager_bf16(const int32_t* acc, const float* xs, const float* ws, int64_t ws_numel,
                            const uint16_t* bias, int64_t m, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      const float sc = xs[i] * ws[ws_numel == 1 ? 0 : j];
      float y = round_bf16((float)acc[i * n + j] * sc);
      if (bias) y = round_bf16(y + bf16_to_f(bias[j]));
      out[i * n + j] = f_to_bf16(y);
    }
}

/* e4m3fn encoding of a finite |v| <= 448, round to nearest even (what
 * torch's float -> float8_e4m3fn cast does for clamped inputs). */
static uint8_t f_to_e4m3(float v) {
  uint8_t sign = 0;
  if (v < 0 || (v == 0 && signbit(v))) {
    sign = 0x80;
    v = -v;
  }
  if (v == 0.0f) return sign;
  /* candidate codes are 0x00..0x7E; pick the nearest, ties to even code */
  int e;
  frexpf(v, &e); /* v = f * 2^e, f in [0.5, 1) */
  int exp_unb = e - 1;           /* v in [2^exp_unb, 2^(exp_unb+1)) */
  double step;
  int base_code;
  if (exp_unb < -6) { /* subnormal range: step 2^-9 */
    step = ldexp(1.0, -9);
    double units = v / step;
    double r = nearbyint(units); /* ties to even under default rounding */
    int code = (int)r;           /* 0..8 (8 = smallest normal 2^-6) */
    return (uint8_t)(sign | code);
  }
  step = ldexp(1.0, exp_unb - 3);
  double units = v / step; /* in [8, 16) */
  double r = nearbyint(units);
  int mant = (int)r - 8;
  int ebias = exp_unb + 7;
  if (mant == 8) {
    mant = 0;
    ebias += 1;
  }
  base_code = (ebias << 3) | mant;
  if (base_code > 0x7E) base_code = 0x7E;
  return (uint8_t)(sign | base_code);
}

/* inference/src/eager.rs:74-88: e4m3(clamp(bf16(x * bf16(1/scale)), +-448)) */
void ref_quantize_fp8_bf16(const uint16_t* x, int64_t numel, float scale, uint8_t* out) {
  const float recip = round_bf16(1.0f / scale);
  for (int64_t i = 0; i < numel; ++i) {
    float t = round_bf16(bf16_to_f(x[i]) * recip);
    if (t > 448.0f) t = 448.0f;
    if (t < -448.0f) t = -448.0f;
    out[i] = f_to_e4m3(t);
  }
}

/* inference/src/eager.rs:176-225 + block_scales.rs:4-31 (bf16 input,
 * cols % 32 == 0): payload [rows, cols], scales in the blocked layout
 * [ceil(rows/128)*128, ceil(cols/128)*4]. */
void ref_quantize_mxfp8_bf16(const uint16_t* x, int64_t rows, int64_t cols, uint8_t* q,
                             uint8_t* sf) {
  const int64_t nkb = cols / 32, ncb = (nkb + 3) / 4;
  const int64_t rows_pad = (rows + 127) / 128 * 128;
  memset(sf, 0, (size_t)(rows_pad * ncb * 4));
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t kb = 0; kb < nkb; ++kb) {
      const uint16_t* xb = x + r * cols + kb * 32;
      float amax = 0.0f;
      for (int j = 0; j < 32; ++j) {
        float v = fabsf(bf16_to_f(xb[j]));
        if (v > amax) amax = v;
      }
      int e = 0;
      float scale_f = 1.0f;
      if (amax != 0.0f) {
        float need = amax / 448.0f;
        if (need < ldexpf(1.0f, -127)) need = ldexpf(1.0f, -127);
        e = (int)ceil(log2((double)need)) + 127;
        if (e < 0) e = 0;
        if (e > 254) e = 254;
        scale_f = ldexpf(1.0f, e - 127);
      }
      for (int j = 0; j < 32; ++j) {
        float t = amax != 0.0f ? bf16_to_f(xb[j]) / scale_f : 0.0f;
        if (t > 448.0f) t = 448.0f;
        if (t < -448.0f) t = -448.0f;
        q[r * cols + kb * 32 + j] = f_to_e4m3(t);
      }
      const int64_t blk = (r / 128) * ncb + kb / 4;
      sf[blk * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (kb % 4)] = (uint8_t)e;
    }
}

/* ---- fused input activation + ConvRot quantiser --------------------------
 * Follows native/comfy-port/kitchen/int8_linear.cu:1197-1314
 * (quantize_int8_rowwise_convrot64_kernel), its FHT stages :881-934 and
 * butterfly rows :253-261, its activations :1175-1200 and :1239-1267, and the
 * element step quant_div_float_to_float :53-57.  x holds the fp32 values of
 * the input elements; dtype is the input dtype code (0 f32, 1 f16, 2 bf16),
 * which sets every rounding to "T".  With eager scales (kitchen = 0), or
 * rotate = 0, the activation restates the unfused sequence instead: the ATen
 * activation of inference/src/int8_linear.rs:37-97, each op rounded to T. */
static float round_t(float v, int dtype) {
  if (dtype == 2) return round_bf16(v);
  if (dtype == 1) return (float)(_Float16)v;
  return v;
}

/* in-place normalised 256-point Hadamard transform of one group: digit
 * strides 1, 4, 16, 64, each output 0.5 * (sum left to right) */
void ref_fht256(float* v) {
  float t[256];
  for (int s = 1; s <= 64; s *= 4) {
    for (int i = 0; i < 256; ++i) {
      const int d = (i / s) & 3, base = i - d * s;
      const float x0 = v[base], x1 = v[base + s], x2 = v[base + 2 * s], x3 = v[base + 3 * s];
      float y;
      switch (d) {
        case 0: y = x0 + x1 + x2 - x3; break;
        case 1: y = x0 + x1 - x2 + x3; break;
        case 2: y = x0 - x1 + x2 + x3; break;
        default: y = -x0 + x1 + x2 + x3; break;
      }
      t[i] = 0.5f * y;
    }
    memcpy(v, t, sizeof(t));
  }
}

static float act_one(int act, int fp32, int dtype, float g, float u) {
  /* fp32: no rounding (the fused kernel with kitchen scales); else each ATen
   * op rounds to T (the eager route) */
#define RT(v) (fp32 ? (v) : round_t((v), dtype))
  switch (act) {
    case 1: return RT(0.5f * g * (1.0f + tanhf(0.7978845608028654f * (g + 0.044715f * g * g * g))));
    case 2: return RT(RT(g / (1.0f + expf(-g))) * u);
    case 4: {
      const float a = RT(25.0f * RT(tanhf(RT(g / 25.0f))));
      const float t4 = RT(4.0f * RT(tanhf(RT(u / 4.0f))));
      const float gated = RT(t4 * RT(1.0f / (1.0f + expf(-u))));
      return RT(a * gated);
    }
    default: return g;
  }
#undef RT
}

/* Row quantiser of the fused kernel on already pre-transformed fp32 values v
 * (rotated first when rotate != 0). */
static void quant_row(float* v, int64_t k, int dtype, int rotate, int kitchen, int8_t* q,
                      float* scale) {
  const float finite = dtype == 2 ? 3.3895313892515355e38f : dtype == 1 ? 65504.0f : 3.4028234663852886e38f;
  const float tiny = dtype == 1 ? 6.103515625e-05f : 1.1754943508222875e-38f;
  if (rotate) for (int64_t g = 0; g < k / 256; ++g) ref_fht256(v + g * 256);
  float amax = 0.0f;
  for (int64_t c = 0; c < k; ++c) amax = fmaxf(amax, fabsf(v[c]));
  float s;
  if (kitchen) {
    s = fmaxf(fminf(amax, finite) * (1.0f / 127.0f), 1.0e-30f);
  } else {
    s = fmaxf(round_t(amax, dtype) / 127.0f, 1.0e-30f);
  }
  *scale = s;
  float d = round_t(s, dtype);
  if (d == 0.0f) d = tiny;
  for (int64_t c = 0; c < k; ++c) {
    float t = rintf(round_t(round_t(v[c], dtype) / d, dtype));
    if (t < -128.0f) t = -128.0f;
    if (t > 127.0f) t = 127.0f;
    q[c] = (int8_t)t;
  }
}

void ref_quantize_act_rot(const float* x, int dtype, int64_t rows, int64_t k, int64_t ldx,
                          int rotate, int act, const float* act_w, float eps, int kitchen,
                          int8_t* q, float* scale) {
  float* v = (float*)malloc(sizeof(float) * (size_t)k);
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * ldx;
    if (act == 3) {
      float ss = 0.0f;
      for (int64_t c = 0; c < k; ++c) ss += xr[c] * xr[c];
      const float rstd = 1.0f / sqrtf(ss / (float)k + eps);
      for (int64_t c = 0; c < k; ++c) {
        const float t = xr[c] * rstd * act_w[c];
        v[c] = (rotate && kitchen) ? t : round_t(t, dtype);
      }
    } else {
      for (int64_t c = 0; c < k; ++c) {
        v[c] = act_one(act, rotate && kitchen, dtype, xr[c], (act == 2 || act == 4) ? xr[k + c] : 0.0f);
      }
    }
    quant_row(v, k, dtype, rotate, kitchen, q + r * k, scale + r);
  }
  free(v);
}

/* Modulations before the linear (mode 0 x*(1+s), 1 rms_norm(x,w)*(1+s),
 * 2 layer_norm(x)*(1+s)+shift, 3 rms_norm(x)*(1+s)+shift).  kitchen: the
 * reference CUDA adaln (KSRC backends/cuda/ops/adaln.cu:103-190): one-pass
 * E[x], E[x^2] statistics, fp32 expression, one rounding.  eager: the ATen
 * sequence (inference/src/backend_eager.rs:176-197, backend_bindings.rs:
 * 329-405): two-pass variance, normalised row rounded, times T(1+s) rounded,
 * plus shift rounded.  Row r uses modulation row r / mod_group. */
void ref_quantize_modulated(const float* x, int dtype, int64_t rows, int64_t k, int mode,
                            const float* norm_w, float eps, const float* mscale,
                            const float* mshift, int64_t mod_group, int rotate, int kitchen,
                            int8_t* q, float* scale) {
  float* v = (float*)malloc(sizeof(float) * (size_t)k);
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * k;
    const float* sc = mscale + (r / mod_group) * k;
    const float* sh = mshift ? mshift + (r / mod_group) * k : NULL;
    float mean = 0.0f, rstd = 1.0f;
    if (mode == 1 || mode == 3) {
      float ss = 0.0f;
      for (int64_t c = 0; c < k; ++c) ss += xr[c] * xr[c];
      rstd = 1.0f / sqrtf(ss / (float)k + eps);
    } else if (mode == 2) {
      float s1 = 0.0f;
      for (int64_t c = 0; c < k; ++c) s1 += xr[c];
      mean = s1 / (float)k;
      if (kitchen) {
        float s2 = 0.0f;
        for (int64_t c = 0; c < k; ++c) s2 += xr[c] * xr[c];
        rstd = 1.0f / sqrtf(fmaxf(s2 / (float)k - mean * mean, 0.0f) + eps);
      } else {
        float s2 = 0.0f;
        for (int64_t c = 0; c < k; ++c) s2 += (xr[c] - mean) * (xr[c] - mean);
        rstd = 1.0f / sqrtf(s2 / (float)k + eps);
      }
    }
    for (int64_t c = 0; c < k; ++c) {
      float y;
      if (mode == 0) {
        y = xr[c] * round_t(1.0f + sc[c], dtype);
      } else if (mode == 1) {
        y = round_t(xr[c] * rstd * norm_w[c], dtype) * round_t(1.0f + sc[c], dtype);
      } else {
        const float nrm = (xr[c] - mean) * rstd;
        if (kitchen) {
          y = fmaf(nrm, 1.0f + sc[c], sh[c]);
        } else {
          y = round_t(round_t(nrm, dtype) * round_t(1.0f + sc[c], dtype), dtype) + sh[c];
        }
      }
      v[c] = round_t(y, dtype);
    }
    quant_row(v, k, dtype, rotate, kitchen, q + r * k, scale + r);
  }
  free(v);
}
