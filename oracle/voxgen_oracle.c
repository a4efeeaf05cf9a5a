/*
 * voxgen_oracle.c — CPU restatement of VoxGen's BaseLM decode step.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
 * baseline. Nothing in the product links it.
 *
 * Each function below restates one reference shader in the arithmetic order of
 * its normal (non-_xtx7900) variant: per-lane strided partial sums over the
 * shader's workgroup size followed by the same shared-memory tree reduction,
 * fp32 throughout, mul and add kept separate (built with -ffp-contract=off).
 * Citations are file:line inside the VoxGen project.
 *
 * Parity status: pinned bit for bit against the reference's own shader code
 * (compiled as C++ by oracle/ref_shim) and its known-answer tests.
 */
#include "voxgen_oracle.h"

#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define GGML_F32 0
#define GGML_F16 1
#define GGML_Q8_0 8

/* ------------------------------------------------------------------------ */
/* IEEE binary16 <-> binary32 (unpackHalf2x16 / packHalf2x16 semantics).     */
/* ------------------------------------------------------------------------ */
float vgo_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: value = man * 2^-24, exactly representable in fp32 */
      float v = (float)man * 5.9604644775390625e-08f;
      memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* float -> half, round to nearest even (packHalf2x16 as implemented by
 * conforming drivers; store_kv.comp:22-23). */
uint16_t vgo_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf or nan */
    return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  }
  if (ax >= 0x477FF000u) { /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7C00u);
  }
  if (ax < 0x38800000u) { /* below the smallest normal half (2^-14): subnormal */
    if (ax < 0x33000000u) return (uint16_t)sign; /* < 2^-25 rounds to zero */
    uint32_t e = ax >> 23;                 /* biased fp32 exponent */
    uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
    uint32_t shift = 126u - e;             /* bring to units of 2^-24 */
    /* value = m * 2^(e-150); half subnormal unit = 2^-24 => q = m >> (126-e) */
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 112u; /* rebias 127 -> 15 */
  uint32_t m = ax & 0x7FFFFFu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q += 1u; /* carry may bump exponent */
  return (uint16_t)(sign | q);
}

static inline float ld_f16(const uint8_t *p) {
  uint16_t h;
  memcpy(&h, p, 2);
  return vgo_half_to_float(h);
}

/* Dequantised weight (row, col) of a GGUF matrix: load_weight,
 * matvec.comp:32-44 / embedding.comp:28-41 / qkv_matvec.comp:40-51. */
static inline float load_weight(int dtype, const uint8_t *w, uint32_t cols, uint32_t row,
                                uint32_t col) {
  if (dtype == GGML_F16) return ld_f16(w + ((size_t)row * cols + col) * 2u);
  size_t block = (size_t)row * (cols / 32u) + col / 32u;
  const uint8_t *base = w + block * 34u;
  float d = ld_f16(base);
  int q = (int8_t)base[2u + (col & 31u)];
  return d * (float)q;
}

/* Whole dequantised row into buf (same values as load_weight). */
static void load_row(int dtype, const uint8_t *w, uint32_t cols, uint32_t row, float *buf) {
  if (dtype == GGML_F16) {
    const uint8_t *p = w + (size_t)row * cols * 2u;
    for (uint32_t c = 0; c < cols; ++c) buf[c] = ld_f16(p + 2u * c);
    return;
  }
  const uint8_t *p = w + (size_t)row * (cols / 32u) * 34u;
  for (uint32_t b = 0; b < cols / 32u; ++b) {
    float d = ld_f16(p + (size_t)b * 34u);
    const int8_t *q = (const int8_t *)(p + (size_t)b * 34u + 2u);
    for (uint32_t k = 0; k < 32u; ++k) buf[b * 32u + k] = d * (float)q[k];
  }
}

/* sum_{col = lane; col < cols; col += 256} w[col]*x[col] per lane, then the
 * shared-memory tree (stride 128 .. 1): matvec.comp:51-60,
 * qkv_matvec.comp:80-89, matvec_swiglu.comp:48-64. */
static float dot256(const float *wrow, const float *x, uint32_t cols) {
  float partial[256];
  for (uint32_t lane = 0; lane < 256u; ++lane) partial[lane] = 0.0f;
  for (uint32_t c0 = 0; c0 < cols; c0 += 256u) {
    uint32_t n = cols - c0 < 256u ? cols - c0 : 256u;
    for (uint32_t lane = 0; lane < n; ++lane) partial[lane] += wrow[c0 + lane] * x[c0 + lane];
  }
  for (uint32_t stride = 128u; stride > 0u; stride >>= 1u)
    for (uint32_t lane = 0; lane < stride; ++lane) partial[lane] += partial[lane + stride];
  return partial[0];
}

static int g_threads = 0;
void vgo_set_threads(int n) { g_threads = n; }
int vgo_get_threads(void) {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

/* matvec.comp:46-62: y[row] = partial[0] * alpha. */
void vgo_matvec(int dtype, const uint8_t *w, uint32_t rows, uint32_t cols, const float *x,
                float *y, float alpha) {
#pragma omp parallel num_threads(vgo_get_threads())
  {
    float *buf = (float *)malloc(sizeof(float) * cols);
#pragma omp for schedule(static)
    for (long r = 0; r < (long)rows; ++r) {
      load_row(dtype, w, cols, (uint32_t)r, buf);
      y[r] = dot256(buf, x, cols) * alpha;
    }
    free(buf);
  }
}

/* qkv_matvec.comp:53-95: same per-row sum, written without alpha. */
static void qkv_matvec(int dtype_q, const uint8_t *wq, int dtype_k, const uint8_t *wk,
                       int dtype_v, const uint8_t *wv, uint32_t q_rows, uint32_t kv_rows,
                       uint32_t cols, const float *x, float *q, float *k, float *v) {
  uint32_t total = q_rows + 2u * kv_rows;
#pragma omp parallel num_threads(vgo_get_threads())
  {
    float *buf = (float *)malloc(sizeof(float) * cols);
#pragma omp for schedule(static)
    for (long cr = 0; cr < (long)total; ++cr) {
      uint32_t r = (uint32_t)cr;
      if (r < q_rows) {
        load_row(dtype_q, wq, cols, r, buf);
        q[r] = dot256(buf, x, cols);
      } else if (r < q_rows + kv_rows) {
        load_row(dtype_k, wk, cols, r - q_rows, buf);
        k[r - q_rows] = dot256(buf, x, cols);
      } else {
        load_row(dtype_v, wv, cols, r - q_rows - kv_rows, buf);
        v[r - q_rows - kv_rows] = dot256(buf, x, cols);
      }
    }
    free(buf);
  }
}

/* matvec_swiglu.comp:44-69: y = (g / (1 + exp(-g))) * u. */
void vgo_swiglu(int dtype, const uint8_t *wg, const uint8_t *wu, uint32_t rows, uint32_t cols,
                const float *x, float *y) {
#pragma omp parallel num_threads(vgo_get_threads())
  {
    float *bg = (float *)malloc(sizeof(float) * cols);
    float *bu = (float *)malloc(sizeof(float) * cols);
#pragma omp for schedule(static)
    for (long r = 0; r < (long)rows; ++r) {
      load_row(dtype, wg, cols, (uint32_t)r, bg);
      load_row(dtype, wu, cols, (uint32_t)r, bu);
      float g = dot256(bg, x, cols);
      float u = dot256(bu, x, cols);
      y[r] = (g / (1.0f + expf(-g))) * u;
    }
    free(bg);
    free(bu);
  }
}

/* embedding.comp:43-48: hidden[i] = load_weight(token, i) * alpha. */
void vgo_embedding(int dtype, const uint8_t *w, uint32_t cols, uint32_t token, float alpha,
                   float *hidden) {
  for (uint32_t i = 0; i < cols; ++i) hidden[i] = load_weight(dtype, w, cols, token, i) * alpha;
}

/* Lane-strided sum of squares over 256 lanes + tree (rmsnorm.comp:23-33). */
static float sumsq256(const float *x, uint32_t n) {
  float partial[256];
  for (uint32_t lane = 0; lane < 256u; ++lane) {
    float s = 0.0f;
    for (uint32_t i = lane; i < n; i += 256u) s += x[i] * x[i];
    partial[lane] = s;
  }
  for (uint32_t stride = 128u; stride > 0u; stride >>= 1u)
    for (uint32_t lane = 0; lane < stride; ++lane) partial[lane] += partial[lane + stride];
  return partial[0];
}

/* rmsnorm.comp:21-42; inversesqrt(v) is taken as 1/sqrt(v). */
void vgo_rmsnorm(const float *x, const float *w, uint32_t n, float eps, float *y) {
  float inv_rms = 1.0f / sqrtf(sumsq256(x, n) / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) y[i] = x[i] * inv_rms * w[i];
}

/* residual_rmsnorm.comp:23-42. */
void vgo_residual_rmsnorm(float *hidden, const float *branch, const float *w, uint32_t n,
                          float eps, float scale, float *y) {
  for (uint32_t i = 0; i < n; ++i) hidden[i] = hidden[i] + branch[i] * scale;
  float inv_rms = 1.0f / sqrtf(sumsq256(hidden, n) / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) y[i] = hidden[i] * inv_rms * w[i];
}

/* rope.comp:22-51: NeoX half split, pair i rotates (i, i + d/2). */
void vgo_rope(float *q, float *k, const float *ext, uint32_t position, uint32_t q_heads,
              uint32_t kv_heads, uint32_t head_dim, float theta, float scaling) {
  uint32_t half_dim = head_dim / 2u;
  for (uint32_t head = 0; head < q_heads + kv_heads; ++head) {
    for (uint32_t pair = 0; pair < half_dim; ++pair) {
      float e = ext[pair];
      float exponent = (float)(pair * 2u) / (float)head_dim;
      float inv_freq = 1.0f / powf(theta, exponent);
      float angle = (float)position * inv_freq / e;
      float c = cosf(angle) * scaling;
      float s = sinf(angle) * scaling;
      float *v = head < q_heads ? q + head * head_dim : k + (head - q_heads) * head_dim;
      float a = v[pair];
      float b = v[pair + half_dim];
      v[pair] = a * c - b * s;
      v[pair + half_dim] = b * c + a * s;
    }
  }
}

/* attn_scores.comp:27-44 + softmax.comp:15-47 + attn_values.comp:25-37 for one layer.
 * k_cache / v_cache: [ctx][kv_dim] fp16 bits (the layer's slice of the reference cache).
 * scores: [heads][ctx] fp32 (normalised probabilities on return). */
void vgo_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                   uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t ctx,
                   uint32_t position, float *scores, float *out) {
  uint32_t kv_dim = kv_heads * head_dim;
  uint32_t q_per_kv = heads / kv_heads;
  float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel for collapse(2) schedule(static) num_threads(vgo_get_threads())
  for (long qh = 0; qh < (long)heads; ++qh) {
    for (long t = 0; t <= (long)position; ++t) {
      /* 128-lane workgroup: lane j holds q*k for dim j (dims >= 128 wrap onto
       * lanes by stride 128; lanes >= head_dim contribute 0), tree 64..1. */
      float partial[128];
      uint32_t kvh = (uint32_t)qh / q_per_kv;
      for (uint32_t lane = 0; lane < 128u; ++lane) {
        float p = 0.0f;
        for (uint32_t d = lane; d < head_dim; d += 128u)
          p += q[qh * head_dim + d] *
               vgo_half_to_float(k_cache[(size_t)t * kv_dim + kvh * head_dim + d]);
        partial[lane] = p;
      }
      for (uint32_t stride = 64u; stride > 0u; stride >>= 1u)
        for (uint32_t lane = 0; lane < stride; ++lane) partial[lane] += partial[lane + stride];
      scores[qh * ctx + t] = partial[0] * scale;
    }
  }
  for (uint32_t head = 0; head < heads; ++head) {
    float *s = scores + (size_t)head * ctx;
    float scratch[256];
    for (uint32_t lane = 0; lane < 256u; ++lane) {
      float m = -3.402823466e+38f;
      for (uint32_t t = lane; t <= position; t += 256u) m = fmaxf(m, s[t]);
      scratch[lane] = m;
    }
    for (uint32_t stride = 128u; stride > 0u; stride >>= 1u)
      for (uint32_t lane = 0; lane < stride; ++lane)
        scratch[lane] = fmaxf(scratch[lane], scratch[lane + stride]);
    float gmax = scratch[0];
    for (uint32_t lane = 0; lane < 256u; ++lane) {
      float sum = 0.0f;
      for (uint32_t t = lane; t <= position; t += 256u) sum += expf(s[t] - gmax);
      scratch[lane] = sum;
    }
    for (uint32_t stride = 128u; stride > 0u; stride >>= 1u)
      for (uint32_t lane = 0; lane < stride; ++lane) scratch[lane] += scratch[lane + stride];
    float inv_sum = 1.0f / scratch[0];
    for (uint32_t t = 0; t <= position; ++t) s[t] = expf(s[t] - gmax) * inv_sum;
  }
#pragma omp parallel for collapse(2) schedule(static) num_threads(vgo_get_threads())
  for (long qh = 0; qh < (long)heads; ++qh) {
    for (long d = 0; d < (long)head_dim; ++d) {
      uint32_t kvh = (uint32_t)qh / q_per_kv;
      float acc = 0.0f;
      for (uint32_t t = 0; t <= position; ++t)
        acc += scores[qh * ctx + t] *
               vgo_half_to_float(v_cache[(size_t)t * kv_dim + kvh * head_dim + d]);
      out[qh * head_dim + d] = acc;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* RX 7900 XTX mode: the _xtx7900 shader variants (baselm.rs:515-546, :1241). */
/* A lane sums its strided share in order; a workgroup reduction is a wave32   */
/* subgroup sum per wave, the waves' sums in shared memory, then one more      */
/* subgroup sum in wave 0 over waves[i] (i < number of waves, else 0). The     */
/* order inside a subgroup sum is not fixed by GLSL; it is taken as the        */
/* balanced pairwise tree over the 32 invocations (what a shuffle-xor          */
/* butterfly computes), the same assumption as the shader emulation that pins  */
/* this restatement.                                                           */
/* ------------------------------------------------------------------------ */
static float xtx_tree32(float *t, int is_max) {
  for (int st = 1; st < 32; st <<= 1)
    for (int i = 0; i < 32; i += 2 * st) t[i] = is_max ? (t[i] < t[i + st] ? t[i + st] : t[i]) : t[i] + t[i + st];
  return t[0];
}
/* reduce_sum / red / rmax of the xtx shaders over nl (128 or 256) lane values */
static float xtx_reduce(const float *lanes, uint32_t nl, int is_max) {
  float waves[8], t[32];
  const uint32_t nw = nl / 32u;
  for (uint32_t w = 0; w < nw; ++w) {
    for (int i = 0; i < 32; ++i) t[i] = lanes[w * 32u + i];
    waves[w] = xtx_tree32(t, is_max);
  }
  for (uint32_t i = 0; i < 32u; ++i) t[i] = i < nw ? waves[i] : (is_max ? -3.402823466e+38f : 0.0f);
  return xtx_tree32(t, is_max);
}
/* One lane's sum of a row (matvec_xtx7900.comp:14-15): columns 4 lane .. 4 lane + 3,
 * then + 1024; Q8_0 as d * (q0 x0 + q1 x1 + q2 x2 + q3 x3), F16 element by element. */
static float xtx_lane(int dtype, const uint8_t *w, uint32_t cols, uint32_t row, const float *x,
                      uint32_t lane) {
  float s = 0.0f;
  for (uint32_t c = lane * 4u; c < cols; c += 1024u) {
    if (dtype == GGML_F16) {
      const uint8_t *rb = w + (size_t)row * cols * 2u + (size_t)c * 2u;
      s += ld_f16(rb) * x[c];
      if (c + 1u < cols) s += ld_f16(rb + 2) * x[c + 1u];
      if (c + 2u < cols) s += ld_f16(rb + 4) * x[c + 2u];
      if (c + 3u < cols) s += ld_f16(rb + 6) * x[c + 3u];
    } else {
      const uint8_t *base = w + ((size_t)row * (cols / 32u) + c / 32u) * 34u;
      const float d = ld_f16(base);
      const int8_t *q = (const int8_t *)(base + 2u + (c & 31u));
      s += d * ((float)q[0] * x[c] + (float)q[1] * x[c + 1u] + (float)q[2] * x[c + 2u] +
                (float)q[3] * x[c + 3u]);
    }
  }
  return s;
}
static float xtx_dot(int dtype, const uint8_t *w, uint32_t cols, uint32_t row, const float *x) {
  float lanes[256];
  for (uint32_t lane = 0; lane < 256u; ++lane) lanes[lane] = xtx_lane(dtype, w, cols, row, x, lane);
  return xtx_reduce(lanes, 256u, 0);
}

/* matvec_xtx7900.comp: y[row] = total * alpha. */
void vgo_matvec_xtx(int dtype, const uint8_t *w, uint32_t rows, uint32_t cols, const float *x,
                    float *y, float alpha) {
#pragma omp parallel for schedule(static) num_threads(vgo_get_threads())
  for (long r = 0; r < (long)rows; ++r) y[r] = xtx_dot(dtype, w, cols, (uint32_t)r, x) * alpha;
}

/* qkv_matvec_xtx7900.comp: the same row sums, written without alpha. */
static void qkv_matvec_xtx(int dtype_q, const uint8_t *wq, int dtype_k, const uint8_t *wk,
                           int dtype_v, const uint8_t *wv, uint32_t q_rows, uint32_t kv_rows,
                           uint32_t cols, const float *x, float *q, float *k, float *v) {
  const long total = (long)q_rows + 2L * kv_rows;
#pragma omp parallel for schedule(static) num_threads(vgo_get_threads())
  for (long cr = 0; cr < total; ++cr) {
    const uint32_t r = (uint32_t)cr;
    if (r < q_rows) q[r] = xtx_dot(dtype_q, wq, cols, r, x);
    else if (r < q_rows + kv_rows) k[r - q_rows] = xtx_dot(dtype_k, wk, cols, r - q_rows, x);
    else v[r - q_rows - kv_rows] = xtx_dot(dtype_v, wv, cols, r - q_rows - kv_rows, x);
  }
}

/* matvec_swiglu_xtx7900.comp: gate and up summed together per lane (vec2), Q8_0 as
 * the sum of four (d q x) terms added to the lane's sum; y = (g / (1 + exp(-g))) * u. */
void vgo_swiglu_xtx(int dtype, const uint8_t *wg, const uint8_t *wu, uint32_t rows, uint32_t cols,
                    const float *x, float *y) {
#pragma omp parallel for schedule(static) num_threads(vgo_get_threads())
  for (long r = 0; r < (long)rows; ++r) {
    float lg[256], lu[256];
    for (uint32_t lane = 0; lane < 256u; ++lane) {
      float sg = 0.0f, su = 0.0f;
      for (uint32_t c = lane * 4u; c < cols; c += 1024u) {
        if (dtype == GGML_F16) {
          const uint8_t *gr = wg + ((size_t)r * cols + c) * 2u, *ur = wu + ((size_t)r * cols + c) * 2u;
          for (uint32_t j = 0; j < 4u; ++j) {
            if (c + j >= cols) break;
            const float xj = x[c + j];
            sg += ld_f16(gr + 2u * j) * xj;
            su += ld_f16(ur + 2u * j) * xj;
          }
        } else {
          const size_t blk = ((size_t)r * (cols / 32u) + c / 32u) * 34u;
          const float gd = ld_f16(wg + blk), ud = ld_f16(wu + blk);
          const int8_t *gq = (const int8_t *)(wg + blk + 2u + (c & 31u));
          const int8_t *uq = (const int8_t *)(wu + blk + 2u + (c & 31u));
          float tg = gd * (float)gq[0] * x[c], tu = ud * (float)uq[0] * x[c];
          for (uint32_t j = 1; j < 4u; ++j) {
            tg = tg + gd * (float)gq[j] * x[c + j];
            tu = tu + ud * (float)uq[j] * x[c + j];
          }
          sg += tg;
          su += tu;
        }
      }
      lg[lane] = sg;
      lu[lane] = su;
    }
    const float g = xtx_reduce(lg, 256u, 0), u = xtx_reduce(lu, 256u, 0);
    y[r] = (g / (1.0f + expf(-g))) * u;
  }
}

/* rmsnorm_xtx7900.comp / residual_rmsnorm_xtx7900.comp: lane-strided sums of
 * squares (stride 256), the wave reduction, then x * inv_rms * w. */
static float xtx_sumsq(const float *x, uint32_t n) {
  float lanes[256];
  for (uint32_t lane = 0; lane < 256u; ++lane) {
    float s = 0.0f;
    for (uint32_t k = lane; k < n; k += 256u) s += x[k] * x[k];
    lanes[lane] = s;
  }
  return xtx_reduce(lanes, 256u, 0);
}
void vgo_rmsnorm_xtx(const float *x, const float *w, uint32_t n, float eps, float *y) {
  const float inv = 1.0f / sqrtf(xtx_sumsq(x, n) / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
}
void vgo_residual_rmsnorm_xtx(float *hidden, const float *branch, const float *w, uint32_t n,
                              float eps, float scale, float *y) {
  for (uint32_t i = 0; i < n; ++i) hidden[i] = hidden[i] + scale * branch[i];
  const float inv = 1.0f / sqrtf(xtx_sumsq(hidden, n) / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) y[i] = hidden[i] * inv * w[i];
}

/* attn_scores_xtx7900.comp (128 lanes, lane = dimension, head_dim <= 128) +
 * softmax_xtx7900.comp (256 lanes, max then sum of exp) + attn_values.comp. */
void vgo_attention_xtx(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                       uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t ctx,
                       uint32_t position, float *scores, float *out) {
  const uint32_t kv_dim = kv_heads * head_dim, q_per_kv = heads / kv_heads;
  const float scale = 1.0f / sqrtf((float)head_dim);
#pragma omp parallel for collapse(2) schedule(static) num_threads(vgo_get_threads())
  for (long qh = 0; qh < (long)heads; ++qh)
    for (long t = 0; t <= (long)position; ++t) {
      float lanes[128];
      const uint32_t kvh = (uint32_t)qh / q_per_kv;
      for (uint32_t lane = 0; lane < 128u; ++lane)
        lanes[lane] = lane < head_dim ? q[qh * head_dim + lane] *
                                            vgo_half_to_float(k_cache[(size_t)t * kv_dim + kvh * head_dim + lane])
                                      : 0.0f;
      scores[qh * ctx + t] = xtx_reduce(lanes, 128u, 0) * scale;
    }
  for (uint32_t head = 0; head < heads; ++head) {
    float *s = scores + (size_t)head * ctx, lanes[256];
    for (uint32_t lane = 0; lane < 256u; ++lane) {
      float m = -3.402823466e+38f;
      for (uint32_t t = lane; t <= position; t += 256u) m = m < s[t] ? s[t] : m;
      lanes[lane] = m;
    }
    const float gmax = xtx_reduce(lanes, 256u, 1);
    for (uint32_t lane = 0; lane < 256u; ++lane) {
      float sum = 0.0f;
      for (uint32_t t = lane; t <= position; t += 256u) sum += expf(s[t] - gmax);
      lanes[lane] = sum;
    }
    const float inv_sum = 1.0f / xtx_reduce(lanes, 256u, 0);
    for (uint32_t t = 0; t <= position; ++t) s[t] = expf(s[t] - gmax) * inv_sum;
  }
#pragma omp parallel for collapse(2) schedule(static) num_threads(vgo_get_threads())
  for (long qh = 0; qh < (long)heads; ++qh)
    for (long d = 0; d < (long)head_dim; ++d) {
      const uint32_t kvh = (uint32_t)qh / q_per_kv;
      float acc = 0.0f;
      for (uint32_t t = 0; t <= position; ++t)
        acc += scores[qh * ctx + t] * vgo_half_to_float(v_cache[(size_t)t * kv_dim + kvh * head_dim + d]);
      out[qh * head_dim + d] = acc;
    }
}
/* ------------------------------------------------------------------------ */
/* GGUF reader: restates load_summary (src/gguf.rs:222-286).                 */
/* ------------------------------------------------------------------------ */
typedef struct {
  char name[96];
  uint32_t n_dims;
  uint64_t dims[8];
  uint32_t type;
  uint64_t offset;
  uint64_t bytes;
  uint64_t elements;
} vgo_tensor;

typedef struct {
  char key[128];
  int kind; /* 0 = number, 1 = string */
  double num;
  char str[128];
} vgo_meta;

struct vgo_model {
  uint8_t *file;
  uint64_t file_bytes;
  uint64_t data_offset;
  vgo_tensor *tensors;
  uint32_t n_tensors;
  vgo_meta *meta;
  uint32_t n_meta;
  /* config (BaseLmConfig::from_gguf, src/baselm.rs:60-180) */
  uint32_t ctx_len, H, L, F, vocab, heads, kv_heads, head_dim, kv_dim, orig_ctx;
  float eps, theta, scaling, emb_scale, res_scale, logit_scale;
  int format, tied, longrope;
  /* per-layer tensors */
  const vgo_tensor **attn_norm, **ffn_norm, **wq, **wk, **wv, **wo, **wg, **wu, **wd;
  const vgo_tensor *tok, *out, *out_norm, *rope_factors;
};

typedef struct {
  const uint8_t *p, *end;
  int ok;
} rdr;

static int take(rdr *r, void *dst, size_t n) {
  if (!r->ok || (size_t)(r->end - r->p) < n) {
    r->ok = 0;
    return 0;
  }
  if (dst) memcpy(dst, r->p, n);
  r->p += n;
  return 1;
}
static uint32_t rd_u32(rdr *r) { uint32_t v = 0; take(r, &v, 4); return v; }
static uint64_t rd_u64(rdr *r) { uint64_t v = 0; take(r, &v, 8); return v; }

static int rd_str(rdr *r, char *dst, size_t cap) {
  uint64_t n = rd_u64(r);
  if (!r->ok || n > (uint64_t)(r->end - r->p)) { r->ok = 0; return 0; }
  if (dst && cap) {
    size_t c = n < cap - 1 ? (size_t)n : cap - 1;
    memcpy(dst, r->p, c);
    dst[c] = 0;
  }
  r->p += n;
  return 1;
}

static void set_err(char *err, size_t len, const char *fmt, ...) {
  if (!err || !len) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, len, fmt, ap);
  va_end(ap);
}

/* read_meta_value (src/gguf.rs:190-220); numbers are kept as doubles. */
static int rd_value(rdr *r, uint32_t ty, int depth, vgo_meta *out) {
  if (depth > 8) { r->ok = 0; return 0; }
  union { uint8_t u8; int8_t i8; uint16_t u16; int16_t i16; uint32_t u32; int32_t i32;
          float f32; uint64_t u64; int64_t i64; double f64; } v;
  v.u64 = 0;
  double num = 0;
  switch (ty) {
    case 0: take(r, &v.u8, 1); num = v.u8; break;
    case 1: take(r, &v.i8, 1); num = v.i8; break;
    case 2: take(r, &v.u16, 2); num = v.u16; break;
    case 3: take(r, &v.i16, 2); num = v.i16; break;
    case 4: take(r, &v.u32, 4); num = v.u32; break;
    case 5: take(r, &v.i32, 4); num = v.i32; break;
    case 6: take(r, &v.f32, 4); num = v.f32; break;
    case 7: take(r, &v.u8, 1); num = v.u8 != 0; break;
    case 8:
      if (out) { out->kind = 1; return rd_str(r, out->str, sizeof out->str); }
      return rd_str(r, NULL, 0);
    case 9: {
      uint32_t et = rd_u32(r);
      uint64_t n = rd_u64(r);
      for (uint64_t i = 0; i < n && r->ok; ++i) rd_value(r, et, depth + 1, NULL);
      if (out) out->kind = 2;
      return r->ok;
    }
    case 10: take(r, &v.u64, 8); num = (double)v.u64; break;
    case 11: take(r, &v.i64, 8); num = (double)v.i64; break;
    case 12: take(r, &v.f64, 8); num = v.f64; break;
    default: r->ok = 0; return 0;
  }
  if (out) { out->kind = 0; out->num = num; }
  return r->ok;
}

static const vgo_meta *find_meta(const vgo_model *m, const char *k) {
  for (uint32_t i = 0; i < m->n_meta; ++i)
    if (!strcmp(m->meta[i].key, k)) return &m->meta[i];
  return NULL;
}
static int meta_num(const vgo_model *m, const char *k, double *v) {
  const vgo_meta *e = find_meta(m, k);
  if (!e || e->kind != 0) return 0;
  *v = e->num;
  return 1;
}
static const vgo_tensor *find_tensor(const vgo_model *m, const char *name) {
  for (uint32_t i = 0; i < m->n_tensors; ++i)
    if (!strcmp(m->tensors[i].name, name)) return &m->tensors[i];
  return NULL;
}

static uint64_t storage_bytes(uint32_t type, uint64_t elements, int *ok) {
  if (type == GGML_F32) return elements * 4u;
  if (type == GGML_F16) return elements * 2u;
  if (type == GGML_Q8_0) {
    if (elements % 32u) { *ok = 0; return 0; }
    return elements / 32u * 34u;
  }
  *ok = 0;
  return 0;
}

static int dims_are(const vgo_tensor *t, uint32_t n, uint64_t d0, uint64_t d1) {
  if (!t || t->n_dims != n || t->dims[0] != d0) return 0;
  return n == 1 || t->dims[1] == d1;
}

int vgo_model_load(const char *path, vgo_model **out, char *err, size_t err_len) {
  *out = NULL;
  FILE *f = fopen(path, "rb");
  if (!f) { set_err(err, err_len, "open %s failed", path); return -2; }
  fseek(f, 0, SEEK_END);
  long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  vgo_model *m = (vgo_model *)calloc(1, sizeof *m);
  m->file = (uint8_t *)malloc((size_t)sz > 0 ? (size_t)sz : 1);
  m->file_bytes = (uint64_t)sz;
  if (fread(m->file, 1, (size_t)sz, f) != (size_t)sz) {
    fclose(f); vgo_model_free(m);
    set_err(err, err_len, "read %s failed", path);
    return -2;
  }
  fclose(f);
  rdr r = {m->file, m->file + sz, 1};
  uint32_t magic = rd_u32(&r);
  if (!r.ok || magic != 0x46554747u) { vgo_model_free(m); set_err(err, err_len, "not a GGUF file"); return -3; }
  uint32_t version = rd_u32(&r);
  if (version < 2 || version > 3) { vgo_model_free(m); set_err(err, err_len, "unsupported GGUF version %u", version); return -3; }
  uint64_t nt = rd_u64(&r), nm = rd_u64(&r);
  if (!r.ok || nt > 200000 || nm > 1000000) { vgo_model_free(m); set_err(err, err_len, "bad GGUF counts"); return -3; }
  m->meta = (vgo_meta *)calloc(nm ? nm : 1, sizeof(vgo_meta));
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < nm && r.ok; ++i) {
    vgo_meta *e = &m->meta[m->n_meta];
    rd_str(&r, e->key, sizeof e->key);
    uint32_t ty = rd_u32(&r);
    rd_value(&r, ty, 0, e);
    if (!r.ok) break;
    if (!strcmp(e->key, "general.alignment") && e->kind == 0 && (ty == 4 || ty == 10))
      alignment = e->num >= 1 ? (uint64_t)e->num : 1;
    m->n_meta++;
  }
  m->tensors = (vgo_tensor *)calloc(nt ? nt : 1, sizeof(vgo_tensor));
  for (uint64_t i = 0; i < nt && r.ok; ++i) {
    vgo_tensor *t = &m->tensors[i];
    rd_str(&r, t->name, sizeof t->name);
    t->n_dims = rd_u32(&r);
    if (!r.ok || t->n_dims == 0 || t->n_dims > 8) { r.ok = 0; break; }
    uint64_t el = 1;
    for (uint32_t d = 0; d < t->n_dims; ++d) {
      t->dims[d] = rd_u64(&r);
      if (t->dims[d] && el > UINT64_MAX / t->dims[d]) { r.ok = 0; break; }
      el *= t->dims[d];
    }
    t->type = rd_u32(&r);
    t->offset = rd_u64(&r);
    int ok = 1;
    t->bytes = storage_bytes(t->type, el, &ok);
    t->elements = el;
    if (!ok) { vgo_model_free(m); set_err(err, err_len, "tensor %s: unsupported type/size", t->name); return -4; }
    m->n_tensors++;
  }
  if (!r.ok) { vgo_model_free(m); set_err(err, err_len, "unexpected EOF while reading GGUF"); return -3; }
  uint64_t pos = (uint64_t)(r.p - m->file);
  m->data_offset = (pos + alignment - 1) / alignment * alignment;
  for (uint32_t i = 0; i < m->n_tensors; ++i) {
    const vgo_tensor *t = &m->tensors[i];
    if (m->data_offset + t->offset + t->bytes > m->file_bytes) {
      set_err(err, err_len, "tensor %s extends beyond end of file", t->name);
      vgo_model_free(m);
      return -3;
    }
  }

  /* ---- config: BaseLmConfig::from_gguf without the fixed-geometry gate ---- */
  const vgo_meta *arch = find_meta(m, "general.architecture");
  if (!arch || arch->kind != 1 || strcmp(arch->str, "minicpm4")) {
    vgo_model_free(m); set_err(err, err_len, "expects general.architecture=minicpm4"); return -4;
  }
  double v;
#define REQ(key, dst) do { if (!meta_num(m, key, &v)) { vgo_model_free(m); set_err(err, err_len, "missing required metadata: %s", key); return -4; } dst = v; } while (0)
  REQ("minicpm4.context_length", m->ctx_len);
  REQ("minicpm4.embedding_length", m->H);
  REQ("minicpm4.block_count", m->L);
  REQ("minicpm4.feed_forward_length", m->F);
  REQ("minicpm4.attention.head_count", m->heads);
  REQ("minicpm4.attention.head_count_kv", m->kv_heads);
  if (meta_num(m, "minicpm4.attention.key_length", &v)) m->head_dim = (uint32_t)v;
  else REQ("minicpm4.rope.dimension_count", m->head_dim);
  uint32_t rope_dim;
  REQ("minicpm4.rope.dimension_count", rope_dim);
  REQ("minicpm4.attention.layer_norm_rms_epsilon", m->eps);
  REQ("minicpm4.rope.freq_base", m->theta);
#undef REQ
  m->orig_ctx = m->ctx_len;
  if (meta_num(m, "minicpm4.rope.scaling.original_context_length", &v)) m->orig_ctx = (uint32_t)v;
  else if (meta_num(m, "minicpm4.rope.scaling.original_context_len", &v)) m->orig_ctx = (uint32_t)v;
  m->emb_scale = meta_num(m, "minicpm4.embedding_scale", &v) ? (float)v : 0.0f;
  m->res_scale = meta_num(m, "minicpm4.residual_scale", &v) ? (float)v : 0.0f;
  m->logit_scale = meta_num(m, "minicpm4.logit_scale", &v) ? (float)v : 0.0f;
  const vgo_meta *st = find_meta(m, "minicpm4.rope.scaling.type");
  m->longrope = st && st->kind == 1 && !strcmp(st->str, "longrope");
  if (m->heads == 0 || m->kv_heads == 0 || m->heads % m->kv_heads || rope_dim != m->head_dim) {
    vgo_model_free(m); set_err(err, err_len, "bad head geometry"); return -4;
  }
  m->kv_dim = m->kv_heads * m->head_dim;
  /* rope_scaling_factor, src/baselm.rs:194-205 */
  if (!m->longrope || m->ctx_len <= m->orig_ctx || m->orig_ctx <= 1) m->scaling = 1.0f;
  else {
    float mx = (float)m->ctx_len, orig = (float)m->orig_ctx;
    m->scaling = sqrtf(1.0f + logf(mx / orig) / logf(orig));
  }
  m->tok = find_tensor(m, "token_embd.weight");
  if (!m->tok || m->tok->n_dims != 2 || m->tok->dims[0] != m->H) {
    vgo_model_free(m); set_err(err, err_len, "token_embd.weight missing or misshaped"); return -4;
  }
  m->vocab = (uint32_t)m->tok->dims[1];
  m->out = find_tensor(m, "output.weight");
  m->tied = m->out == NULL;
  if (m->tied) m->out = m->tok;
  m->out_norm = find_tensor(m, "output_norm.weight");
  if (!dims_are(m->out_norm, 1, m->H, 0) || m->out_norm->type != GGML_F32) {
    vgo_model_free(m); set_err(err, err_len, "output_norm.weight missing or misshaped"); return -4;
  }
  if (m->longrope) {
    /* record_transformer picks the factor set once per model, src/baselm.rs:902-913 */
    m->rope_factors = find_tensor(m, m->ctx_len > m->orig_ctx ? "rope_factors_long.weight"
                                                              : "rope_factors_short.weight");
    if (!dims_are(m->rope_factors, 1, m->head_dim / 2, 0) || m->rope_factors->type != GGML_F32) {
      vgo_model_free(m); set_err(err, err_len, "rope factors missing or misshaped"); return -4;
    }
  }
  size_t L = m->L;
  m->attn_norm = calloc(L, sizeof(void *)); m->ffn_norm = calloc(L, sizeof(void *));
  m->wq = calloc(L, sizeof(void *)); m->wk = calloc(L, sizeof(void *)); m->wv = calloc(L, sizeof(void *));
  m->wo = calloc(L, sizeof(void *)); m->wg = calloc(L, sizeof(void *)); m->wu = calloc(L, sizeof(void *));
  m->wd = calloc(L, sizeof(void *));
  uint64_t q8 = 0, f16 = 0;
  for (uint32_t l = 0; l < m->L; ++l) {
    char nm_[96];
#define GETT(field, suffix, nd, d0, d1, isvec) do { snprintf(nm_, sizeof nm_, "blk.%u." suffix, l); \
      m->field[l] = find_tensor(m, nm_); \
      if (!dims_are(m->field[l], nd, d0, d1) || (isvec ? m->field[l]->type != GGML_F32 : \
          (m->field[l]->type != GGML_F16 && m->field[l]->type != GGML_Q8_0))) { \
        vgo_model_free(m); set_err(err, err_len, "tensor %s missing or misshaped", nm_); return -4; } } while (0)
    GETT(attn_norm, "attn_norm.weight", 1, m->H, 0, 1);
    GETT(ffn_norm, "ffn_norm.weight", 1, m->H, 0, 1);
    GETT(wq, "attn_q.weight", 2, m->H, m->H, 0);
    GETT(wk, "attn_k.weight", 2, m->H, m->kv_dim, 0);
    GETT(wv, "attn_v.weight", 2, m->H, m->kv_dim, 0);
    GETT(wo, "attn_output.weight", 2, m->H, m->H, 0);
    GETT(wg, "ffn_gate.weight", 2, m->H, m->F, 0);
    GETT(wu, "ffn_up.weight", 2, m->H, m->F, 0);
    GETT(wd, "ffn_down.weight", 2, m->F, m->H, 0);
#undef GETT
  }
  for (uint32_t i = 0; i < m->n_tensors; ++i) {
    const vgo_tensor *t = &m->tensors[i];
    /* primary_base_format, src/gguf.rs:117-133 */
    if (t->n_dims < 2 || t->elements < 4096) continue;
    if (t->type == GGML_Q8_0) q8 += t->bytes;
    if (t->type == GGML_F16) f16 += t->bytes;
  }
  m->format = (q8 > 0 && q8 >= f16) ? GGML_Q8_0 : GGML_F16;
  *out = m;
  return 0;
}

void vgo_model_free(vgo_model *m) {
  if (!m) return;
  free(m->file); free(m->tensors); free(m->meta);
  free(m->attn_norm); free(m->ffn_norm); free(m->wq); free(m->wk); free(m->wv);
  free(m->wo); free(m->wg); free(m->wu); free(m->wd);
  free(m);
}

void vgo_model_geometry(const vgo_model *m, uint32_t *o) {
  o[VGO_CTX_LEN] = m->ctx_len; o[VGO_H] = m->H; o[VGO_LAYERS] = m->L; o[VGO_FFN] = m->F;
  o[VGO_VOCAB] = m->vocab; o[VGO_HEADS] = m->heads; o[VGO_KV_HEADS] = m->kv_heads;
  o[VGO_HEAD_DIM] = m->head_dim; o[VGO_KV_DIM] = m->kv_dim; o[VGO_FORMAT] = (uint32_t)m->format;
  o[VGO_TIED] = (uint32_t)m->tied; o[VGO_ORIG_CTX] = m->orig_ctx;
}
void vgo_model_scalars(const vgo_model *m, float *o) {
  o[0] = m->eps; o[1] = m->theta; o[2] = m->scaling; o[3] = m->emb_scale; o[4] = m->res_scale;
  o[5] = m->logit_scale;
}

/* ------------------------------------------------------------------------ */
/* Engine state: BaseLmEngine buffers (src/baselm.rs:484-506).               */
/* ------------------------------------------------------------------------ */
struct vgo_state {
  const vgo_model *m;
  uint32_t ctx, position;
  float *hidden, *norm, *q, *k, *v, *attention, *gate, *branch, *logits, *scores;
  uint16_t *kv_k, *kv_v; /* [layer][ctx][kv_dim] */
  int xtx;               /* record the RX 7900 XTX mode's shader variants */
  char err[256];
};

void vgo_set_xtx(vgo_state *s, int on) { s->xtx = on != 0; }

int vgo_state_create(const vgo_model *m, uint32_t max_context, vgo_state **out) {
  *out = NULL;
  if (max_context == 0 || max_context > m->ctx_len) return -1;
  vgo_state *s = (vgo_state *)calloc(1, sizeof *s);
  s->m = m;
  s->ctx = max_context;
  s->hidden = calloc(m->H, 4); s->norm = calloc(m->H, 4); s->q = calloc(m->H, 4);
  s->k = calloc(m->kv_dim, 4); s->v = calloc(m->kv_dim, 4); s->attention = calloc(m->H, 4);
  s->gate = calloc(m->F, 4); s->branch = calloc(m->H, 4); s->logits = calloc(m->vocab, 4);
  s->scores = calloc((size_t)m->heads * max_context, 4);
  size_t kv = (size_t)m->L * max_context * m->kv_dim;
  s->kv_k = calloc(kv, 2); s->kv_v = calloc(kv, 2);
  if (!s->kv_k || !s->kv_v || !s->scores) { vgo_state_free(s); return -8; }
  *out = s;
  return 0;
}

void vgo_state_free(vgo_state *s) {
  if (!s) return;
  free(s->hidden); free(s->norm); free(s->q); free(s->k); free(s->v); free(s->attention);
  free(s->gate); free(s->branch); free(s->logits); free(s->scores); free(s->kv_k); free(s->kv_v);
  free(s);
}

void vgo_reset(vgo_state *s) { s->position = 0; }
uint32_t vgo_position(const vgo_state *s) { return s->position; }
int vgo_set_position(vgo_state *s, uint32_t pos) {
  if (pos > s->ctx) return -1;
  s->position = pos;
  return 0;
}

int vgo_write_kv(vgo_state *s, const uint16_t *k, const uint16_t *v, uint32_t n) {
  const vgo_model *m = s->m;
  if (n > s->ctx) return -6;
  for (uint32_t l = 0; l < m->L; ++l) {
    memcpy(s->kv_k + ((size_t)l * s->ctx) * m->kv_dim, k + (size_t)l * n * m->kv_dim,
           (size_t)n * m->kv_dim * 2);
    memcpy(s->kv_v + ((size_t)l * s->ctx) * m->kv_dim, v + (size_t)l * n * m->kv_dim,
           (size_t)n * m->kv_dim * 2);
  }
  s->position = n;
  return 0;
}

int vgo_read_kv(const vgo_state *s, uint16_t *k, uint16_t *v, uint32_t n) {
  const vgo_model *m = s->m;
  if (n > s->ctx) return -6;
  for (uint32_t l = 0; l < m->L; ++l) {
    memcpy(k + (size_t)l * n * m->kv_dim, s->kv_k + ((size_t)l * s->ctx) * m->kv_dim,
           (size_t)n * m->kv_dim * 2);
    memcpy(v + (size_t)l * n * m->kv_dim, s->kv_v + ((size_t)l * s->ctx) * m->kv_dim,
           (size_t)n * m->kv_dim * 2);
  }
  return 0;
}

static inline const uint8_t *tdata(const vgo_model *m, const vgo_tensor *t) {
  return m->file + m->data_offset + t->offset;
}
static inline const float *tf32(const vgo_model *m, const vgo_tensor *t) {
  return (const float *)(const void *)tdata(m, t);
}
/* effective_scale, src/baselm.rs:1262-1264 */
static inline float eff(float v) { return v == 0.0f ? 1.0f : v; }

/* record_transformer, src/baselm.rs:892-1052. */
static int record_transformer(vgo_state *s, int compute_logits) {
  const vgo_model *m = s->m;
  uint32_t pos = s->position;
  float rs = eff(m->res_scale);
  if (!m->longrope) {
    snprintf(s->err, sizeof s->err, "MiniCPM4 BaseLM without LongRoPE factors is not enabled");
    return -4;
  }
  const float *ext = tf32(m, m->rope_factors);
  /* the XTX mode swaps rmsnorm, residual_rmsnorm, qkv_matvec, matvec_swiglu,
   * matvec, attn_scores and softmax for their _xtx7900 variants */
  const int x = s->xtx;
  (x ? vgo_rmsnorm_xtx : vgo_rmsnorm)(s->hidden, tf32(m, m->attn_norm[0]), m->H, m->eps, s->norm);
  for (uint32_t l = 0; l < m->L; ++l) {
    (x ? qkv_matvec_xtx : qkv_matvec)((int)m->wq[l]->type, tdata(m, m->wq[l]), (int)m->wk[l]->type,
                                      tdata(m, m->wk[l]), (int)m->wv[l]->type, tdata(m, m->wv[l]), m->H,
                                      m->kv_dim, m->H, s->norm, s->q, s->k, s->v);
    vgo_rope(s->q, s->k, ext, pos, m->heads, m->kv_heads, m->head_dim, m->theta, m->scaling);
    /* store_kv.comp:16-24 */
    uint16_t *kl = s->kv_k + (size_t)l * s->ctx * m->kv_dim;
    uint16_t *vl = s->kv_v + (size_t)l * s->ctx * m->kv_dim;
    for (uint32_t j = 0; j < m->kv_dim; ++j) {
      kl[(size_t)pos * m->kv_dim + j] = vgo_float_to_half(s->k[j]);
      vl[(size_t)pos * m->kv_dim + j] = vgo_float_to_half(s->v[j]);
    }
    (x ? vgo_attention_xtx : vgo_attention)(s->q, kl, vl, m->heads, m->kv_heads, m->head_dim, s->ctx, pos,
                                            s->scores, s->attention);
    (x ? vgo_matvec_xtx : vgo_matvec)((int)m->wo[l]->type, tdata(m, m->wo[l]), m->H, m->H, s->attention,
                                      s->branch, 1.0f);
    (x ? vgo_residual_rmsnorm_xtx : vgo_residual_rmsnorm)(s->hidden, s->branch, tf32(m, m->ffn_norm[l]), m->H,
                                                          m->eps, rs, s->norm);
    (x ? vgo_swiglu_xtx : vgo_swiglu)((int)m->wg[l]->type, tdata(m, m->wg[l]), tdata(m, m->wu[l]), m->F, m->H,
                                      s->norm, s->gate);
    (x ? vgo_matvec_xtx : vgo_matvec)((int)m->wd[l]->type, tdata(m, m->wd[l]), m->H, m->F, s->gate,
                                      s->branch, 1.0f);
    const float *next = l + 1 < m->L ? tf32(m, m->attn_norm[l + 1]) : tf32(m, m->out_norm);
    (x ? vgo_residual_rmsnorm_xtx : vgo_residual_rmsnorm)(s->hidden, s->branch, next, m->H, m->eps, rs, s->norm);
  }
  if (compute_logits)
    (x ? vgo_matvec_xtx : vgo_matvec)((int)m->out->type, tdata(m, m->out), m->vocab, m->H, s->norm,
                                      s->logits, eff(m->logit_scale));
  return 0;
}

/* decode_token, src/baselm.rs:622-655 (and decode_token_gpu_only :689-721). */
int vgo_decode_token(vgo_state *s, uint32_t token, int want_logits) {
  const vgo_model *m = s->m;
  if (token >= m->vocab) {
    snprintf(s->err, sizeof s->err, "token id %u is outside vocabulary 0..%u", token, m->vocab);
    return -5;
  }
  if (s->position >= s->ctx) {
    snprintf(s->err, sizeof s->err, "BaseLM KV cache is full at %u tokens", s->ctx);
    return -6;
  }
  vgo_embedding((int)m->tok->type, tdata(m, m->tok), m->H, token, eff(m->emb_scale), s->hidden);
  int rc = record_transformer(s, want_logits);
  if (rc) return rc;
  s->position += 1;
  return 0;
}

/* decode_embedding, src/baselm.rs:657-681. */
int vgo_decode_embedding(vgo_state *s, const float *h, int want_logits) {
  const vgo_model *m = s->m;
  if (s->position >= s->ctx) {
    snprintf(s->err, sizeof s->err, "BaseLM KV cache is full at %u tokens", s->ctx);
    return -6;
  }
  memcpy(s->hidden, h, sizeof(float) * m->H);
  int rc = record_transformer(s, want_logits);
  if (rc) return rc;
  s->position += 1;
  return 0;
}

const float *vgo_output(const vgo_state *s) { return s->norm; }
const float *vgo_logits(const vgo_state *s) { return s->logits; }
const char *vgo_last_error(const vgo_state *s) { return s->err; }

const float *vgo_buffer(const vgo_state *s, const char *name) {
  if (!strcmp(name, "hidden")) return s->hidden;
  if (!strcmp(name, "norm")) return s->norm;
  if (!strcmp(name, "q")) return s->q;
  if (!strcmp(name, "k")) return s->k;
  if (!strcmp(name, "v")) return s->v;
  if (!strcmp(name, "attention")) return s->attention;
  if (!strcmp(name, "gate")) return s->gate;
  if (!strcmp(name, "branch")) return s->branch;
  if (!strcmp(name, "scores")) return s->scores;
  if (!strcmp(name, "logits")) return s->logits;
  return NULL;
}
