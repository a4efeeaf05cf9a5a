/*
 * voxgen_oracle.h — CPU oracle for the BaseLM per-token decode step.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * GLSL shaders on the hot path (normal variants) and of the Rust sequencing
 * that records them, used as the checker for the CUDA path and as the timed
 * CPU baseline. Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
 * may load it; the product library never links or calls it.
 *
 * Parity pinning: the reference's Rust host cannot be built here (no cargo)
 * and its shaders cannot run on Vulkan (no glslc, no Vulkan stack). Its GLSL
 * compute shaders are instead compiled as C++ and run on the CPU by
 * oracle/ref_shim (workgroups emulated with fibers); this restatement matches
 * that build bit for bit, shader by shader and over whole decode steps, on
 * head_dim 128 models (tests/test_cpu_ref_pin.py, with committed golden
 * vectors in tests/golden/). It also matches the reference's known-answer
 * tests (src/baselm.rs:1315-1358, src/gguf.rs:41-45).
 */
#ifndef VOXGEN_ORACLE_H
#define VOXGEN_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct vgo_model vgo_model;
typedef struct vgo_state vgo_state;

/* geometry indices for vgo_model_geometry */
enum {
  VGO_CTX_LEN = 0, VGO_H, VGO_LAYERS, VGO_FFN, VGO_VOCAB, VGO_HEADS, VGO_KV_HEADS,
  VGO_HEAD_DIM, VGO_KV_DIM, VGO_FORMAT, VGO_TIED, VGO_ORIG_CTX, VGO_NGEOM
};

int vgo_model_load(const char *path, vgo_model **out, char *err, size_t err_len);
void vgo_model_free(vgo_model *m);
void vgo_model_geometry(const vgo_model *m, uint32_t *out /* VGO_NGEOM */);
void vgo_model_scalars(const vgo_model *m, float *out /* eps, theta, scaling, emb, res, logit */);

int vgo_state_create(const vgo_model *m, uint32_t max_context, vgo_state **out);
void vgo_state_free(vgo_state *s);
void vgo_reset(vgo_state *s);
uint32_t vgo_position(const vgo_state *s);
int vgo_set_position(vgo_state *s, uint32_t pos);
/* k, v: [layer][n][kv_dim] fp16 bits */
int vgo_write_kv(vgo_state *s, const uint16_t *k, const uint16_t *v, uint32_t n);
int vgo_read_kv(const vgo_state *s, uint16_t *k, uint16_t *v, uint32_t n);

int vgo_decode_token(vgo_state *s, uint32_t token, int want_logits);
int vgo_decode_embedding(vgo_state *s, const float *h, int want_logits);
const float *vgo_output(const vgo_state *s);
const float *vgo_logits(const vgo_state *s);
/* intermediate buffers of the last step: "hidden", "q", "k", "v", "attention",
 * "gate", "branch", "norm", "scores" */
const float *vgo_buffer(const vgo_state *s, const char *name);
const char *vgo_last_error(const vgo_state *s);

void vgo_set_threads(int n);
/* The RX 7900 XTX mode (the _xtx7900 shader variants' summation order) for
 * every later step of this state. */
void vgo_set_xtx(vgo_state *s, int on);
void vgo_matvec_xtx(int dtype, const uint8_t *w, uint32_t rows, uint32_t cols, const float *x,
                    float *y, float alpha);
void vgo_swiglu_xtx(int dtype, const uint8_t *wg, const uint8_t *wu, uint32_t rows, uint32_t cols,
                    const float *x, float *y);
void vgo_rmsnorm_xtx(const float *x, const float *w, uint32_t n, float eps, float *y);
void vgo_residual_rmsnorm_xtx(float *hidden, const float *branch, const float *w, uint32_t n,
                              float eps, float scale, float *y);
void vgo_attention_xtx(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                       uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t ctx,
                       uint32_t position, float *scores, float *out);
int vgo_get_threads(void);

/* ---- shader-level restatements (raw GGUF tensor bytes) ---- */
float vgo_half_to_float(uint16_t h);
uint16_t vgo_float_to_half(float f);
void vgo_matvec(int dtype, const uint8_t *w, uint32_t rows, uint32_t cols,
                const float *x, float *y, float alpha);
void vgo_embedding(int dtype, const uint8_t *w, uint32_t cols, uint32_t token,
                   float alpha, float *hidden);
void vgo_rmsnorm(const float *x, const float *w, uint32_t n, float eps, float *y);
void vgo_residual_rmsnorm(float *hidden, const float *branch, const float *w,
                          uint32_t n, float eps, float scale, float *y);
void vgo_swiglu(int dtype, const uint8_t *wg, const uint8_t *wu, uint32_t rows,
                uint32_t cols, const float *x, float *y);
void vgo_rope(float *q, float *k, const float *ext, uint32_t position,
              uint32_t q_heads, uint32_t kv_heads, uint32_t head_dim,
              float theta, float scaling);
/* attention over one layer of a reference-layout cache [ctx][kv_dim] */
void vgo_attention(const float *q, const uint16_t *k_cache, const uint16_t *v_cache,
                   uint32_t heads, uint32_t kv_heads, uint32_t head_dim,
                   uint32_t ctx, uint32_t position, float *scores, float *out);

#ifdef __cplusplus
}
#endif
#endif
