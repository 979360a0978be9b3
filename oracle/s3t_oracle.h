/* CPU restatement of the SAM 3 ViT vision trunk (test infrastructure only).
 *
 * This is the checker that the CUDA path is compared against; it is never the
 * thing measured or shipped.  It restates, in plain C, the arithmetic of the
 * reference's ggml CPU path for src/vision_trunk.cpp, including the activation
 * rounding ggml's mul_mat applies per weight type.  Parity of this file with
 * the reference itself is pinned by tests/test_oracle_pins.py (ggml op-level
 * checks through oracle/_ref) and by the full-trunk golden fixtures under
 * tests/golden/ (made by running the reference's VisionTrunk::run).
 */
#ifndef S3T_ORACLE_H
#define S3T_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 8 };

uint16_t or_fp32_to_fp16(float f);
float    or_fp16_to_fp32(uint16_t h);
void     or_fp32_to_fp16_row(const float *x, uint16_t *y, int64_t n);
void     or_dequantize(int type, const void *src, int64_t n, float *y);
void     or_quantize_q8_0_act(const float *x, int64_t n, uint8_t *blocks);
void     or_round_activations(int wtype, const float *x, int64_t n, float *y);

void or_set_sum_variant(int variant);
void or_linear(int wtype, const void *w, int64_t N, int64_t K, const float *x, int64_t M,
               const float *bias, float *y);
void or_layer_norm(const float *x, int64_t rows, int64_t cols, const float *gamma,
                   const float *beta, float eps, float *y);
void or_rope_table(float freq_scale, int npos, float *cos_out, float *sin_out);
void or_rope_axial(float *x, int64_t tokens, int64_t heads, const int32_t *pos_x,
                   const int32_t *pos_y, float freq_scale);
void or_attention(const float *q, const float *k, const float *v, int64_t nq, int64_t nk,
                  int64_t heads, int64_t d, float scale, float *out);
void or_attention_masked(const float *q, const float *k, const float *v, int64_t nq, int64_t nk,
                         int64_t heads, int64_t d, float scale, const float *key_mask, float *out);
void or_attention_softmax(const float *q, const float *k, const float *v, int64_t nq, int64_t nk,
                          int64_t heads, int64_t d, float scale, const float *bias, const float *key_mask,
                          float *out);
void or_gelu_erf(const float *x, int64_t n, float *y);
void or_patch_embed(int wtype, const void *w, const float *image, float *out);
/* uint8 RGB (h x w x 3) -> normalized [3][1008][1008] fp32, the reference's
 * bilinear_resize_rgb (tools/sam3_vision_trunk.cpp:33-66). */
void or_bilinear_resize_rgb(const uint8_t *src, int w, int h, float *out);

typedef struct {
    int qkv_t, proj_t, fc1_t, fc2_t;
    const void *qkv_w, *proj_w, *fc1_w, *fc2_w;
    const float *n1w, *n1b, *qkv_b, *proj_b, *n2w, *n2b, *fc1_b, *fc2_b;
} or_layer;

typedef struct {
    int patch_t;
    const void *patch_w;      /* GGUF [O=1024, KH=14, KW=14, I=3] of type patch_t */
    const float *pos_embed;   /* [577][1024] */
    const float *ln_pre_w, *ln_pre_b;
    int n_layers;
    or_layer layer[32];
} or_trunk;

/* Runs the stem and layers [0, n_run) on one [3,1008,1008] image.
 * out_tokens (may be NULL): the residual stream [5184][1024] token-major.
 * out_nchw (may be NULL): the same as [1024][72][72]. */
int or_trunk_run(const or_trunk *t, const float *image, int n_run, float *out_tokens,
                 float *out_nchw);

#ifdef __cplusplus
}
#endif
#endif
