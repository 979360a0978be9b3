/* CPU restatement of the SAM 3 ViT vision trunk — TEST INFRASTRUCTURE ONLY.
 *
 * The checker the CUDA path is compared against (tests/, smoke(), and the
 * bench's cpu_baseline leg).  It is never linked into the product.  Each
 * function states the reference code whose arithmetic it restates; paths are
 * relative to the reference project (ggml/ = third_party/ggml/).
 *
 * Pinning: tests/test_oracle_pins.py compares every op here with the same ggml
 * op run through oracle/_ref (the reference compiled from its own sources),
 * and tests/golden/ holds full-trunk outputs of the reference's
 * VisionTrunk::run on the seeded F32/F16/Q8_0 files, which or_trunk_run is
 * checked against.
 */
#include "s3t_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- fp16 --- */

/* IEEE binary32 -> binary16, round to nearest even (the rounding F16C's
 * vcvtps2ph uses for GGML_CPU_FP32_TO_FP16, ggml/src/ggml-cpu/simd-mappings.h,
 * and ggml_compute_fp32_to_fp16, ggml/src/ggml-impl.h:400-431). */
uint16_t or_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t) (sign | 0x7c00u);          /* >= 65520 rounds to inf */
    if (ax < 0x38800000u) {                                             /* below 2^-14: subnormal */
        float af;
        memcpy(&af, &ax, 4);
        const uint32_t m = (uint32_t) nearbyintf(af * 16777216.0f);     /* units of 2^-24, RNE */
        return (uint16_t) (sign | m);
    }
    const uint32_t mant = ax & 0x7fffffu;
    const uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t h = (e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t) (sign | h);
}

/* binary16 -> binary32, exact (ggml_compute_fp16_to_fp32, ggml-impl.h:378-399). */
float or_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        float v = (float) m * (1.0f / 16777216.0f);
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e - 15 + 127) << 23) | (m << 13);
    }
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

void or_fp32_to_fp16_row(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = or_fp32_to_fp16(x[i]);
}

/* --------------------------------------------------------------- Q8_0 --- */

/* File-format dequantization: F16 -> fp32 (exact), Q8_0 -> qs[j] * fp32(d)
 * (dequantize_row_q8_0, ggml/src/ggml-quants.c:436-450; block_q8_0 is
 * {fp16 d; int8 qs[32]}, ggml/src/ggml-common.h:230-234). */
void or_dequantize(int type, const void *src, int64_t n, float *y) {
    if (type == OR_F32) {
        memcpy(y, src, (size_t) n * 4);
    } else if (type == OR_F16) {
        const uint16_t *h = (const uint16_t *) src;
        for (int64_t i = 0; i < n; i++) y[i] = or_fp16_to_fp32(h[i]);
    } else {
        const uint8_t *b = (const uint8_t *) src;
        for (int64_t i = 0; i < n / 32; i++, b += 34) {
            uint16_t dh;
            memcpy(&dh, b, 2);
            const float d = or_fp16_to_fp32(dh);
            const int8_t *qs = (const int8_t *) (b + 2);
            for (int j = 0; j < 32; j++) y[i * 32 + j] = qs[j] * d;
        }
    }
}

/* The activation quantizer ggml's CPU mul_mat applies to src1 before a Q8_0
 * dot (vec_dot_type of Q8_0 is Q8_0, ggml-cpu.c:252-256): the x86 variant
 * quantize_row_q8_0 (ggml/src/ggml-cpu/arch/x86/quants.c:290-340):
 * d = amax/127 stored as fp16, id = 127/amax, q = round-to-nearest-even(x*id). */
void or_quantize_q8_0_act(const float *x, int64_t n, uint8_t *blocks) {
    for (int64_t i = 0; i < n / 32; i++) {
        const float *xb = x + i * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            const float a = fabsf(xb[j]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / 127.f;
        const uint16_t dh = or_fp32_to_fp16(d);
        const float id = (amax != 0.0f) ? 127.f / amax : 0.0f;
        uint8_t *b = blocks + i * 34;
        memcpy(b, &dh, 2);
        for (int j = 0; j < 32; j++) b[2 + j] = (uint8_t) (int8_t) (int) nearbyintf(xb[j] * id);
    }
}

/* What ggml's mul_mat does to the f32 activations for a given weight type
 * (ggml-cpu.c:1297-1332 with the traits at :208-260): F32 unchanged; F16
 * rounded to fp16; Q8_0 quantized per 32-block (returned dequantized). */
void or_round_activations(int wtype, const float *x, int64_t n, float *y) {
    if (wtype == OR_F32) {
        if (y != x) memcpy(y, x, (size_t) n * 4);
    } else if (wtype == OR_F16) {
        for (int64_t i = 0; i < n; i++) y[i] = or_fp16_to_fp32(or_fp32_to_fp16(x[i]));
    } else {
        uint8_t blk[34];
        for (int64_t i = 0; i < n / 32; i++) {
            or_quantize_q8_0_act(x + i * 32, 32, blk);
            or_dequantize(OR_Q8_0, blk, 32, y + i * 32);
        }
    }
}

/* ------------------------------------------------------------- linear --- */

/* Summation-order variant of the dot products (0: ascending K, 1: descending
 * K).  Both are equally faithful to ggml; comparing them measures how much a
 * trunk result moves under a pure change of floating-point summation order. */
static int g_sum_variant = 0;
void or_set_sum_variant(int v) { g_sum_variant = v; }

static void gemm_nt_rev(const float *x, const float *w, int64_t M, int64_t N, int64_t K,
                        const float *bias, float *y) {
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t m = 0; m < M; m++) {
        const float *x0 = x + m * K;
        for (int64_t n = 0; n < N; n++) {
            const float *wr = w + n * K;
            float a0 = 0;
#pragma omp simd reduction(+ : a0)
            for (int64_t k = K - 1; k >= 0; k--) a0 += x0[k] * wr[k];
            y[m * N + n] = a0 + (bias ? bias[n] : 0.0f);
        }
    }
}

static void gemm_nt(const float *x, const float *w, int64_t M, int64_t N, int64_t K,
                    const float *bias, float *y) {
    if (g_sum_variant) {
        gemm_nt_rev(x, w, M, N, K, bias, y);
        return;
    }
    const int64_t MB = 16, NB = 64;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t m0 = 0; m0 < M; m0 += MB) {
        for (int64_t n0 = 0; n0 < N; n0 += NB) {
            const int64_t m1 = m0 + MB < M ? m0 + MB : M;
            const int64_t n1 = n0 + NB < N ? n0 + NB : N;
            int64_t m = m0;
            for (; m + 4 <= m1; m += 4) {
                const float *x0 = x + m * K, *x1 = x0 + K, *x2 = x1 + K, *x3 = x2 + K;
                for (int64_t n = n0; n < n1; n++) {
                    const float *wr = w + n * K;
                    float a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma omp simd reduction(+ : a0, a1, a2, a3)
                    for (int64_t k = 0; k < K; k++) {
                        a0 += x0[k] * wr[k];
                        a1 += x1[k] * wr[k];
                        a2 += x2[k] * wr[k];
                        a3 += x3[k] * wr[k];
                    }
                    const float b = bias ? bias[n] : 0.0f;
                    y[(m + 0) * N + n] = a0 + b;
                    y[(m + 1) * N + n] = a1 + b;
                    y[(m + 2) * N + n] = a2 + b;
                    y[(m + 3) * N + n] = a3 + b;
                }
            }
            for (; m < m1; m++) {
                const float *x0 = x + m * K;
                for (int64_t n = n0; n < n1; n++) {
                    const float *wr = w + n * K;
                    float a0 = 0;
#pragma omp simd reduction(+ : a0)
                    for (int64_t k = 0; k < K; k++) a0 += x0[k] * wr[k];
                    y[m * N + n] = a0 + (bias ? bias[n] : 0.0f);
                }
            }
        }
    }
}

/* linear() of src/vision_trunk.cpp:50-62: y = mul_mat(W, x) + b, with W of
 * ggml type wtype, ne = [K, N] (row n = output channel, K contiguous), and the
 * activations rounded the way ggml's CPU mul_mat rounds them for that type. */
void or_linear(int wtype, const void *w, int64_t N, int64_t K, const float *x, int64_t M,
               const float *bias, float *y) {
    float *wf = (float *) malloc((size_t) N * K * 4);
    float *xr = (float *) malloc((size_t) M * K * 4);
    or_dequantize(wtype, w, N * K, wf);
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) or_round_activations(wtype, x + m * K, K, xr + m * K);
    gemm_nt(xr, wf, M, N, K, bias, y);
    free(wf);
    free(xr);
}

/* ---------------------------------------------------------- layernorm --- */

/* layer_norm() of src/vision_trunk.cpp:64-74: ggml_norm (ggml-cpu/ops.cpp:
 * 3646-3690: mean and centred variance summed in double, y=(x-mean)/sqrt(var+eps))
 * then * gamma + beta as two separate f32 ops. */
void or_layer_norm(const float *x, int64_t rows, int64_t cols, const float *gamma,
                   const float *beta, float eps, float *y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * cols;
        float *yr = y + r * cols;
        double sum = 0.0;
        for (int64_t c = 0; c < cols; c++) sum += (double) xr[c];
        const float mean = (float) sum / (float) cols;
        double sq = 0.0;
        for (int64_t c = 0; c < cols; c++) {
            const float v = xr[c] - mean;
            yr[c] = v;
            sq += (double) (v * v);
        }
        const float var = (float) (sq / (double) cols);
        const float scale = 1.0f / sqrtf(var + eps);
        for (int64_t c = 0; c < cols; c++) {
            float v = yr[c] * scale;
            if (gamma) v = v * gamma[c];
            if (beta) v = v + beta[c];
            yr[c] = v;
        }
    }
}

/* --------------------------------------------------------------- rope --- */

/* cos/sin of ggml's NORMAL-mode rope for n_dims = 32 (ggml-cpu/ops.cpp:
 * 5603-5640 rope_yarn + ggml_rope_cache_init, ext_factor 0, attn_factor 1):
 * theta starts at the position, is multiplied by 10000^(-2/32) per pair in
 * f32, and cos/sin are taken of freq_scale * theta.  Tables are [npos][16]. */
void or_rope_table(float freq_scale, int npos, float *cos_out, float *sin_out) {
    const float theta_scale = powf(10000.0f, -2.0f / 32.0f);
    for (int p = 0; p < npos; p++) {
        float theta = (float) p;
        for (int j = 0; j < 16; j++) {
            const float t = freq_scale * theta;
            cos_out[p * 16 + j] = cosf(t);
            sin_out[p * 16 + j] = sinf(t);
            theta *= theta_scale;
        }
    }
}

/* apply_axial_rope (src/vision_trunk.cpp:145-205): per head of 64, dims 0..31
 * are rotated in adjacent pairs (2j, 2j+1) by pos_x, dims 32..63 by pos_y
 * (ggml-cpu/ops.cpp:5708-5722 rotate_pairs).  x is [tokens][heads][64], in place. */
void or_rope_axial(float *x, int64_t tokens, int64_t heads, const int32_t *pos_x,
                   const int32_t *pos_y, float freq_scale) {
    int maxp = 0;
    for (int64_t t = 0; t < tokens; t++) {
        if (pos_x[t] > maxp) maxp = pos_x[t];
        if (pos_y[t] > maxp) maxp = pos_y[t];
    }
    float *c = (float *) malloc((size_t) (maxp + 1) * 16 * 4);
    float *s = (float *) malloc((size_t) (maxp + 1) * 16 * 4);
    or_rope_table(freq_scale, maxp + 1, c, s);
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < tokens; t++) {
        for (int64_t h = 0; h < heads; h++) {
            float *v = x + (t * heads + h) * 64;
            for (int half = 0; half < 2; half++) {
                const int p = half ? pos_y[t] : pos_x[t];
                for (int j = 0; j < 16; j++) {
                    const float ct = c[p * 16 + j], st = s[p * 16 + j];
                    const float x0 = v[half * 32 + 2 * j], x1 = v[half * 32 + 2 * j + 1];
                    v[half * 32 + 2 * j] = x0 * ct - x1 * st;
                    v[half * 32 + 2 * j + 1] = x0 * st + x1 * ct;
                }
            }
        }
    }
    free(c);
    free(s);
}

/* ---------------------------------------------------------- attention --- */

/* ggml_flash_attn_ext, no mask, prec F32 (apply_attention, src/vision_trunk.cpp:
 * 207-228; ggml-cpu/ops.cpp:8130-8860): out = softmax(q k^T * scale) v per head,
 * f32 throughout.  q: [nq][heads][d], k/v: [nk][heads][d], out: [nq][heads][d]. */
void or_attention(const float *q, const float *k, const float *v, int64_t nq, int64_t nk,
                  int64_t heads, int64_t d, float scale, float *out) {
#pragma omp parallel
    {
        float *sc = (float *) malloc((size_t) nk * 4);
        float *acc = (float *) malloc((size_t) d * 4);
#pragma omp for collapse(2) schedule(static)
        for (int64_t h = 0; h < heads; h++) {
            for (int64_t i = 0; i < nq; i++) {
                const float *qi = q + (i * heads + h) * d;
                float mx = -INFINITY;
                for (int64_t j = 0; j < nk; j++) {
                    const float *kj = k + (j * heads + h) * d;
                    float s = 0.0f;
#pragma omp simd reduction(+ : s)
                    for (int64_t e = 0; e < d; e++) s += qi[e] * kj[e];
                    s *= scale;
                    sc[j] = s;
                    mx = s > mx ? s : mx;
                }
                for (int64_t e = 0; e < d; e++) acc[e] = 0.0f;
                float sum = 0.0f;
                for (int64_t j = 0; j < nk; j++) {
                    const float p = expf(sc[j] - mx);
                    sum += p;
                    const float *vj = v + (j * heads + h) * d;
#pragma omp simd
                    for (int64_t e = 0; e < d; e++) acc[e] += p * vj[e];
                }
                float *o = out + (i * heads + h) * d;
                const float inv = 1.0f / sum;
                for (int64_t e = 0; e < d; e++) o[e] = acc[e] * inv;
            }
        }
        free(sc);
        free(acc);
    }
}

/* ggml_flash_attn_ext, prec F32, with an additive mask that is the same for
 * every query row: mha() of src/encoder_fusion.cpp:63-88 (head dim 32, scale
 * 1/sqrt(32)), whose prompt mask (:120-133) repeats one 0 / -inf row.  As in
 * ggml-cpu/ops.cpp:8254-8271 a key whose mask is -inf is skipped and any other
 * mask value is added to the scaled score; as in :8353-8354 a row with no
 * unskipped key (sum 0) comes out as 0.  f32 throughout.  key_mask: [nk] or
 * NULL.  q: [nq][heads][d], k/v: [nk][heads][d], out: [nq][heads][d]. */
void or_attention_masked(const float *q, const float *k, const float *v, int64_t nq, int64_t nk,
                         int64_t heads, int64_t d, float scale, const float *key_mask, float *out) {
#pragma omp parallel
    {
        float *sc = (float *) malloc((size_t) nk * 4);
        float *acc = (float *) malloc((size_t) d * 4);
#pragma omp for collapse(2) schedule(static)
        for (int64_t h = 0; h < heads; h++) {
            for (int64_t i = 0; i < nq; i++) {
                const float *qi = q + (i * heads + h) * d;
                float mx = -INFINITY;
                for (int64_t j = 0; j < nk; j++) {
                    const float mv = key_mask ? key_mask[j] : 0.0f;
                    if (mv == -INFINITY) {
                        sc[j] = -INFINITY;
                        continue;
                    }
                    const float *kj = k + (j * heads + h) * d;
                    float s = 0.0f;
#pragma omp simd reduction(+ : s)
                    for (int64_t e = 0; e < d; e++) s += qi[e] * kj[e];
                    s = s * scale + mv;
                    sc[j] = s;
                    mx = s > mx ? s : mx;
                }
                for (int64_t e = 0; e < d; e++) acc[e] = 0.0f;
                float sum = 0.0f;
                for (int64_t j = 0; j < nk; j++) {
                    if (sc[j] == -INFINITY) continue;
                    const float p = expf(sc[j] - mx);
                    sum += p;
                    const float *vj = v + (j * heads + h) * d;
#pragma omp simd
                    for (int64_t e = 0; e < d; e++) acc[e] += p * vj[e];
                }
                float *o = out + (i * heads + h) * d;
                const float inv = sum == 0.0f ? 0.0f : 1.0f / sum;
                for (int64_t e = 0; e < d; e++) o[e] = acc[e] * inv;
            }
        }
        free(sc);
        free(acc);
    }
}

/* The decoder's attention, mha() of src/decoder.cpp:95-127: scores = k.q per
 * head (ggml_mul_mat, f32 dots), ggml_soft_max_ext(scores, mask, scale) and
 * probs.v (ggml_mul_mat).  The softmax follows ggml-cpu/ops.cpp:5284-5330:
 * w = s*scale + mask, m = max w, p = expf(w - m) summed in double, p *= 1/sum
 * (so a row with every entry -inf is NaN, as there).  The mask is either a full
 * bias [heads][nq][nk] (the image cross attention's box relative-position
 * bias, :401-418, :457-465) or one row [nk] repeated for every query (the text
 * cross attention's prompt mask, :131-143, :443-451); either may be NULL.
 * q: [nq][heads][d], k/v: [nk][heads][d], out: [nq][heads][d]. */
void or_attention_softmax(const float *q, const float *k, const float *v, int64_t nq, int64_t nk,
                          int64_t heads, int64_t d, float scale, const float *bias, const float *key_mask,
                          float *out) {
#pragma omp parallel
    {
        float *w = (float *) malloc((size_t) nk * 4);
#pragma omp for collapse(2) schedule(static)
        for (int64_t h = 0; h < heads; h++) {
            for (int64_t i = 0; i < nq; i++) {
                const float *qi = q + (i * heads + h) * d;
                const float *brow = bias ? bias + (h * nq + i) * nk : NULL;
                float mx = -INFINITY;
                for (int64_t j = 0; j < nk; j++) {
                    const float *kj = k + (j * heads + h) * d;
                    float s = 0.0f;
                    for (int64_t e = 0; e < d; e++) s += qi[e] * kj[e];
                    s *= scale;
                    if (brow) s += brow[j];
                    if (key_mask) s += key_mask[j];
                    w[j] = s;
                    mx = s > mx ? s : mx;
                }
                double sum = 0.0;
                for (int64_t j = 0; j < nk; j++) {
                    w[j] = expf(w[j] - mx);
                    sum += (double) w[j];
                }
                const float inv = (float) (1.0 / sum);
                float *o = out + (i * heads + h) * d;
                for (int64_t e = 0; e < d; e++) o[e] = 0.0f;
                for (int64_t j = 0; j < nk; j++) {
                    const float p = w[j] * inv;
                    const float *vj = v + (j * heads + h) * d;
                    for (int64_t e = 0; e < d; e++) o[e] += p * vj[e];
                }
            }
        }
        free(w);
    }
}

/* ggml_vec_gelu_erf_f32 (ggml-cpu/vec.h:1018-1023). */
void or_gelu_erf(const float *x, int64_t n, float *y) {
    const float sqrt_2_inv = 0.70710678118654752440f;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = 0.5f * x[i] * (1.0f + erff(x[i] * sqrt_2_inv));
}

/* ------------------------------------------------------------ patches --- */

/* conv2d_patch_embed + the token-major permute (src/vision_trunk.cpp:284-291,
 * 364-368; ggml_conv_2d = im2col typed like the kernel, then mul_mat,
 * ggml/src/ggml.c:4551-4573).  w is the GGUF tensor [O][KH][KW][I] of type
 * wtype; the image is rounded to that type as im2col does (F16 -> fp16).
 * out: [5184][1024], token t = y*72 + x. */
void or_patch_embed(int wtype, const void *w, const float *image, float *out) {
    const int64_t KK = 3 * 14 * 14;
    float *wf = (float *) malloc((size_t) 1024 * KK * 4);
    float *wr = (float *) malloc((size_t) 1024 * KK * 4);
    float *cols = (float *) malloc((size_t) 5184 * KK * 4);
    or_dequantize(wtype, w, 1024 * KK, wf);
    /* reorder the weight to (ic, kh, kw), the im2col column order */
    for (int o = 0; o < 1024; o++)
        for (int kh = 0; kh < 14; kh++)
            for (int kw = 0; kw < 14; kw++)
                for (int ic = 0; ic < 3; ic++)
                    wr[o * KK + ic * 196 + kh * 14 + kw] = wf[((o * 14 + kh) * 14 + kw) * 3 + ic];
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < 5184; t++) {
        const int64_t ty = t / 72, tx = t % 72;
        for (int ic = 0; ic < 3; ic++)
            for (int kh = 0; kh < 14; kh++)
                for (int kw = 0; kw < 14; kw++) {
                    const float v = image[((int64_t) ic * 1008 + ty * 14 + kh) * 1008 + tx * 14 + kw];
                    cols[t * KK + ic * 196 + kh * 14 + kw] =
                        wtype == OR_F32 ? v : or_fp16_to_fp32(or_fp32_to_fp16(v));
                }
    }
    gemm_nt(cols, wr, 5184, 1024, KK, NULL, out);
    free(wf);
    free(wr);
    free(cols);
}

/* -------------------------------------------------------------- trunk --- */

static int is_global(int layer) { return layer == 7 || layer == 15 || layer == 23 || layer == 31; }

/* VisionTrunk::run (src/vision_trunk.cpp:297-488) for one image, stopping
 * after n_run layers.  Windowed layers attend inside each 24x24 window with
 * window-local RoPE positions (make_axis_positions(24), scale 1); global
 * layers 7/15/23/31 attend over all 5184 tokens with positions on the 72x72
 * grid and RoPE scale 24/72 (:14-25, :388-427). */
int or_trunk_run(const or_trunk *t, const float *image, int n_run, float *out_tokens,
                 float *out_nchw) {
    const int64_t T = 5184, C = 1024, F = 4736;
    float *x = (float *) malloc((size_t) T * C * 4);
    float *a = (float *) malloc((size_t) T * C * 4);
    float *qkv = (float *) malloc((size_t) T * 3 * C * 4);
    float *attn = (float *) malloc((size_t) T * C * 4);
    float *h = (float *) malloc((size_t) T * F * 4);
    float *gq = (float *) malloc((size_t) T * C * 4);
    float *gk = (float *) malloc((size_t) T * C * 4);
    float *gv = (float *) malloc((size_t) T * C * 4);
    float *go = (float *) malloc((size_t) T * C * 4);
    int32_t *px = (int32_t *) malloc(T * 4), *py = (int32_t *) malloc(T * 4);
    int64_t *idx = (int64_t *) malloc(T * 8);
    if (!x || !a || !qkv || !attn || !h || !gq || !gk || !gv || !go || !px || !py || !idx) return -1;

    or_patch_embed(t->patch_t, t->patch_w, image, x);
    /* make_tiled_abs_pos (:111-132): pos token 1 + (y%24)*24 + (x%24) */
    for (int64_t tok = 0; tok < T; tok++) {
        const int64_t ty = tok / 72, tx = tok % 72;
        const float *p = t->pos_embed + (1 + (ty % 24) * 24 + (tx % 24)) * C;
        for (int64_t c = 0; c < C; c++) x[tok * C + c] += p[c];
    }
    or_layer_norm(x, T, C, t->ln_pre_w, t->ln_pre_b, 1e-5f, x);

    for (int l = 0; l < n_run; l++) {
        const or_layer *L = &t->layer[l];
        or_layer_norm(x, T, C, L->n1w, L->n1b, 1e-5f, a);
        or_linear(L->qkv_t, L->qkv_w, 3 * C, C, a, T, L->qkv_b, qkv);
        const int glob = is_global(l);
        const int ngroups = glob ? 1 : 9;
        const int64_t len = glob ? T : 576;
        const float scale = glob ? (float) 24 / (float) 72 : 1.0f;
        for (int g = 0; g < ngroups; g++) {
            for (int64_t i = 0; i < len; i++) {
                int64_t tok;
                if (glob) {
                    tok = i;
                    px[i] = (int32_t) (i % 72);
                    py[i] = (int32_t) (i / 72);
                } else {
                    const int64_t wy = g / 3, wx = g % 3, ly = i / 24, lx = i % 24;
                    tok = (wy * 24 + ly) * 72 + wx * 24 + lx;
                    px[i] = (int32_t) lx;
                    py[i] = (int32_t) ly;
                }
                idx[i] = tok;
                memcpy(gq + i * C, qkv + tok * 3 * C, C * 4);
                memcpy(gk + i * C, qkv + tok * 3 * C + C, C * 4);
                memcpy(gv + i * C, qkv + tok * 3 * C + 2 * C, C * 4);
            }
            or_rope_axial(gq, len, 16, px, py, scale);
            or_rope_axial(gk, len, 16, px, py, scale);
            or_attention(gq, gk, gv, len, len, 16, 64, 0.125f, go);
            for (int64_t i = 0; i < len; i++) memcpy(attn + idx[i] * C, go + i * C, C * 4);
        }
        or_linear(L->proj_t, L->proj_w, C, C, attn, T, L->proj_b, a);
        for (int64_t i = 0; i < T * C; i++) x[i] = x[i] + a[i];
        or_layer_norm(x, T, C, L->n2w, L->n2b, 1e-5f, a);
        or_linear(L->fc1_t, L->fc1_w, F, C, a, T, L->fc1_b, h);
        or_gelu_erf(h, T * F, h);
        or_linear(L->fc2_t, L->fc2_w, C, F, h, T, L->fc2_b, a);
        for (int64_t i = 0; i < T * C; i++) x[i] = x[i] + a[i];
    }
    if (out_tokens) memcpy(out_tokens, x, (size_t) T * C * 4);
    if (out_nchw) {
        for (int64_t c = 0; c < C; c++)
            for (int64_t tok = 0; tok < T; tok++) out_nchw[c * T + tok] = x[tok * C + c];
    }
    free(x); free(a); free(qkv); free(attn); free(h);
    free(gq); free(gk); free(gv); free(go); free(px); free(py); free(idx);
    return 0;
}

/* Image preprocessing of tools/sam3_vision_trunk.cpp:33-66 (bilinear_resize_rgb;
 * the same arithmetic as src/pipeline.cpp:45-83 load_image_rgb after stbi_load):
 * uint8 RGB, row-major HWC -> [3][1008][1008] fp32, half-pixel-centre bilinear
 * sampling with the source index clamped (the weight is taken from the clamped
 * index, so it extrapolates at the top/left edge), p/255, then (v - 0.5)/0.5.
 * Every product and sum is rounded on its own, as in the reference's scalar
 * x86-64 build (no fused multiply-add). */
__attribute__((optimize("fp-contract=off")))
void or_bilinear_resize_rgb(const uint8_t *src, int w, int h, float *out) {
    const int S = 1008;
    const float xs = (float) w / (float) S, ys = (float) h / (float) S;
    for (int dy = 0; dy < S; dy++) {
        const float sy = ((float) dy + 0.5f) * ys - 0.5f;
        int y0 = (int) floorf(sy);
        y0 = y0 < 0 ? 0 : (y0 > h - 1 ? h - 1 : y0);
        const int y1 = y0 + 1 > h - 1 ? h - 1 : y0 + 1;
        const float wy = sy - (float) y0;
        for (int dx = 0; dx < S; dx++) {
            const float sx = ((float) dx + 0.5f) * xs - 0.5f;
            int x0 = (int) floorf(sx);
            x0 = x0 < 0 ? 0 : (x0 > w - 1 ? w - 1 : x0);
            const int x1 = x0 + 1 > w - 1 ? w - 1 : x0 + 1;
            const float wx = sx - (float) x0;
            for (int c = 0; c < 3; c++) {
                const float p00 = (float) src[((int64_t) y0 * w + x0) * 3 + c] / 255.0f;
                const float p01 = (float) src[((int64_t) y0 * w + x1) * 3 + c] / 255.0f;
                const float p10 = (float) src[((int64_t) y1 * w + x0) * 3 + c] / 255.0f;
                const float p11 = (float) src[((int64_t) y1 * w + x1) * 3 + c] / 255.0f;
                const float top = p00 + (p01 - p00) * wx;
                const float bot = p10 + (p11 - p10) * wx;
                const float v = top + (bot - top) * wy;
                out[((int64_t) c * S + dy) * S + dx] = (v - 0.5f) / 0.5f;
            }
        }
    }
}
