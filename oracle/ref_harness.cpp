// Test-infrastructure harness around the reference's own CPU code.
//
// Compiled by oracle/Makefile together with the reference's ggml sources and
// src/vision_trunk.cpp + src/gguf_model.cpp, straight from where they lie in
// the reference tree, into oracle/_ref/libsam3ref_*.so.  It is only ever used
// as a checker (pinning the C restatement in s3t_oracle.c) and as the timed
// CPU baseline; nothing in the product links it.
//
// Every entry point runs one small ggml graph on the ggml CPU backend, in the
// style of ggml/tests/test-backend-ops.cpp, or the reference trunk itself.
// All functions return 0 on success and -1 on failure.

#include "ggml.h"
#include "ggml-cpu.h"
#include "ggml-backend.h"
#include "sam3/gguf_model.h"
#include "sam3/vision_trunk.h"
#include "sam3/vision_neck.h"

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

struct Ctx {
    ggml_context * ctx = nullptr;
    explicit Ctx(size_t bytes) {
        ggml_init_params p{bytes, nullptr, false};
        ctx = ggml_init(p);
    }
    ~Ctx() { if (ctx) ggml_free(ctx); }
};

int compute(ggml_context * ctx, ggml_tensor * out, int n_threads) {
    ggml_cgraph * gf = ggml_new_graph_custom(ctx, 4096, false);
    ggml_build_forward_expand(gf, out);
    return ggml_graph_compute_with_ctx(ctx, gf, n_threads) == GGML_STATUS_SUCCESS ? 0 : -1;
}

}  // namespace

extern "C" {

const char * ref_last_error(void) { return g_err.c_str(); }

// sam3::VisionTrunk::run (src/vision_trunk.cpp:297) on the ggml CPU backend.
// image: [1,3,1008,1008] fp32; out: [1,1024,72,72] fp32.  *seconds receives the
// wall time of run() alone (model load excluded).
int ref_trunk_run(const char * gguf_path, const float * image, float * out,
                  int n_threads, double * seconds) {
    try {
        sam3::GgufModel model;
        if (!model.load(gguf_path, /*prefer_gpu=*/false)) {
            g_err = "failed to load model";
            return -1;
        }
        if (n_threads > 0) ggml_backend_cpu_set_n_threads(model.backend(), n_threads);
        std::vector<float> img(image, image + 3ull * 1008 * 1008);
        sam3::VisionTrunk trunk(model);
        auto t0 = std::chrono::steady_clock::now();
        sam3::VisionTrunkOutput r = trunk.run(img, {1, 3, 1008, 1008});
        auto t1 = std::chrono::steady_clock::now();
        if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
        std::memcpy(out, r.trunk_nchw.data(), r.trunk_nchw.size() * sizeof(float));
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
        return -1;
    }
}

// Load once, run many: keeps the GgufModel alive so the CPU baseline can time
// repeated VisionTrunk::run calls without the load.
void * ref_model_load(const char * gguf_path, int n_threads) {
    auto * m = new sam3::GgufModel();
    if (!m->load(gguf_path, false)) { delete m; g_err = "failed to load model"; return nullptr; }
    if (n_threads > 0) ggml_backend_cpu_set_n_threads(m->backend(), n_threads);
    return m;
}

int ref_model_run(void * handle, const float * image, float * out, double * seconds) {
    try {
        auto * m = static_cast<sam3::GgufModel *>(handle);
        std::vector<float> img(image, image + 3ull * 1008 * 1008);
        sam3::VisionTrunk trunk(*m);
        auto t0 = std::chrono::steady_clock::now();
        sam3::VisionTrunkOutput r = trunk.run(img, {1, 3, 1008, 1008});
        auto t1 = std::chrono::steady_clock::now();
        if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
        if (out) std::memcpy(out, r.trunk_nchw.data(), r.trunk_nchw.size() * sizeof(float));
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
        return -1;
    }
}

void ref_model_free(void * handle) { delete static_cast<sam3::GgufModel *>(handle); }

// y[M][N] = ggml_mul_mat(W, x): W has ggml type wtype (0=F32, 1=F16, 8=Q8_0)
// and ne = [K, N] (row n holds output channel n, K contiguous); x is f32 [M][K].
int ref_mul_mat(int wtype, const void * w, int64_t N, int64_t K, const float * x,
                int64_t M, float * y, int n_threads) {
    const ggml_type t = (ggml_type) wtype;
    const size_t wbytes = ggml_row_size(t, K) * N;
    Ctx c(wbytes + (size_t) (M * K + M * N) * 4 * 2 + 64 * 1024 * 1024);
    ggml_tensor * tw = ggml_new_tensor_2d(c.ctx, t, K, N);
    ggml_tensor * tx = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, K, M);
    std::memcpy(tw->data, w, wbytes);
    std::memcpy(tx->data, x, (size_t) M * K * 4);
    ggml_tensor * ty = ggml_mul_mat(c.ctx, tw, tx);
    if (compute(c.ctx, ty, n_threads)) return -1;
    std::memcpy(y, ty->data, (size_t) M * N * 4);
    return 0;
}

// ggml_norm (eps) over rows of x [rows][cols]; no affine part.
int ref_norm(const float * x, int64_t rows, int64_t cols, float eps, float * y) {
    Ctx c((size_t) rows * cols * 4 * 3 + 16 * 1024 * 1024);
    ggml_tensor * tx = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, cols, rows);
    std::memcpy(tx->data, x, (size_t) rows * cols * 4);
    ggml_tensor * ty = ggml_norm(c.ctx, tx, eps);
    if (compute(c.ctx, ty, 4)) return -1;
    std::memcpy(y, ty->data, (size_t) rows * cols * 4);
    return 0;
}

// The axial RoPE of src/vision_trunk.cpp:145-205 built from the same ggml ops:
// x is [tokens][heads][64] f32; dims 0..31 rotate with pos_x, 32..63 with pos_y.
int ref_rope_axial(const float * x, int64_t tokens, int64_t heads, const int32_t * pos_x,
                   const int32_t * pos_y, float freq_scale, float * y) {
    const size_t n = (size_t) tokens * heads * 64;
    Ctx c(n * 4 * 8 + 16 * 1024 * 1024);
    ggml_tensor * tx = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, 64, heads, tokens, 1);
    ggml_tensor * px = ggml_new_tensor_1d(c.ctx, GGML_TYPE_I32, tokens);
    ggml_tensor * py = ggml_new_tensor_1d(c.ctx, GGML_TYPE_I32, tokens);
    std::memcpy(tx->data, x, n * 4);
    std::memcpy(px->data, pos_x, tokens * 4);
    std::memcpy(py->data, pos_y, tokens * 4);
    ggml_tensor * first = ggml_view_4d(c.ctx, tx, 32, heads, tokens, 1, tx->nb[1], tx->nb[2], tx->nb[3], 0);
    ggml_tensor * second = ggml_view_4d(c.ctx, tx, 32, heads, tokens, 1, tx->nb[1], tx->nb[2], tx->nb[3], 32 * 4);
    first = ggml_rope_ext(c.ctx, first, px, nullptr, 32, 0, 32768, 10000.0f, freq_scale, 0.0f, 1.0f, 0.0f, 0.0f);
    second = ggml_rope_ext(c.ctx, second, py, nullptr, 32, 0, 32768, 10000.0f, freq_scale, 0.0f, 1.0f, 0.0f, 0.0f);
    ggml_tensor * ty = ggml_concat(c.ctx, first, second, 0);
    if (compute(c.ctx, ty, 4)) return -1;
    std::memcpy(y, ty->data, n * 4);
    return 0;
}

// ggml_flash_attn_ext with no mask, prec F32, as src/vision_trunk.cpp:207-228.
// q: [nq][heads][d], k/v: [nk][heads][d] f32; out: [nq][heads][d] f32.
int ref_flash_attn(const float * q, const float * k, const float * v, int64_t nq, int64_t nk,
                   int64_t heads, int64_t d, float scale, float * out, int n_threads) {
    const size_t bytes = (size_t) (2 * nq + 2 * nk) * heads * d * 4;
    Ctx c(bytes * 2 + (size_t) nq * nk * 8 + 64 * 1024 * 1024);
    ggml_tensor * tq = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, d, heads, nq, 1);
    ggml_tensor * tk = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, d, heads, nk, 1);
    ggml_tensor * tv = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, d, heads, nk, 1);
    std::memcpy(tq->data, q, (size_t) nq * heads * d * 4);
    std::memcpy(tk->data, k, (size_t) nk * heads * d * 4);
    std::memcpy(tv->data, v, (size_t) nk * heads * d * 4);
    ggml_tensor * r = ggml_flash_attn_ext(c.ctx, ggml_permute(c.ctx, tq, 0, 2, 1, 3),
                                          ggml_permute(c.ctx, tk, 0, 2, 1, 3),
                                          ggml_permute(c.ctx, tv, 0, 2, 1, 3), nullptr, scale, 0.0f, 0.0f);
    ggml_flash_attn_ext_set_prec(r, GGML_PREC_F32);
    if (compute(c.ctx, r, n_threads)) return -1;
    std::memcpy(out, r->data, (size_t) nq * heads * d * 4);
    return 0;
}

// ggml_flash_attn_ext, prec F32, with an F16 mask [nq][nk] (ne0 = nk), as
// mha() of src/encoder_fusion.cpp:63-88 builds it (:120-133, :229).  The mask
// row is key_mask (f32 [nk], converted to f16) repeated for every query; a
// null key_mask gives no mask tensor.  Layouts as ref_flash_attn.
int ref_flash_attn_masked(const float * q, const float * k, const float * v, int64_t nq, int64_t nk,
                          int64_t heads, int64_t d, float scale, const float * key_mask, float * out,
                          int n_threads) {
    const size_t bytes = (size_t) (2 * nq + 2 * nk) * heads * d * 4 + (size_t) nq * nk * 2;
    Ctx c(bytes * 2 + (size_t) nq * nk * 8 + 64 * 1024 * 1024);
    ggml_tensor * tq = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, d, heads, nq, 1);
    ggml_tensor * tk = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, d, heads, nk, 1);
    ggml_tensor * tv = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, d, heads, nk, 1);
    std::memcpy(tq->data, q, (size_t) nq * heads * d * 4);
    std::memcpy(tk->data, k, (size_t) nk * heads * d * 4);
    std::memcpy(tv->data, v, (size_t) nk * heads * d * 4);
    ggml_tensor * tm = nullptr;
    if (key_mask) {
        tm = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F16, nk, nq);
        ggml_fp16_t * m = (ggml_fp16_t *) tm->data;
        for (int64_t i = 0; i < nq; ++i)
            for (int64_t j = 0; j < nk; ++j) m[i * nk + j] = ggml_fp32_to_fp16(key_mask[j]);
    }
    ggml_tensor * r = ggml_flash_attn_ext(c.ctx, ggml_permute(c.ctx, tq, 0, 2, 1, 3),
                                          ggml_permute(c.ctx, tk, 0, 2, 1, 3),
                                          ggml_permute(c.ctx, tv, 0, 2, 1, 3), tm, scale, 0.0f, 0.0f);
    ggml_flash_attn_ext_set_prec(r, GGML_PREC_F32);
    if (compute(c.ctx, r, n_threads)) return -1;
    std::memcpy(out, r->data, (size_t) nq * heads * d * 4);
    return 0;
}

// The decoder's mha() (src/decoder.cpp:95-127) as a ggml graph: the same
// views, ggml_mul_mat for the scores, ggml_soft_max_ext with the mask and
// ggml_mul_mat with the transposed V.  bias: F32 [heads][nq][nk] as
// image_bias_t (:418); key_mask: [nk] written as the F16 prompt mask rows
// (:131-143, :414).  q: [nq][heads*d], k/v: [nk][heads*d]; out [nq][heads*d].
int ref_decoder_mha(const float * q, const float * k, const float * v, int64_t nq, int64_t nk, int64_t heads,
                    int64_t d, float scale, const float * bias, const float * key_mask, float * out,
                    int n_threads) {
    const size_t bytes = (size_t) (2 * nq + 2 * nk) * heads * d * 4 + (size_t) nq * nk * heads * 4 * 4;
    Ctx c(bytes * 3 + 64 * 1024 * 1024);
    ggml_tensor * tq = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, heads * d, nq);
    ggml_tensor * tk = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, heads * d, nk);
    ggml_tensor * tv = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F32, heads * d, nk);
    std::memcpy(tq->data, q, (size_t) nq * heads * d * 4);
    std::memcpy(tk->data, k, (size_t) nk * heads * d * 4);
    std::memcpy(tv->data, v, (size_t) nk * heads * d * 4);
    ggml_tensor * tm = nullptr;
    if (bias) {
        tm = ggml_new_tensor_3d(c.ctx, GGML_TYPE_F32, nk, nq, heads);
        std::memcpy(tm->data, bias, (size_t) nk * nq * heads * 4);
    } else if (key_mask) {
        tm = ggml_new_tensor_2d(c.ctx, GGML_TYPE_F16, nk, nq);
        ggml_fp16_t * m = (ggml_fp16_t *) tm->data;
        for (int64_t i = 0; i < nq; ++i)
            for (int64_t j = 0; j < nk; ++j) m[i * nk + j] = ggml_fp32_to_fp16(key_mask[j]);
    }
    ggml_tensor * qh = ggml_permute(c.ctx, ggml_cont_3d(c.ctx, tq, d, heads, nq), 0, 2, 1, 3);
    ggml_tensor * kh = ggml_permute(c.ctx, ggml_cont_3d(c.ctx, tk, d, heads, nk), 0, 2, 1, 3);
    ggml_tensor * vh = ggml_cont_3d(c.ctx, ggml_permute(c.ctx, ggml_cont_3d(c.ctx, tv, d, heads, nk), 1, 2, 0, 3),
                                    nk, d, heads);
    ggml_tensor * scores = ggml_mul_mat(c.ctx, kh, qh);
    ggml_tensor * probs = ggml_soft_max_ext(c.ctx, scores, tm, scale, 0.0f);
    ggml_tensor * attn = ggml_mul_mat(c.ctx, vh, probs);
    ggml_tensor * r = ggml_cont_2d(c.ctx, ggml_permute(c.ctx, attn, 0, 2, 1, 3), heads * d, nq);
    if (compute(c.ctx, r, n_threads)) return -1;
    std::memcpy(out, r->data, (size_t) nq * heads * d * 4);
    return 0;
}

int ref_gelu_erf(const float * x, int64_t n, float * y) {
    Ctx c((size_t) n * 4 * 3 + 16 * 1024 * 1024);
    ggml_tensor * tx = ggml_new_tensor_1d(c.ctx, GGML_TYPE_F32, n);
    std::memcpy(tx->data, x, n * 4);
    ggml_tensor * ty = ggml_gelu_erf(c.ctx, tx);
    if (compute(c.ctx, ty, 1)) return -1;
    std::memcpy(y, ty->data, n * 4);
    return 0;
}

// The activation quantizer ggml's CPU mul_mat applies before a Q8_0 dot
// (type_traits_cpu[Q8_0].from_float, ggml-cpu/arch/x86/quants.c).
int ref_quantize_q8_0_act(const float * x, int64_t n, void * blocks) {
    ggml_cpu_init();
    const auto * tr = ggml_get_type_traits_cpu(GGML_TYPE_Q8_0);
    tr->from_float(x, blocks, n);
    return 0;
}

// The file-format dequantizers (ggml type_traits.to_float): F16 and Q8_0.
int ref_to_float(int type, const void * src, int64_t n, float * y) {
    const auto * tr = ggml_get_type_traits((ggml_type) type);
    if (!tr->to_float) { g_err = "no to_float"; return -1; }
    tr->to_float(src, y, n);
    return 0;
}

int ref_fp32_to_fp16(const float * x, int64_t n, uint16_t * y) {
    ggml_fp32_to_fp16_row(x, (ggml_fp16_t *) y, n);
    return 0;
}

// Patch embed + token-major permute as src/vision_trunk.cpp:284-291,364-368.
// w: GGUF patch_embed.proj.weight bytes, ne = [3,14,14,1024] of type wtype;
// image [3][1008][1008] f32; out [5184][1024] f32 (token-major, x fastest).
int ref_patch_embed(int wtype, const void * w, const float * image, float * out, int n_threads) {
    const ggml_type t = (ggml_type) wtype;
    const int64_t wn = 3 * 14 * 14 * 1024;
    Ctx c((size_t) 1024 * 1024 * 1024);
    ggml_tensor * tw = ggml_new_tensor_4d(c.ctx, t, 3, 14, 14, 1024);
    ggml_tensor * ti = ggml_new_tensor_4d(c.ctx, GGML_TYPE_F32, 1008, 1008, 3, 1);
    std::memcpy(tw->data, w, ggml_row_size(t, wn));
    std::memcpy(ti->data, image, (size_t) 3 * 1008 * 1008 * 4);
    ggml_tensor * wg = ggml_cont(c.ctx, ggml_permute(c.ctx, tw, 2, 0, 1, 3));
    ggml_tensor * r = ggml_conv_2d(c.ctx, wg, ti, 14, 14, 0, 0, 1, 1);
    r = ggml_cont(c.ctx, ggml_permute(c.ctx, r, 1, 2, 0, 3));
    if (compute(c.ctx, r, n_threads)) return -1;
    std::memcpy(out, r->data, (size_t) 5184 * 1024 * 4);
    return 0;
}


// ---------------------------------------------------------------------------
// The stem and one trunk block, each as its own ggml graph (per-block parity).
//
// src/vision_trunk.cpp builds the stem and all 32 blocks into one graph
// (:362-459) from helpers private to that file, so the harness states the same
// ggml ops in the same order: layer_norm (:64-74); linear over row chunks of
// qkv (:50-62, :76-102); gpu_win_part / gpu_win_unpart (:235-282);
// apply_axial_rope (:145-205); apply_attention (:207-228); gelu_erf and the
// residual adds (:439-458).  ggml's own CPU kernels do all of the arithmetic.
// That these graphs compute exactly what VisionTrunk::run computes is pinned
// by tests/golden/block_pin_<fmt>.npz: VisionTrunk::run on files whose other
// blocks are exact identities (zero proj/fc2 weights and biases).

}  // extern "C"

namespace {

const std::string kTrunkPrefix = "backbone.vision_backbone.trunk";
constexpr int64_t kC = 1024, kG = 72, kW = 24, kNh = 16, kHd = 64, kPre = 24;

ggml_tensor * need(const sam3::GgufModel & m, const std::string & name) {
    ggml_tensor * t = m.find_weight(name);
    if (!t) throw std::runtime_error("missing tensor: " + name);
    return t;
}

ggml_tensor * f32(ggml_context * ctx, ggml_tensor * t) {
    return t->type == GGML_TYPE_F32 ? t : ggml_cast(ctx, t, GGML_TYPE_F32);
}

ggml_tensor * norm_affine(ggml_context * ctx, ggml_tensor * x, ggml_tensor * g, ggml_tensor * b) {
    ggml_tensor * y = ggml_norm(ctx, f32(ctx, x), 1e-5f);
    y = ggml_mul(ctx, y, ggml_repeat(ctx, f32(ctx, g), y));
    return ggml_add(ctx, y, ggml_repeat(ctx, f32(ctx, b), y));
}

ggml_tensor * dense(ggml_context * ctx, ggml_tensor * w, ggml_tensor * b, ggml_tensor * x) {
    ggml_tensor * y = f32(ctx, ggml_mul_mat(ctx, w, x));
    return ggml_add(ctx, y, ggml_repeat(ctx, f32(ctx, b), y));
}

// rows [row0, row0 + n) of a [K, N] weight and of its bias
ggml_tensor * dense_rows(ggml_context * ctx, ggml_tensor * w, ggml_tensor * b, int64_t row0, int64_t n,
                         ggml_tensor * x) {
    ggml_tensor * wv = ggml_view_2d(ctx, w, w->ne[0], n, w->nb[1], size_t(row0) * w->nb[1]);
    ggml_tensor * bv = ggml_view_1d(ctx, b, n, size_t(row0) * ggml_element_size(b));
    return dense(ctx, wv, bv, x);
}

// [C, W, H, 1] -> [C, win, win, nWy * nWx], windows numbered wy + nWy * wx
ggml_tensor * to_windows(ggml_context * ctx, ggml_tensor * x) {
    const int64_t nw = kG / kW;
    ggml_tensor * t = ggml_reshape_4d(ctx, x, kC, kW, nw, kG);
    t = ggml_cont(ctx, ggml_permute(ctx, t, 0, 1, 3, 2));
    return ggml_reshape_4d(ctx, t, kC, kW, kW, nw * nw);
}

ggml_tensor * from_windows(ggml_context * ctx, ggml_tensor * x) {
    const int64_t nw = kG / kW;
    ggml_tensor * t = ggml_reshape_4d(ctx, x, kC, kW, kG, nw);
    t = ggml_cont(ctx, ggml_permute(ctx, t, 0, 1, 3, 2));
    return ggml_reshape_4d(ctx, t, kC, kG, kG, 1);
}

ggml_tensor * rope_xy(ggml_context * ctx, ggml_tensor * x, ggml_tensor * px, ggml_tensor * py, float scale) {
    const int64_t h = x->ne[0] / 2;
    ggml_tensor * a = ggml_view_4d(ctx, x, h, x->ne[1], x->ne[2], x->ne[3], x->nb[1], x->nb[2], x->nb[3], 0);
    ggml_tensor * b = ggml_view_4d(ctx, x, h, x->ne[1], x->ne[2], x->ne[3], x->nb[1], x->nb[2], x->nb[3],
                                   size_t(h) * ggml_element_size(x));
    a = ggml_rope_ext(ctx, a, px, nullptr, int(h), 0, 32768, 10000.0f, scale, 0.0f, 1.0f, 0.0f, 0.0f);
    b = ggml_rope_ext(ctx, b, py, nullptr, int(h), 0, 32768, 10000.0f, scale, 0.0f, 1.0f, 0.0f, 0.0f);
    return ggml_concat(ctx, a, b, 0);
}

std::vector<int32_t> axis_positions(int64_t grid, bool x_axis) {
    std::vector<int32_t> p(size_t(grid * grid));
    for (int64_t i = 0; i < grid * grid; ++i) p[size_t(i)] = int32_t(x_axis ? i % grid : i / grid);
    return p;
}

// A no_alloc context for one graph plus the scheduler over the model's backend.
struct OneGraph {
    static constexpr size_t kNodes = 8192;
    std::vector<uint8_t> meta;
    ggml_context * ctx = nullptr;
    ggml_backend_sched_t sched = nullptr;
    ggml_backend_t backend = nullptr;
    std::vector<std::pair<ggml_tensor *, const void *>> inputs;

    explicit OneGraph(const sam3::GgufModel & m) : backend(m.backend()) {
        meta.resize(ggml_tensor_overhead() * kNodes + ggml_graph_overhead_custom(kNodes, false));
        ggml_init_params p{meta.size(), meta.data(), true};
        ctx = ggml_init(p);
        sched = ggml_backend_sched_new(&backend, nullptr, 1, kNodes, false, true);
        if (!ctx || !sched) throw std::runtime_error("graph setup failed");
    }
    ~OneGraph() {
        if (sched) ggml_backend_sched_free(sched);
        if (ctx) ggml_free(ctx);
    }
    ggml_tensor * input(ggml_type t, int64_t n0, int64_t n1, int64_t n2, int64_t n3, const void * data) {
        ggml_tensor * x = ggml_new_tensor_4d(ctx, t, n0, n1, n2, n3);
        inputs.emplace_back(x, data);
        return x;
    }
    void run(ggml_tensor * out, float * dst) {
        ggml_cgraph * gf = ggml_new_graph_custom(ctx, kNodes, false);
        ggml_build_forward_expand(gf, out);
        for (auto & in : inputs) ggml_backend_sched_set_tensor_backend(sched, in.first, backend);
        if (!ggml_backend_sched_alloc_graph(sched, gf)) throw std::runtime_error("graph allocation failed");
        for (auto & in : inputs) ggml_backend_tensor_set(in.first, in.second, 0, ggml_nbytes(in.first));
        if (ggml_backend_sched_graph_compute(sched, gf) != GGML_STATUS_SUCCESS)
            throw std::runtime_error("graph compute failed");
        ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
    }
};

}  // namespace

extern "C" {

// Patch embed + tiled position embedding + ln_pre (src/vision_trunk.cpp:284-291,
// 111-132, 362-374) of the model behind `handle` (ref_model_load).
// image [3][1008][1008] f32 -> out [5184][1024] f32, token t = y*72 + x.
int ref_trunk_stem(void * handle, const float * image, float * out) {
    try {
        const auto & m = *static_cast<const sam3::GgufModel *>(handle);
        ggml_tensor * pe = need(m, kTrunkPrefix + ".pos_embed");
        if (ggml_nelements(pe) != (kPre * kPre + 1) * kC) throw std::runtime_error("unexpected trunk.pos_embed size");
        std::vector<float> pos(size_t(ggml_nelements(pe)));
        ggml_backend_tensor_get(pe, pos.data(), 0, pos.size() * 4);
        std::vector<float> tiled(size_t(kG * kG * kC));
        for (int64_t t = 0; t < kG * kG; ++t) {
            const int64_t src = 1 + (t / kG % kPre) * kPre + (t % kG % kPre);
            std::memcpy(&tiled[size_t(t * kC)], &pos[size_t(src * kC)], kC * 4);
        }
        OneGraph g(m);
        ggml_tensor * img = g.input(GGML_TYPE_F32, 1008, 1008, 3, 1, image);
        ggml_tensor * abs_pos = g.input(GGML_TYPE_F32, kC, kG, kG, 1, tiled.data());
        ggml_tensor * w = need(m, kTrunkPrefix + ".patch_embed.proj.weight");
        ggml_tensor * cur = ggml_conv_2d(g.ctx, ggml_cont(g.ctx, ggml_permute(g.ctx, w, 2, 0, 1, 3)), img,
                                         14, 14, 0, 0, 1, 1);
        cur = ggml_cont(g.ctx, ggml_permute(g.ctx, cur, 1, 2, 0, 3));
        cur = ggml_add(g.ctx, cur, abs_pos);
        cur = norm_affine(g.ctx, cur, need(m, kTrunkPrefix + ".ln_pre.weight"), need(m, kTrunkPrefix + ".ln_pre.bias"));
        g.run(cur, out);
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
        return -1;
    }
}

// Block `layer` of the trunk (src/vision_trunk.cpp:377-459) on the model behind
// `handle`: x [5184][1024] f32 (the block's input residual, token-major) ->
// out [5184][1024] f32 (its output residual).
int ref_trunk_block(void * handle, int layer, const float * x, float * out) {
    try {
        const auto & m = *static_cast<const sam3::GgufModel *>(handle);
        const std::string b = kTrunkPrefix + ".blocks." + std::to_string(layer);
        const bool global = layer == 7 || layer == 15 || layer == 23 || layer == 31;
        const int64_t side = global ? kG : kW;
        const std::vector<int32_t> px = axis_positions(side, true), py = axis_positions(side, false);
        OneGraph g(m);
        ggml_context * ctx = g.ctx;
        ggml_tensor * inp = g.input(GGML_TYPE_F32, kC, kG, kG, 1, x);
        ggml_tensor * pos_x = g.input(GGML_TYPE_I32, side * side, 1, 1, 1, px.data());
        ggml_tensor * pos_y = g.input(GGML_TYPE_I32, side * side, 1, 1, 1, py.data());

        ggml_tensor * cur = norm_affine(ctx, inp, need(m, b + ".norm1.weight"), need(m, b + ".norm1.bias"));
        if (!global) cur = to_windows(ctx, cur);
        const int64_t w = cur->ne[1], h = cur->ne[2], nb = cur->ne[3], tokens = w * h;
        ggml_tensor * qw = need(m, b + ".attn.qkv.weight");
        ggml_tensor * qb = need(m, b + ".attn.qkv.bias");
        ggml_tensor * q = ggml_reshape_4d(ctx, dense_rows(ctx, qw, qb, 0, kC, cur), kHd, kNh, tokens, nb);
        ggml_tensor * k = ggml_reshape_4d(ctx, dense_rows(ctx, qw, qb, kC, kC, cur), kHd, kNh, tokens, nb);
        ggml_tensor * v = ggml_reshape_4d(ctx, dense_rows(ctx, qw, qb, 2 * kC, kC, cur), kHd, kNh, tokens, nb);
        const float scale = global ? float(kW) / float(kG) : 1.0f;
        q = rope_xy(ctx, q, pos_x, pos_y, scale);
        k = rope_xy(ctx, k, pos_x, pos_y, scale);
        ggml_tensor * att = ggml_flash_attn_ext(ctx, ggml_permute(ctx, q, 0, 2, 1, 3), ggml_permute(ctx, k, 0, 2, 1, 3),
                                                ggml_permute(ctx, v, 0, 2, 1, 3), nullptr, 1.0f / std::sqrt(float(kHd)),
                                                0.0f, 0.0f);
        ggml_flash_attn_ext_set_prec(att, GGML_PREC_F32);
        att = ggml_reshape_2d(ctx, att, att->ne[0] * att->ne[1], att->ne[2] * att->ne[3]);
        att = ggml_reshape_4d(ctx, att, kC, w, h, nb);
        att = dense(ctx, need(m, b + ".attn.proj.weight"), need(m, b + ".attn.proj.bias"), att);
        if (!global) att = from_windows(ctx, att);
        cur = ggml_add(ctx, inp, att);

        ggml_tensor * ffn = norm_affine(ctx, cur, need(m, b + ".norm2.weight"), need(m, b + ".norm2.bias"));
        ffn = dense(ctx, need(m, b + ".mlp.fc1.weight"), need(m, b + ".mlp.fc1.bias"), ffn);
        ffn = ggml_gelu_erf(ctx, ffn);
        ffn = dense(ctx, need(m, b + ".mlp.fc2.weight"), need(m, b + ".mlp.fc2.bias"), ffn);
        g.run(ggml_add(ctx, cur, ffn), out);
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The vision neck (src/vision_neck.cpp), the consumer of the trunk's output.

extern "C" {

// sam3::VisionNeck::run (src/vision_neck.cpp:203-393) for one level
// (only_level) of the model behind `handle`: trunk [1][1024][72][72] fp32 NCHW
// -> out, the level's NCHW feature map.  shape[4] receives its shape.
int ref_neck_run(void * handle, int level, const float * trunk, float * out, int64_t * shape) {
    try {
        const auto & m = *static_cast<const sam3::GgufModel *>(handle);
        std::vector<float> x(trunk, trunk + size_t(kC) * kG * kG);
        sam3::VisionNeck neck(m);
        const sam3::VisionNeckOutput r = neck.run(x, {1, kC, kG, kG}, std::optional<int>(level));
        std::memcpy(out, r.levels[0].data(), r.levels[0].size() * sizeof(float));
        for (int i = 0; i < 4; ++i) shape[i] = r.shapes[0][i];
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"

namespace {

ggml_tensor * conv_bias(ggml_context * ctx, ggml_tensor * w, ggml_tensor * b, ggml_tensor * x) {
    // MLX [OC, KH, KW, IC] lands in ggml as ne [IC, KW, KH, OC]; ggml_conv_2d
    // takes [KW, KH, IC, OC].  1x1, stride 1, no padding.
    ggml_tensor * wk = ggml_cont(ctx, ggml_permute(ctx, w, 2, 0, 1, 3));
    ggml_tensor * y = ggml_conv_2d(ctx, wk, x, 1, 1, 0, 0, 1, 1);
    ggml_tensor * bb = ggml_reshape_4d(ctx, f32(ctx, b), 1, 1, wk->ne[3], 1);
    return ggml_add(ctx, y, bb);
}

// 2x2 stride-2 transposed conv as one mul_mat over the channels plus a pixel
// shuffle, on x [W, H, IC, 1] -> [W*2, H*2, OC, 1] (NCHW order).
ggml_tensor * deconv_bias(ggml_context * ctx, ggml_tensor * w, ggml_tensor * b, ggml_tensor * x) {
    const int64_t ic = w->ne[0], oc = w->ne[3], wd = x->ne[0], ht = x->ne[1];
    ggml_tensor * wf = ggml_reshape_2d(ctx, ggml_cont(ctx, ggml_permute(ctx, w, 0, 2, 3, 1)), ic, oc * 4);
    ggml_tensor * xf = ggml_reshape_2d(ctx, ggml_cont(ctx, ggml_permute(ctx, x, 2, 0, 1, 3)), ic, wd * ht);
    ggml_tensor * y = ggml_mul_mat(ctx, wf, xf);                                  // [oc*4, W*H], row oc + oc*(kw + 2 kh)
    y = ggml_reshape_4d(ctx, y, oc * 2, 2, wd, ht);                               // [oc, kw | kh | W | H]
    y = ggml_cont(ctx, ggml_permute(ctx, y, 0, 2, 1, 3));                         // [oc*2, W, kh, H]
    y = ggml_reshape_4d(ctx, y, oc, 2 * wd, 2 * ht, 1);                           // [oc, 2W, 2H]
    y = ggml_add(ctx, y, ggml_reshape_4d(ctx, f32(ctx, b), oc, 1, 1, 1));
    return ggml_cont(ctx, ggml_permute(ctx, y, 2, 0, 1, 3));                      // [2W, 2H, oc]
}

}  // namespace

extern "C" {

// The first operation of neck level `level` (src/vision_neck.cpp:262-345) on
// trunk [1][1024][72][72] fp32 NCHW, as its own ggml graph: level 0 the first
// 2x2 deconv + bias followed by its GELU, level 1 the 2x2 deconv + bias,
// level 2 the 1x1 conv + bias, level 3 the 2x2 max pool then the 1x1 conv +
// bias.  out receives the NCHW result, shape[4] its shape.
int ref_neck_first(void * handle, int level, const float * trunk, float * out, int64_t * shape) {
    try {
        const auto & m = *static_cast<const sam3::GgufModel *>(handle);
        const std::string p = "backbone.vision_backbone.convs." + std::to_string(level) + ".";
        OneGraph g(m);
        ggml_context * ctx = g.ctx;
        ggml_tensor * x = g.input(GGML_TYPE_F32, kG, kG, kC, 1, trunk);
        ggml_tensor * y = nullptr;
        if (level == 0) {
            y = ggml_gelu_erf(ctx, deconv_bias(ctx, need(m, p + "dconv_2x2_0.weight"), need(m, p + "dconv_2x2_0.bias"), x));
        } else if (level == 1) {
            y = deconv_bias(ctx, need(m, p + "dconv_2x2.weight"), need(m, p + "dconv_2x2.bias"), x);
        } else if (level == 2 || level == 3) {
            if (level == 3) x = ggml_pool_2d(ctx, x, GGML_OP_POOL_MAX, 2, 2, 2, 2, 0, 0);
            y = conv_bias(ctx, need(m, p + "conv_1x1.weight"), need(m, p + "conv_1x1.bias"), x);
        } else {
            throw std::runtime_error("level must be in [0, 3]");
        }
        g.run(y, out);
        shape[0] = 1;
        shape[1] = y->ne[2];
        shape[2] = y->ne[1];
        shape[3] = y->ne[0];
        return 0;
    } catch (const std::exception & e) {
        g_err = e.what();
        return -1;
    }
}

}  // extern "C"
