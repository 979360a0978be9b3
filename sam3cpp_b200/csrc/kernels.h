// Host-side launch interface of the trunk kernels (sm_100a).  Every launcher
// returns a cudaError_t and never synchronizes.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace s3t {

constexpr int kImage = 1008, kPatch = 14, kGrid = 72, kTokens = 5184, kDim = 1024;
constexpr int kHeads = 16, kHeadDim = 64, kMlp = 4736, kLayers = 32, kWindow = 24;
constexpr int kPatchK = 3 * 14 * 14;       // 588
constexpr int kPatchKPad = 640;            // padded to the 64-wide K block
constexpr int kMaxSourceSide = 32768;      // largest source image side the preprocessing accepts

// Error codes written to the device status word (first writer wins).
enum : int {
    kErrNone = 0,
    kErrTimeoutProducer = 1,
    kErrTimeoutMma = 2,
    kErrTimeoutEpilogue = 3,
    kErrTimeoutDrain = 4,
    kErrTimeoutProbe = 5,    // the wait-timeout self-test (s3t_selftest_wait_timeout)
};

enum GemmEpilogue : int {
    kEpiF16 = 0,     // out16 = act(acc + bias) [optional GELU, optional Q8_0 rounding]
    kEpiQkv = 1,     // acc + bias, RoPE on q/k, scattered into the attention layout
    kEpiResid = 2,   // x += acc + bias (fp32 residual), optional NCHW copy
    kEpiPatch = 3,   // x = acc + tiled pos_embed (fp32)
};

struct GemmArgs {
    int M, N, K;
    const float* bias;        // [N] or null
    __half* out16;            // kEpiF16: [M][N]
    int gelu;                 // kEpiF16: apply GELU (erf)
    int q8;                   // kEpiF16: Q8_0 activation rounding of the output
    float* resid;             // kEpiResid / kEpiPatch: x [M][N] fp32
    float* out_nchw;          // kEpiResid: also write [img][N][5184] (or null)
    const float* pos;         // kEpiPatch: pos_embed [577][1024]
    __half* qkv;              // kEpiQkv: q block; k at +qkv_stride, v at +2*qkv_stride
    int64_t qkv_stride;
    int windowed;             // kEpiQkv: 24x24 windows (1) or whole image (0)
    const float* rope_local;  // [24][2][16] cos,sin for scale 1
    const float* rope_global; // [72][2][16] cos,sin for scale 24/72
    const float* rope_local_t;  // the same tables transposed: [2][16][24]
    const float* rope_global_t; // [2][16][72]
    int* status;              // device status word
    // Stream-K split of the pair kernel's K loop (null: whole tiles only).
    // sk_work: kSkSlotFloats floats per CTA pair, sk_flags: kSkSlotFlags ints
    // per CTA pair, all zero between launches.  sk is set by the launcher.
    float* sk_work;
    int* sk_flags;
    int sk_slots;             // CTA pairs the two buffers have room for
    int sk;
};
constexpr int kSkSlotFloats = 256 * 256;       // a pair's raw 256 x 256 fp32 accumulator
constexpr int kSkSlotFlags = 2 * 8;            // one per epilogue warp of each CTA

// Programmatic dependent launch for the trunk's chain of kernels.  While a
// PdlScope(true) lives on this thread, the trunk launchers (pair GEMM,
// attention, LayerNorm, im2col) add the programmatic-stream-serialization
// attribute: a kernel is scheduled while its predecessor drains, runs its
// prologue (barrier set-up, TMEM allocation, the first weight tiles) and then
// waits in griddep_wait for the predecessor's results.  Off by default, so a
// standalone op launch is ordered as usual.
bool& pdl_enabled();
struct PdlScope {
    bool prev;
    explicit PdlScope(bool on) : prev(pdl_enabled()) { pdl_enabled() = on; }
    ~PdlScope() { pdl_enabled() = prev; }
    PdlScope(const PdlScope&) = delete;
    PdlScope& operator=(const PdlScope&) = delete;
};

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (pdl_enabled()) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// C[M,N] = A[M,K] * B[N,K]^T with A, B fp16 row-major (K contiguous).
// Requires K % 64 == 0 and N % 32 == 0; A and B 16-byte aligned rows.
cudaError_t launch_gemm(const __half* A, const __half* B, const GemmArgs& args, int epi, int num_sms,
                        cudaStream_t stream);

struct AttnArgs {
    const void* q;            // [groups*16][L][64]
    const void* k;
    const void* v;
    int groups;               // images * windows-per-image
    int L;                    // tokens per group (576 windowed, 5184 global)
    int windowed;             // output token mapping
    float scale_log2;         // softmax scale * log2(e)
    int bf16;                 // operand type: fp16 (0) or bf16 (1)
    int q8;                   // Q8_0 activation rounding of the output
    void* out;                // [images*5184][1024] (fp16 or bf16), token-major, natural order
    int* status;
};

cudaError_t launch_attention(const AttnArgs& args, cudaStream_t stream);

// Row LayerNorm over 1024 columns (eps 1e-5).  Mode 0: y16 = LN(x); mode 1
// (stem): x = LN_a(x) kept in fp32, then y16 = LN_b(x).
cudaError_t launch_layernorm(const float* x, int rows, const float* g, const float* b, __half* y16, int q8,
                             cudaStream_t stream);
cudaError_t launch_layernorm_stem(float* x, int rows, const float* g0, const float* b0, const float* g1,
                                  const float* b1, __half* y16, int q8, cudaStream_t stream);

// images [B][3][1008][1008] fp32 -> patches [B*5184][640] fp16, column
// ic*196 + kh*14 + kw, zero beyond 588.  round_f16: the pixel values become
// fp16 (true for every weight format: the MMA operands are fp16).
cudaError_t launch_im2col(const float* images, int batch, __half* cols, cudaStream_t stream);
// One thread waits (limit_ns) on an mbarrier nothing arrives at; *gave_up = 1
// and kErrTimeoutProbe in *status when the bounded wait ran out.
cudaError_t launch_wait_timeout_probe(int* status, uint64_t limit_ns, int* gave_up, cudaStream_t stream);

// uint8 RGB [batch][height][width][3] -> normalized [batch][3][1008][1008] fp32
// (the reference's bilinear_resize_rgb, bit-exact).
cudaError_t launch_resize_rgb8(const uint8_t* rgb, int width, int height, int batch, float* out, cudaStream_t stream);

// Weight preparation (once per model).
cudaError_t launch_dequant_q8_0_to_f16(const uint8_t* blocks, int64_t n, __half* out, cudaStream_t stream);
cudaError_t launch_dequant_q8_0_to_f32(const uint8_t* blocks, int64_t n, float* out, cudaStream_t stream);
cudaError_t launch_f16_to_f32(const __half* in, int64_t n, float* out, cudaStream_t stream);
cudaError_t launch_f32_to_f16(const float* in, int64_t n, __half* out, cudaStream_t stream);

// Standalone axial RoPE on [groups*16][L][64] (attention microbench input).
cudaError_t launch_rope_inplace(void* x, int groups, int L, int windowed, int bf16, const float* rope_local,
                                const float* rope_global, cudaStream_t stream);

// Per-device one-time setup (dynamic shared-memory limits); call with the
// device current before the first launch and outside stream capture.
cudaError_t gemm_prepare();
cudaError_t attention_prepare();

// The neck's first operation around the pair GEMM (s3t_neck_first): the
// trunk's NCHW fp32 output [batch][1024][72][72] -> the fp16 A operand
// (levels 0/1: the 2x2 deconv's input order; 2: tokens; 3: 2x2 max-pooled
// tokens), and the GEMM's fp16 [batch*T][rows] -> the level's NCHW fp32 map.
cudaError_t launch_neck_tokens(const float* x, int batch, int level, __half* a, cudaStream_t stream);
cudaError_t launch_neck_out(const __half* y, int batch, int level, int oc, float* out, cudaStream_t stream);
cudaError_t neck_prepare();

// Multi-head attention of the encoder fusion (src/encoder_fusion.cpp:63-88):
// 8 heads of 32 over token-major [len][256] q/k/v, ggml_flash_attn_ext
// semantics with an optional additive per-key mask; `batch` independent
// sequences of the same lengths, back to back.
struct MhaArgs {
    const void* q;            // [batch][q_len][256] fp16 / bf16
    const void* k;            // [batch][kv_len][256]
    const void* v;            // [batch][kv_len][256]
    const float* key_mask;    // [batch][kv_len] additive, -inf = key skipped; may be null;
                              // with `bias`: [batch][8 heads][q_len][kv_len]
    int batch;
    int q_len;
    int kv_len;
    float scale_log2;         // softmax scale * log2(e)
    int bf16;                 // operand type: fp16 (0) or bf16 (1)
    int out_f16;              // output fp16/bf16 (1, operand type) or fp32 (0)
    int bias;                 // key_mask holds one row per (sequence, head, query)
    int splits;               // key-range splits per (query tile, head, sequence); 1 = direct output
    float* ws_o;              // splits > 1: unnormalised O partials [items][128][splits][32]
    float* ws_ml;             // splits > 1: (m, l) of each partial
    void* out;                // [batch][q_len][256]
    int* status;
};
cudaError_t launch_mha32(const MhaArgs& a, cudaStream_t stream);
cudaError_t mha32_prepare();

// Stem weights of a finalized context, for entry points defined outside
// runtime.cu.  Returns false if the context is null or not finalized.
struct StemView {
    int device;
    int num_sms;
    const __half* patch_w;   // [1024][640] fp16, column ic*196 + kh*14 + kw
    const float* pos;        // [577][1024]
    const float* ln_w;
    const float* ln_b;
    int* status;
    cudaStream_t stream;     // the context's own stream
};

// Tensor-map creation through the driver entry point.
bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);
bool make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t d0,
                  uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

}  // namespace s3t

struct s3t_ctx;
namespace s3t {
bool ctx_stem_view(const s3t_ctx* ctx, StemView* out);
// The context's own stream (what a NULL stream argument means), or null.
cudaStream_t ctx_stream(const s3t_ctx* ctx);
// Records the thread-local message returned by s3t_last_error(); returns -1.
int set_last_error(const char* msg);
}  // namespace s3t
