// Allocation-free stem: patch embedding + tiled position embedding + ln_pre
// for callers that cannot allocate device memory.
//
// Some callers of this library cannot call cudaMalloc: a plugin hosted by an
// application that owns every device allocation and forbids its plugins to
// allocate, or a fixed-budget loop whose memory was reserved up front.  For
// them, s3t_stem_noalloc() computes the same stem as
// s3t_trunk_run_layers(ctx, ..., n_layers = 0, ...), with the one scratch
// buffer it needs (the fp16 patch matrix fed to the patch-embed GEMM) held in
// the file-scope device array below instead of the context's workspace.
//
// The array holds one image's patch matrix (5184 x 640 fp16 = 6,635,520
// bytes).  Every GPU that loads this library keeps it until the process
// exits.  All calls on a GPU share that GPU's copy, and it keeps the last
// call's contents; each call writes every element it later reads, so
// nothing has to be cleared first, but two calls whose work overlaps on the
// same GPU (for example, issued on two different streams) race on it.
#include "s3t.h"
#include "kernels.h"
#include "ptx.cuh"

#include <mutex>
#include <string>

using namespace s3t;

namespace {

constexpr int kStaticImages = 1;
constexpr size_t kStaticPatchElems = size_t(kStaticImages) * kTokens * kPatchKPad;

// The scratch.  Host code must not use this name as a device address: it is
// a host-side stand-in.  The device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) __half g_static_patches[kStaticPatchElems];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
__half* g_patches_dev[kMaxDevices] = {};

// Per-device set-up: the device address of g_static_patches, looked up once
// with that device current (the first call on each device does it).
int static_patches(int device, __half** out) {
    if (device < 0 || device >= kMaxDevices) return set_last_error("device index out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_patches_dev[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_patches);
        if (e != cudaSuccess)
            return set_last_error((std::string("cudaGetSymbolAddress(g_static_patches): ") + cudaGetErrorString(e)).c_str());
        g_patches_dev[device] = static_cast<__half*>(p);
    }
    *out = g_patches_dev[device];
    return 0;
}

// ln_pre in place on fp32 token rows (layer_norm, src/vision_trunk.cpp:64-74):
// one warp per 1024-wide row, mean and centred variance reduced over the warp.
__global__ void __launch_bounds__(256) ln_inplace_kernel(float* __restrict__ x, int rows, const float* __restrict__ g,
                                                         const float* __restrict__ b) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float* xr = x + int64_t(row) * kDim;
    float v[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float4 t = *reinterpret_cast<const float4*>(xr + 128 * k + 4 * lane);
        v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
    }
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) s += v[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.0f / kDim);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        v[i] -= mean;
        q += v[i] * v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = 1.0f / sqrtf(q * (1.0f / kDim) + 1e-5f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int c = 128 * k + 4 * lane;
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g + c));
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b + c));
        *reinterpret_cast<float4*>(xr + c) =
            make_float4(v[4 * k] * rstd * gg.x + bb.x, v[4 * k + 1] * rstd * gg.y + bb.y,
                        v[4 * k + 2] * rstd * gg.z + bb.z, v[4 * k + 3] * rstd * gg.w + bb.w);
    }
}

// 0 if p is device (or managed) memory of `device`; otherwise the message.
int check_device_pointer(const void* p, int device, const char* what) {
    cudaPointerAttributes a{};
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_last_error((std::string(what) + " is not a CUDA pointer").c_str());
    }
    if ((a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) || a.device != device)
        return set_last_error((std::string(what) + " is not device memory of the context's GPU " +
                               std::to_string(device)).c_str());
    return 0;
}

}  // namespace

extern "C" int s3t_stem_noalloc(s3t_ctx* ctx, const float* images_dev, int batch, float* out_tokens_dev, void* stream) {
    try {
        StemView w;
        if (!ctx_stem_view(ctx, &w)) return set_last_error("ctx is null or its weights are not finalized");
        if (!images_dev || !out_tokens_dev) return set_last_error("images or out is null");
        // The patch gather reads the image and the GEMM epilogue and ln_pre
        // write the tokens with 16-byte vector accesses.
        if ((reinterpret_cast<uintptr_t>(images_dev) | reinterpret_cast<uintptr_t>(out_tokens_dev)) & 15)
            return set_last_error("s3t_stem_noalloc: images and out must be 16-byte aligned");
        if (batch < 1 || batch > kStaticImages)
            return set_last_error(("s3t_stem_noalloc: batch " + std::to_string(batch) + " is outside 1.." +
                                   std::to_string(kStaticImages) + " (its static scratch holds " +
                                   std::to_string(kStaticImages) + " image)").c_str());
        cudaError_t e = cudaSetDevice(w.device);
        if (e != cudaSuccess) return set_last_error(cudaGetErrorString(e));
        if (check_device_pointer(images_dev, w.device, "images") ||
            check_device_pointer(out_tokens_dev, w.device, "out"))
            return -1;
        __half* patches = nullptr;
        if (static_patches(w.device, &patches)) return -1;
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : w.stream;
        const int M = batch * kTokens;

        if ((e = launch_im2col(images_dev, batch, patches, st)) != cudaSuccess)
            return set_last_error((std::string("im2col: ") + cudaGetErrorString(e)).c_str());
        GemmArgs g{};
        g.M = M;
        g.N = kDim;
        g.K = kPatchKPad;
        g.resid = out_tokens_dev;
        g.pos = w.pos;
        g.status = w.status;
        if ((e = launch_gemm(patches, w.patch_w, g, kEpiPatch, w.num_sms, st)) != cudaSuccess)
            return set_last_error((std::string("patch GEMM: ") + cudaGetErrorString(e)).c_str());
        ln_inplace_kernel<<<(M + 7) / 8, 256, 0, st>>>(out_tokens_dev, M, w.ln_w, w.ln_b);
        if ((e = cudaGetLastError()) != cudaSuccess)
            return set_last_error((std::string("ln_pre: ") + cudaGetErrorString(e)).c_str());
        return 0;
    } catch (...) {
        return set_last_error("s3t_stem_noalloc: internal error");
    }
}
