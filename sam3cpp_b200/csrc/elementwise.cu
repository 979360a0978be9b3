// HBM-bound kernels of the trunk: LayerNorm (fp32 residual in, fp16 GEMM
// operand out, with the Q8_0 activation rounding fused), the patchify gather
// feeding the patch-embed GEMM, weight dequantization, a standalone RoPE (for
// the attention microbenchmark) and a token-major -> NCHW copy.
#include "kernels.h"
#include "ptx.cuh"

namespace s3t {

namespace {

// One warp per 1024-wide row.  Lane l owns float4 chunks at columns
// 128*k + 4*l (k = 0..7), so every load/store instruction of the warp covers
// 512 contiguous bytes.  Q8_0 blocks (32 columns) are the 8-lane groups of
// one k: amax is reduced over xor-shuffles 1, 2, 4.
__device__ __forceinline__ void ln_row(const float (&x)[32], const float* g, const float* b, int lane, float (&y)[32]) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) s += x[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.0f / kDim);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float d = x[i] - mean;
        y[i] = d;
        q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = 1.0f / sqrtf(q * (1.0f / kDim) + 1e-5f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const int c = 128 * k + 4 * lane;
        const float4 gg = __ldg(reinterpret_cast<const float4*>(g + c));
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b + c));
        y[4 * k + 0] = y[4 * k + 0] * rstd * gg.x + bb.x;
        y[4 * k + 1] = y[4 * k + 1] * rstd * gg.y + bb.y;
        y[4 * k + 2] = y[4 * k + 2] * rstd * gg.z + bb.z;
        y[4 * k + 3] = y[4 * k + 3] * rstd * gg.w + bb.w;
    }
}

__device__ __forceinline__ void store_act_row(__half* out, const float (&y)[32], int lane, int q8) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float v0 = y[4 * k], v1 = y[4 * k + 1], v2 = y[4 * k + 2], v3 = y[4 * k + 3];
        if (q8) {
            float amax = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
            const float d = __half2float(__float2half_rn(__fdiv_rn(amax, 127.f)));
            const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
            v0 = rintf(__fmul_rn(v0, id)) * d;
            v1 = rintf(__fmul_rn(v1, id)) * d;
            v2 = rintf(__fmul_rn(v2, id)) * d;
            v3 = rintf(__fmul_rn(v3, id)) * d;
        }
        uint2 u = make_uint2(pack_half2(v0, v1), pack_half2(v2, v3));
        *reinterpret_cast<uint2*>(out + 128 * k + 4 * lane) = u;
    }
}

__device__ __forceinline__ void load_row(const float* xr, int lane, float (&x)[32]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float4 t = *reinterpret_cast<const float4*>(xr + 128 * k + 4 * lane);
        x[4 * k] = t.x; x[4 * k + 1] = t.y; x[4 * k + 2] = t.z; x[4 * k + 3] = t.w;
    }
}

// layer_norm of src/vision_trunk.cpp:64-74 (ggml_norm, eps 1e-5, then *gamma
// +beta), producing the fp16 operand of the next GEMM.
__global__ void __launch_bounds__(256) layernorm_kernel(const float* __restrict__ x, int rows, const float* g,
                                                        const float* b, __half* __restrict__ y, int q8) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float v[32], o[32];
    load_row(x + int64_t(row) * kDim, lane, v);
    ln_row(v, g, b, lane, o);
    store_act_row(y + int64_t(row) * kDim, o, lane, q8);
}

// Stem: x = ln_pre(x) stays the fp32 residual (src/vision_trunk.cpp:370-376),
// then blocks.0.norm1 of it becomes the first QKV operand.
__global__ void __launch_bounds__(256) layernorm_stem_kernel(float* __restrict__ x, int rows, const float* g0,
                                                             const float* b0, const float* g1, const float* b1,
                                                             __half* __restrict__ y, int q8) {
    griddep_launch_dependents();
    griddep_wait();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float v[32], o[32];
    float* xr = x + int64_t(row) * kDim;
    load_row(xr, lane, v);
    ln_row(v, g0, b0, lane, o);
#pragma unroll
    for (int k = 0; k < 8; ++k)
        *reinterpret_cast<float4*>(xr + 128 * k + 4 * lane) = make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
    ln_row(o, g1, b1, lane, v);
    store_act_row(y + int64_t(row) * kDim, v, lane, q8);
}

// im2col of ggml_conv_2d (ggml/src/ggml.c:4551, 14x14 stride 14, no padding)
// for the patch-embed GEMM: row = image*5184 + (py*72 + px), column
// ic*196 + kh*14 + kw (zero for the 52 pad columns up to 640).  One thread
// writes 8 consecutive columns (16 bytes).
__global__ void im2col_kernel(const float* __restrict__ img, int batch, __half* __restrict__ cols) {
    griddep_launch_dependents();   // the patch GEMM's prologue overlaps this kernel
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = int64_t(batch) * kTokens * (kPatchKPad / 8);
    if (idx >= total) return;
    const int k8 = int(idx % (kPatchKPad / 8));
    const int64_t row = idx / (kPatchKPad / 8);
    const int n = int(row / kTokens), t = int(row % kTokens);
    const int py = t / kGrid, px = t % kGrid;
    const float* base = img + int64_t(n) * 3 * kImage * kImage;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int k = k8 * 8 + e;
        if (k < kPatchK) {
            const int ic = k / 196, rem = k % 196, kh = rem / 14, kw = rem % 14;
            v[e] = __ldg(base + (int64_t(ic) * kImage + py * kPatch + kh) * kImage + px * kPatch + kw);
        } else {
            v[e] = 0.f;
        }
    }
    *reinterpret_cast<uint4*>(cols + row * kPatchKPad + k8 * 8) =
        make_uint4(pack_half2(v[0], v[1]), pack_half2(v[2], v[3]), pack_half2(v[4], v[5]), pack_half2(v[6], v[7]));
}

// dequantize_row_q8_0 (ggml/src/ggml-quants.c:436-450): y = qs[j] * fp32(d).
__global__ void dequant_q8_0_f32_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks, float* __restrict__ y) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nblocks * 32) return;
    const uint8_t* b = blocks + (i >> 5) * 34;
    const float d = __half2float(__ushort_as_half(uint16_t(b[0]) | (uint16_t(b[1]) << 8)));
    y[i] = float(int8_t(b[2 + (i & 31)])) * d;
}

// The same value rounded to the fp16 GEMM operand.
__global__ void dequant_q8_0_f16_kernel(const uint8_t* __restrict__ blocks, int64_t nblocks, __half* __restrict__ y) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nblocks * 32) return;
    const uint8_t* b = blocks + (i >> 5) * 34;
    const float d = __half2float(__ushort_as_half(uint16_t(b[0]) | (uint16_t(b[1]) << 8)));
    y[i] = __float2half_rn(float(int8_t(b[2 + (i & 31)])) * d);
}

__global__ void f16_to_f32_kernel(const __half* __restrict__ in, int64_t n, float* __restrict__ out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __half2float(in[i]);
}

__global__ void f32_to_f16_kernel(const float* __restrict__ in, int64_t n, __half* __restrict__ out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(in[i]);
}

// Axial RoPE in place on [groups*16][L][64]; one thread per (row, 8-dim
// slice): one 16-byte load and store, cos/sin as float4 loads.  Row counts
// fit in 32 bits (<= 64 images x 9 x 16 x 576).
template <typename T>
__global__ void rope_kernel(T* x, int groups, int L, int windowed, const float* rl, const float* rg) {
    const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t total = uint32_t(groups) * kHeads * L * 8;
    if (idx >= total) return;
    const uint32_t slice = idx & 7;          // dims 8*slice .. 8*slice+7
    const uint32_t r = idx >> 3;
    const uint32_t i = r % uint32_t(L);
    const int half = slice >> 2;             // dims 0..31 -> x position, 32..63 -> y position
    const int grid = windowed ? kWindow : kGrid;
    const int pos = half ? int(i) / grid : int(i) % grid;
    const float* cs = (windowed ? rl : rg) + pos * 32 + (slice & 3) * 4;   // pair index j = 4*(slice&3) + u
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(cs + 16));
    const float c[4] = {c4.x, c4.y, c4.z, c4.w}, s[4] = {s4.x, s4.y, s4.z, s4.w};
    uint4* p = reinterpret_cast<uint4*>(x + size_t(r) * kHeadDim + slice * 8);
    uint4 u = *p;
    T* v = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float x0 = float(v[2 * j]), x1 = float(v[2 * j + 1]);
        v[2 * j] = T(x0 * c[j] - x1 * s[j]);
        v[2 * j + 1] = T(x0 * s[j] + x1 * c[j]);
    }
    *p = u;
}

}  // namespace

cudaError_t launch_layernorm(const float* x, int rows, const float* g, const float* b, __half* y16, int q8,
                             cudaStream_t stream) {
    return launch_kernel(layernorm_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, x, rows, g, b, y16, q8);
}

cudaError_t launch_layernorm_stem(float* x, int rows, const float* g0, const float* b0, const float* g1,
                                  const float* b1, __half* y16, int q8, cudaStream_t stream) {
    return launch_kernel(layernorm_stem_kernel, dim3((rows + 7) / 8), dim3(256), 0, stream, x, rows, g0, b0, g1, b1,
                         y16, q8);
}

cudaError_t launch_im2col(const float* images, int batch, __half* cols, cudaStream_t stream) {
    const int64_t total = int64_t(batch) * kTokens * (kPatchKPad / 8);
    im2col_kernel<<<unsigned((total + 255) / 256), 256, 0, stream>>>(images, batch, cols);
    return cudaGetLastError();
}

cudaError_t launch_dequant_q8_0_to_f16(const uint8_t* blocks, int64_t n, __half* out, cudaStream_t stream) {
    dequant_q8_0_f16_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(blocks, n / 32, out);
    return cudaGetLastError();
}

cudaError_t launch_dequant_q8_0_to_f32(const uint8_t* blocks, int64_t n, float* out, cudaStream_t stream) {
    dequant_q8_0_f32_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(blocks, n / 32, out);
    return cudaGetLastError();
}

cudaError_t launch_f16_to_f32(const __half* in, int64_t n, float* out, cudaStream_t stream) {
    f16_to_f32_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(in, n, out);
    return cudaGetLastError();
}

cudaError_t launch_f32_to_f16(const float* in, int64_t n, __half* out, cudaStream_t stream) {
    f32_to_f16_kernel<<<unsigned((n + 255) / 256), 256, 0, stream>>>(in, n, out);
    return cudaGetLastError();
}

cudaError_t launch_rope_inplace(void* x, int groups, int L, int windowed, int bf16, const float* rl, const float* rg,
                                cudaStream_t stream) {
    const int64_t total = int64_t(groups) * kHeads * L * 8;
    if (total >= (int64_t(1) << 32)) return cudaErrorInvalidValue;
    const unsigned blocks = unsigned((total + 255) / 256);
    if (bf16)
        rope_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(static_cast<__nv_bfloat16*>(x), groups, L, windowed, rl, rg);
    else
        rope_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<__half*>(x), groups, L, windowed, rl, rg);
    return cudaGetLastError();
}

}  // namespace s3t
