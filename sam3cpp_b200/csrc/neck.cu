// Layout kernels around the neck's first operation (s3t_neck_first): the
// trunk's NCHW output becomes the fp16 A operand of the pair GEMM, and the
// GEMM's token-major fp16 result becomes the level's NCHW fp32 feature map.
// All three are HBM-bound copies that stage through shared memory so both
// their reads and their writes are contiguous runs.
//
// The A operand reproduces what the reference's ggml graph multiplies
// (src/vision_neck.cpp):
// * 1x1 conv (levels 2, 3): ggml_conv_2d's im2col, one row per position
//   t = y * W + x holding the position's channels, rounded to the F16 weights'
//   type; level 3 first takes the 2x2 max (ggml_pool_2d) of each 2x2 block.
// * 2x2 deconv (levels 0, 1): deconv2d_bias (:70-125) with input_ch_first
//   false, whose ggml_permute(x, 2, 0, 1, 3) on x = [W, H, C] gives an
//   [H, C, W] array (source axis i goes to position axis_i), reshaped to
//   [C, W*H]: GEMM row j holds values [1024 j, 1024 j + 1024) of that array,
//   i.e. P[w][c][h] = x[c][h][w] read flat.
#include "kernels.h"

namespace s3t {

namespace {

constexpr int kG = kGrid;              // 72
constexpr int kPlane = kG * kG;        // 5184

// Levels 2: A[b*5184 + t][c] = fp16(x[b][c][t]); 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) neck_tokens_kernel(const float* __restrict__ x, __half* __restrict__ a) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z, t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const float* xb = x + int64_t(b) * kDim * kPlane;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int t = t0 + threadIdx.x;
        tile[i][threadIdx.x] = t < kPlane ? xb[int64_t(c0 + i) * kPlane + t] : 0.f;
    }
    __syncthreads();
    __half* ab = a + int64_t(b) * kPlane * kDim;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int t = t0 + i;
        if (t < kPlane) ab[int64_t(t) * kDim + c0 + threadIdx.x] = __float2half_rn(tile[threadIdx.x][i]);
    }
}

// Level 3: A[b*1296 + t3][c] = fp16(max over the 2x2 block of position t3 = y3*36 + x3).
__global__ void __launch_bounds__(256) neck_pool_tokens_kernel(const float* __restrict__ x, __half* __restrict__ a) {
    constexpr int kP = kG / 2, kPP = kP * kP;   // 36, 1296
    __shared__ float tile[32][33];
    const int b = blockIdx.z, t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const float* xb = x + int64_t(b) * kDim * kPlane;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int t = t0 + threadIdx.x;
        float v = 0.f;
        if (t < kPP) {
            const int y3 = t / kP, x3 = t - y3 * kP;
            const float* p = xb + int64_t(c0 + i) * kPlane + (2 * y3) * kG + 2 * x3;
            v = fmaxf(fmaxf(p[0], p[1]), fmaxf(p[kG], p[kG + 1]));
        }
        tile[i][threadIdx.x] = v;
    }
    __syncthreads();
    __half* ab = a + int64_t(b) * kPP * kDim;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int t = t0 + i;
        if (t < kPP) ab[int64_t(t) * kDim + c0 + threadIdx.x] = __float2half_rn(tile[threadIdx.x][i]);
    }
}

// Levels 0, 1: a flat per image = P[w][c][h] = fp16(x[c][h][w]).  A block
// takes 4 channels: it reads their 4 x 72 x 72 values row by row, then for
// every w writes the 4 x 72 values (c, h) of those channels, which are
// consecutive in P.
constexpr int kDeconvC = 4;
__global__ void __launch_bounds__(256) neck_deconv_tokens_kernel(const float* __restrict__ x, __half* __restrict__ a) {
    extern __shared__ float sx[];            // [kDeconvC][72][73]
    const int b = blockIdx.y, c0 = blockIdx.x * kDeconvC;
    const float* xb = x + (int64_t(b) * kDim + c0) * kPlane;
    for (int i = threadIdx.x; i < kDeconvC * kPlane; i += blockDim.x) {
        const int cc = i / kPlane, r = i - cc * kPlane, h = r / kG, w = r - h * kG;
        sx[(cc * kG + h) * (kG + 1) + w] = xb[i];
    }
    __syncthreads();
    __half* ab = a + int64_t(b) * kDim * kPlane;
    for (int i = threadIdx.x; i < kDeconvC * kPlane; i += blockDim.x) {
        const int w = i / (kDeconvC * kG), r = i - w * (kDeconvC * kG), cc = r / kG, h = r - cc * kG;
        ab[int64_t(w) * kDim * kG + int64_t(c0 + cc) * kG + h] = __float2half_rn(sx[(cc * kG + h) * (kG + 1) + w]);
    }
}

// 1x1 conv result: out[b][o][t] = y[b*T + t][o] (fp16 -> fp32), 32 x 32 tiles.
__global__ void __launch_bounds__(256) neck_conv_out_kernel(const __half* __restrict__ y, int T, int O,
                                                            float* __restrict__ out) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z, t0 = blockIdx.x * 32, o0 = blockIdx.y * 32;
    const __half* yb = y + int64_t(b) * T * O;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int t = t0 + i;
        tile[i][threadIdx.x] = t < T ? __half2float(yb[int64_t(t) * O + o0 + threadIdx.x]) : 0.f;
    }
    __syncthreads();
    float* ob = out + int64_t(b) * O * T;
    for (int i = threadIdx.y; i < 32; i += 8) {
        const int t = t0 + threadIdx.x;
        if (t < T) ob[int64_t(o0 + i) * T + t] = tile[threadIdx.x][i];
    }
}

// 2x2 deconv result, pixel shuffle: out[b][oc][2h+kh][2w+kw] = y[b*5184 + w + 72h][oc + OC*(kw + 2 kh)].
// A block takes one h and 32 output channels: it stages the 72 rows' 4 x 32
// columns, then writes 2 x 32 output rows of 144 floats.
__global__ void __launch_bounds__(256) neck_deconv_out_kernel(const __half* __restrict__ y, int OC,
                                                              float* __restrict__ out) {
    __shared__ __half st[kG][4][32];
    const int b = blockIdx.z, h = blockIdx.x, oc0 = blockIdx.y * 32, R = 4 * OC;
    const __half* yb = y + (int64_t(b) * kPlane + int64_t(h) * kG) * R;
    for (int i = threadIdx.x; i < kG * 4 * 32; i += blockDim.x) {
        const int w = i / 128, q = (i / 32) & 3, o = i & 31;
        st[w][q][o] = yb[int64_t(w) * R + q * OC + oc0 + o];
    }
    __syncthreads();
    constexpr int kOut = 2 * kG;   // 144
    float* ob = out + int64_t(b) * OC * kOut * kOut;
    for (int i = threadIdx.x; i < 32 * 2 * kOut; i += blockDim.x) {
        const int o = i / (2 * kOut), r = i - o * (2 * kOut), kh = r / kOut, wo = r - kh * kOut;
        const int w = wo >> 1, kw = wo & 1;
        ob[(int64_t(oc0 + o) * kOut + 2 * h + kh) * kOut + wo] = __half2float(st[w][kw + 2 * kh][o]);
    }
}

}  // namespace

cudaError_t launch_neck_tokens(const float* x, int batch, int level, __half* a, cudaStream_t stream) {
    if (level == 2) {
        neck_tokens_kernel<<<dim3((kPlane + 31) / 32, kDim / 32, batch), dim3(32, 8), 0, stream>>>(x, a);
    } else if (level == 3) {
        const int pp = (kG / 2) * (kG / 2);
        neck_pool_tokens_kernel<<<dim3((pp + 31) / 32, kDim / 32, batch), dim3(32, 8), 0, stream>>>(x, a);
    } else {
        const size_t smem = size_t(kDeconvC) * kG * (kG + 1) * sizeof(float);
        neck_deconv_tokens_kernel<<<dim3(kDim / kDeconvC, batch), 256, smem, stream>>>(x, a);
    }
    return cudaGetLastError();
}

cudaError_t launch_neck_out(const __half* y, int batch, int level, int oc, float* out, cudaStream_t stream) {
    if (oc % 32) return cudaErrorInvalidValue;
    if (level >= 2) {
        const int T = level == 2 ? kPlane : (kG / 2) * (kG / 2);
        neck_conv_out_kernel<<<dim3((T + 31) / 32, oc / 32, batch), dim3(32, 8), 0, stream>>>(y, T, oc, out);
    } else {
        neck_deconv_out_kernel<<<dim3(kG, oc / 32, batch), 256, 0, stream>>>(y, oc, out);
    }
    return cudaGetLastError();
}

cudaError_t neck_prepare() {
    return cudaFuncSetAttribute(neck_deconv_tokens_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(size_t(kDeconvC) * kG * (kG + 1) * sizeof(float)));
}

}  // namespace s3t
