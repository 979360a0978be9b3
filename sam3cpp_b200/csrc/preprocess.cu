// Image preprocessing on the device: decoded uint8 RGB (height x width x 3,
// row-major HWC, the layout stbi_load returns) -> normalized
// [3][1008][1008] fp32, the reference's bilinear_resize_rgb
// (tools/sam3_vision_trunk.cpp:33-66; the same arithmetic as
// src/pipeline.cpp:45-83 load_image_rgb):
//   s = (d + 0.5) * (src / 1008) - 0.5,  i0 = clamp(floor(s)), i1 = clamp(i0 + 1),
//   w = s - i0 (from the clamped i0, so the top/left edge extrapolates),
//   p = u8 / 255, two horizontal lerps, one vertical lerp, (v - 0.5) / 0.5.
// Every product, sum and quotient is a separately rounded IEEE operation
// (__fmul_rn / __fadd_rn / __fsub_rn / __fdiv_rn are never contracted into
// FMAs), as in the reference's scalar x86-64 build, so the result is bit-exact.
//
// One thread per output pixel (all three channels); a block covers 256
// consecutive pixels of one output row, so each channel plane is written with
// coalesced 4-byte stores.  HBM-bound: 12.2 MB written per image, the source
// (a few MB of uint8) is read through L1/L2.
#include "kernels.h"

namespace s3t {

namespace {

__global__ void resize_rgb8_kernel(const uint8_t* __restrict__ src, int w, int h, float* __restrict__ out) {
    __shared__ float unit[256];   // u8 / 255, correctly rounded
    for (int i = threadIdx.x; i < 256; i += blockDim.x) unit[i] = __fdiv_rn(float(i), 255.0f);
    __syncthreads();
    const int dx = blockIdx.x * blockDim.x + threadIdx.x;
    const int dy = blockIdx.y;
    const int n = blockIdx.z;
    if (dx >= kImage) return;

    const float xs = __fdiv_rn(float(w), float(kImage)), ys = __fdiv_rn(float(h), float(kImage));
    const float sy = __fsub_rn(__fmul_rn(__fadd_rn(float(dy), 0.5f), ys), 0.5f);
    const int y0 = min(max(int(floorf(sy)), 0), h - 1);
    const int y1 = min(y0 + 1, h - 1);
    const float wy = __fsub_rn(sy, float(y0));
    const float sx = __fsub_rn(__fmul_rn(__fadd_rn(float(dx), 0.5f), xs), 0.5f);
    const int x0 = min(max(int(floorf(sx)), 0), w - 1);
    const int x1 = min(x0 + 1, w - 1);
    const float wx = __fsub_rn(sx, float(x0));

    const uint8_t* img = src + int64_t(n) * h * w * 3;
    const uint8_t* r00 = img + (int64_t(y0) * w + x0) * 3;
    const uint8_t* r01 = img + (int64_t(y0) * w + x1) * 3;
    const uint8_t* r10 = img + (int64_t(y1) * w + x0) * 3;
    const uint8_t* r11 = img + (int64_t(y1) * w + x1) * 3;
    float* o = out + (int64_t(n) * 3 * kImage + dy) * kImage + dx;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        const float p00 = unit[__ldg(r00 + c)], p01 = unit[__ldg(r01 + c)];
        const float p10 = unit[__ldg(r10 + c)], p11 = unit[__ldg(r11 + c)];
        const float top = __fadd_rn(p00, __fmul_rn(__fsub_rn(p01, p00), wx));
        const float bot = __fadd_rn(p10, __fmul_rn(__fsub_rn(p11, p10), wx));
        const float v = __fadd_rn(top, __fmul_rn(__fsub_rn(bot, top), wy));
        o[int64_t(c) * kImage * kImage] = __fdiv_rn(__fsub_rn(v, 0.5f), 0.5f);
    }
}

}  // namespace

cudaError_t launch_resize_rgb8(const uint8_t* rgb, int width, int height, int batch, float* out, cudaStream_t stream) {
    if (!rgb || !out || width <= 0 || height <= 0 || width > kMaxSourceSide || height > kMaxSourceSide || batch <= 0 ||
        batch > 65535)
        return cudaErrorInvalidValue;
    const dim3 grid((kImage + 255) / 256, kImage, batch);
    resize_rgb8_kernel<<<grid, 256, 0, stream>>>(rgb, width, height, out);
    return cudaGetLastError();
}

}  // namespace s3t
