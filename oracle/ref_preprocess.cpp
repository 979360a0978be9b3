// Test infrastructure only: exposes the reference's own image preprocessing,
// bilinear_resize_rgb of tools/sam3_vision_trunk.cpp:33-66 (the arithmetic of
// src/pipeline.cpp:45-83 load_image_rgb after stbi_load), to the parity tests.
//
// The function lives in an anonymous namespace of the tool's source, so this
// file compiles that source where it lies (the include path points into the
// reference tree; nothing is copied) with the tool's main renamed, and adds a
// C entry point.  It is compiled with the reference's default flags for its
// tools (-O3, no -march), like the reference's own CMake build of
// sam3-vision-trunk: scalar SSE arithmetic without fused multiply-adds.
#define main sam3_vision_trunk_tool_main
#include "tools/sam3_vision_trunk.cpp"
#undef main

#include <cstring>

extern "C" int ref_bilinear_resize_rgb(const uint8_t* src, int width, int height, float* out) {
    if (!src || !out || width <= 0 || height <= 0) return -1;
    const std::vector<float> v = bilinear_resize_rgb(src, width, height);
    std::memcpy(out, v.data(), v.size() * sizeof(float));
    return 0;
}
