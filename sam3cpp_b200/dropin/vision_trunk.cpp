// Drop-in replacement for the reference's src/vision_trunk.cpp: the same
// sam3::VisionTrunk class (include/sam3/vision_trunk.h), computed by the B200
// kernels behind include/s3t.h.
//
// Build it in place of src/vision_trunk.cpp and link libs3t.so.  Weights are
// taken from the caller's GgufModel by name (GgufModel::find_weight, alias
// aware, src/gguf_model.cpp:190-204) and uploaded once per model: pipeline.cpp
// constructs a VisionTrunk per request (src/pipeline.cpp:159), so the device
// context is cached per GgufModel and lives until the process exits.  The GPU
// is S3T_DEVICE (default 0).  Errors are std::runtime_error with the
// reference's messages for the shape checks (src/vision_trunk.cpp:301-306).
#include "sam3/vision_trunk.h"

#include "s3t.h"

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace sam3 {

namespace {

constexpr int64_t kImageSize = 1008;
constexpr int kMaxLayers = 32;

std::string trunk_name(const std::string & suffix) {
    return "backbone.vision_backbone.trunk." + suffix;
}

void upload(s3t_ctx * ctx, const GgufModel & model, const std::string & name) {
    ggml_tensor * t = model.find_weight(name);
    if (t == nullptr) {
        throw std::runtime_error("missing tensor: " + name);
    }
    const size_t nbytes = ggml_nbytes(t);
    std::vector<uint8_t> bytes(nbytes);
    ggml_backend_tensor_get(t, bytes.data(), 0, nbytes);
    const int64_t ne[4] = {t->ne[0], t->ne[1], t->ne[2], t->ne[3]};
    if (s3t_set_weight(ctx, name.c_str(), static_cast<int>(t->type), ne, bytes.data(), nbytes) != 0) {
        throw std::runtime_error(s3t_last_error());
    }
}

s3t_ctx * context_for(const GgufModel & model) {
    static std::mutex mu;
    static std::unordered_map<const GgufModel *, s3t_ctx *> contexts;
    std::lock_guard<std::mutex> lock(mu);
    auto it = contexts.find(&model);
    if (it != contexts.end()) {
        return it->second;
    }
    const char * dev = std::getenv("S3T_DEVICE");
    s3t_ctx * ctx = s3t_create(dev ? std::atoi(dev) : 0);
    if (ctx == nullptr) {
        throw std::runtime_error(std::string("s3t_create failed: ") + s3t_last_error());
    }
    try {
        for (const char * s : {"patch_embed.proj.weight", "pos_embed", "ln_pre.weight", "ln_pre.bias"}) {
            upload(ctx, model, trunk_name(s));
        }
        for (int layer = 0; layer < kMaxLayers; ++layer) {
            const std::string b = "blocks." + std::to_string(layer) + ".";
            if (model.find_weight(trunk_name(b + "attn.qkv.weight")) == nullptr) {
                break;
            }
            for (const char * s : {"norm1.weight", "norm1.bias", "attn.qkv.weight", "attn.qkv.bias",
                                   "attn.proj.weight", "attn.proj.bias", "norm2.weight", "norm2.bias",
                                   "mlp.fc1.weight", "mlp.fc1.bias", "mlp.fc2.weight", "mlp.fc2.bias"}) {
                upload(ctx, model, trunk_name(b + s));
            }
        }
        if (s3t_finalize_weights(ctx) != 0) {
            throw std::runtime_error(s3t_last_error());
        }
    } catch (...) {
        s3t_destroy(ctx);
        throw;
    }
    contexts.emplace(&model, ctx);
    return ctx;
}

}  // namespace

VisionTrunk::VisionTrunk(const GgufModel & model) : model_(model) {}

VisionTrunkOutput VisionTrunk::run(
    const std::vector<float> & image_nchw,
    const std::vector<int64_t> & shape_nchw
) const {
    if (shape_nchw != std::vector<int64_t>({1, 3, kImageSize, kImageSize})) {
        throw std::runtime_error("vision trunk expects NCHW image shape [1, 3, 1008, 1008]");
    }
    if (static_cast<int64_t>(image_nchw.size()) != 1LL * 3 * kImageSize * kImageSize) {
        throw std::runtime_error("vision trunk input payload size mismatch");
    }
    s3t_ctx * ctx = context_for(model_);
    VisionTrunkOutput out;
    out.shape_nchw = {1, 1024, 72, 72};
    out.trunk_nchw.resize(1024ull * 72 * 72);
    if (s3t_trunk_run(ctx, image_nchw.data(), 1, out.trunk_nchw.data(), 0, nullptr) != 0) {
        throw std::runtime_error(std::string("vision trunk compute failed: ") + s3t_last_error());
    }
    return out;
}

}  // namespace sam3
