// Drop-in replacement for the reference's src/vision_trunk.cpp: the same
// sam3::VisionTrunk class (include/sam3/vision_trunk.h), computed by the B200
// kernels behind include/s3t.h.
//
// Build it in place of src/vision_trunk.cpp and link libs3t.so.  Weights are
// taken from the caller's GgufModel by name (GgufModel::find_weight, alias
// aware, src/gguf_model.cpp:190-204) and uploaded once per model: pipeline.cpp
// constructs a VisionTrunk per request (src/pipeline.cpp:159), so the device
// context (0.9 GB of fp16 weights plus the workspace) is cached.  The cache
// key is the GgufModel's address together with a fingerprint of the loaded
// weights (the types, shapes and data addresses of the trunk's tensors and a
// 64-bit hash of sampled bytes of several of them): a GgufModel that was
// reloaded (GgufModel::load clears and refills it) or a new model that lands
// at a freed model's address gets a fresh context, and the stale one is
// destroyed.  At most S3T_MAX_CONTEXTS contexts (default 2) are kept; the
// least recently used one is destroyed beyond that.  The GPU is S3T_DEVICE
// (default 0).  Errors are std::runtime_error with the reference's messages
// for the shape checks (src/vision_trunk.cpp:301-306).
#include "sam3/vision_trunk.h"

#include "s3t.h"

#include <algorithm>
#include <cstdint>
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

// FNV-1a over `n` bytes, continuing from h.
uint64_t fnv1a(uint64_t h, const void * p, size_t n) {
    const auto * b = static_cast<const uint8_t *>(p);
    for (size_t i = 0; i < n; ++i) {
        h = (h ^ b[i]) * 0x100000001b3ull;
    }
    return h;
}

// Identity of the weights a GgufModel holds right now: type, shape and data
// address of the stem tensors and of every block's qkv/fc2 weight, plus up
// to 4 KB from the start and the end of the pos embedding, the patch
// embedding, the first block's qkv weight and the last block's fc2 weight.
uint64_t weights_fingerprint(const GgufModel & model) {
    uint64_t h = 0xcbf29ce484222325ull;
    std::vector<std::string> names = {"patch_embed.proj.weight", "pos_embed", "ln_pre.weight", "ln_pre.bias"};
    int layers = 0;
    while (layers < kMaxLayers && model.find_weight(trunk_name("blocks." + std::to_string(layers) + ".attn.qkv.weight"))) {
        names.push_back("blocks." + std::to_string(layers) + ".attn.qkv.weight");
        names.push_back("blocks." + std::to_string(layers) + ".mlp.fc2.weight");
        ++layers;
    }
    std::vector<uint8_t> buf(4096);
    for (size_t i = 0; i < names.size(); ++i) {
        ggml_tensor * t = model.find_weight(trunk_name(names[i]));
        if (t == nullptr) {
            continue;
        }
        const uint64_t meta[6] = {uint64_t(t->type), uint64_t(t->ne[0]), uint64_t(t->ne[1]), uint64_t(t->ne[2]),
                                  uint64_t(t->ne[3]), uint64_t(reinterpret_cast<uintptr_t>(t->data))};
        h = fnv1a(h, meta, sizeof meta);
        const bool sampled = i < 2 || names[i] == "blocks.0.attn.qkv.weight" || i + 1 == names.size();
        if (!sampled) {
            continue;
        }
        const size_t nbytes = ggml_nbytes(t), n = std::min(nbytes, buf.size());
        ggml_backend_tensor_get(t, buf.data(), 0, n);
        h = fnv1a(h, buf.data(), n);
        ggml_backend_tensor_get(t, buf.data(), nbytes - n, n);
        h = fnv1a(h, buf.data(), n);
    }
    return h;
}

s3t_ctx * create_context(const GgufModel & model) {
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
    return ctx;
}

struct CachedContext {
    const GgufModel * model;
    uint64_t fingerprint;
    s3t_ctx * ctx;
    uint64_t last_use;
};

// Returns the context of `model`, creating it on first use.  Callers hold
// the returned context only while the cache mutex is held by run().
s3t_ctx * context_for(const GgufModel & model, std::unique_lock<std::mutex> & held) {
    static std::mutex mu;
    static std::vector<CachedContext> cache;
    static uint64_t clock = 0;
    held = std::unique_lock<std::mutex>(mu);
    const uint64_t fp = weights_fingerprint(model);
    for (size_t i = 0; i < cache.size(); ++i) {
        if (cache[i].model != &model) {
            continue;
        }
        if (cache[i].fingerprint == fp) {
            cache[i].last_use = ++clock;
            return cache[i].ctx;
        }
        s3t_destroy(cache[i].ctx);          // the model was reloaded with other weights
        cache.erase(cache.begin() + long(i));
        break;
    }
    const char * env = std::getenv("S3T_MAX_CONTEXTS");
    const size_t max_contexts = size_t(std::max(1, env ? std::atoi(env) : 2));
    while (cache.size() >= max_contexts) {
        auto lru = std::min_element(cache.begin(), cache.end(), [](const CachedContext & a, const CachedContext & b) {
            return a.last_use < b.last_use;
        });
        s3t_destroy(lru->ctx);
        cache.erase(lru);
    }
    s3t_ctx * ctx = create_context(model);
    cache.push_back({&model, fp, ctx, ++clock});
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
    std::unique_lock<std::mutex> held;
    s3t_ctx * ctx = context_for(model_, held);
    VisionTrunkOutput out;
    out.shape_nchw = {1, 1024, 72, 72};
    out.trunk_nchw.resize(1024ull * 72 * 72);
    if (s3t_trunk_run(ctx, image_nchw.data(), 1, out.trunk_nchw.data(), 0, nullptr) != 0) {
        throw std::runtime_error(std::string("vision trunk compute failed: ") + s3t_last_error());
    }
    return out;
}

}  // namespace sam3
