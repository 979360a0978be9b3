// Host runtime of the trunk behind the C ABI in include/s3t.h.
//
// Replaces, for the vision trunk, what the reference does per call in
// VisionTrunk::run (src/vision_trunk.cpp:297-488): instead of building a
// ~262k-node ggml graph, creating a scheduler and allocating every call, the
// context holds the converted weights and a workspace sized for the largest
// batch seen, and replays a captured CUDA graph of the fixed launch sequence
// (im2col, patch GEMM, stem LayerNorms, then per block: QKV GEMM + RoPE,
// attention, proj GEMM + residual, LayerNorm, fc1 GEMM + GELU, fc2 GEMM +
// residual + next LayerNorm).
#include "s3t.h"
#include "kernels.h"

#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <unordered_map>
#include <vector>

using namespace s3t;

bool& s3t::pdl_enabled() {
    static thread_local bool on = false;
    return on;
}

namespace {

thread_local std::string g_last_error;

int fail(const std::string& msg) {
    g_last_error = msg;
    return -1;
}

#define S3T_CUDA(call)                                                                    \
    do {                                                                                  \
        cudaError_t _e = (call);                                                          \
        if (_e != cudaSuccess) return fail(std::string(#call) + ": " + cudaGetErrorString(_e)); \
    } while (0)

const char* kPrefix = "backbone.vision_backbone.trunk";
const char* kNeckPrefix = "backbone.vision_backbone.convs.";   // the neck (src/vision_neck.cpp)

bool is_global_attention_block(int layer) {  // src/vision_trunk.cpp:46-48
    return layer == 7 || layer == 15 || layer == 23 || layer == 31;
}

int64_t type_nbytes(int type, int64_t n) {
    switch (type) {
        case S3T_TYPE_F32: return n * 4;
        case S3T_TYPE_F16: return n * 2;
        case S3T_TYPE_Q8_0: return (n % 32) ? -1 : n / 32 * 34;
    }
    return -1;
}

// RoPE cos/sin tables exactly as ggml's CPU rope builds them for n_dims = 32
// (ggml-cpu/ops.cpp: theta starts at the position, is multiplied by
// powf(10000, -2/32) per pair in f32; cos/sin of freq_scale*theta), laid out
// [pos][cos 0..15 | sin 0..15].
std::vector<float> rope_table(float freq_scale, int npos) {
    std::vector<float> t(size_t(npos) * 32);
    const float theta_scale = powf(10000.0f, -2.0f / 32.0f);
    for (int p = 0; p < npos; ++p) {
        float theta = float(p);
        for (int j = 0; j < 16; ++j) {
            const float th = freq_scale * theta;
            t[p * 32 + j] = cosf(th);
            t[p * 32 + 16 + j] = sinf(th);
            theta *= theta_scale;
        }
    }
    return t;
}

// Per-device state shared by contexts and the op-level entry points.
struct DeviceState {
    bool ready = false;
    int num_sms = 0;
    float* rope_local = nullptr;
    float* rope_global = nullptr;
    float* rope_local_t = nullptr;    // [cos|sin][16][pos]: one frequency of consecutive positions is contiguous
    float* rope_global_t = nullptr;
    int* status = nullptr;
};

std::mutex g_dev_mu;
std::map<int, DeviceState> g_dev;

int device_state(int device, DeviceState** out) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceState& d = g_dev[device];
    if (!d.ready) {
        S3T_CUDA(cudaSetDevice(device));
        cudaDeviceProp prop;
        S3T_CUDA(cudaGetDeviceProperties(&prop, device));
        if (prop.major != 10) return fail("s3t requires an sm_100 (B200-class) GPU; device " + std::to_string(device) +
                                          " is sm_" + std::to_string(prop.major * 10 + prop.minor));
        d.num_sms = prop.multiProcessorCount;
        S3T_CUDA(gemm_prepare());
        S3T_CUDA(attention_prepare());
        S3T_CUDA(mha32_prepare());
        S3T_CUDA(neck_prepare());
        const std::vector<float> rl = rope_table(1.0f, kWindow);
        const std::vector<float> rg = rope_table(float(kWindow) / float(kGrid), kGrid);
        S3T_CUDA(cudaMalloc(&d.rope_local, rl.size() * 4));
        S3T_CUDA(cudaMalloc(&d.rope_global, rg.size() * 4));
        S3T_CUDA(cudaMalloc(&d.status, sizeof(int)));
        S3T_CUDA(cudaMemcpy(d.rope_local, rl.data(), rl.size() * 4, cudaMemcpyHostToDevice));
        S3T_CUDA(cudaMemcpy(d.rope_global, rg.data(), rg.size() * 4, cudaMemcpyHostToDevice));
        S3T_CUDA(cudaMemset(d.status, 0, sizeof(int)));
        for (int g = 0; g < 2; ++g) {
            const std::vector<float>& tab = g ? rg : rl;
            const int P = g ? kGrid : kWindow;
            std::vector<float> t(tab.size());
            for (int pos = 0; pos < P; ++pos)
                for (int r = 0; r < 32; ++r) t[size_t(r) * P + pos] = tab[size_t(pos) * 32 + r];
            float** dst = g ? &d.rope_global_t : &d.rope_local_t;
            S3T_CUDA(cudaMalloc(dst, t.size() * 4));
            S3T_CUDA(cudaMemcpy(*dst, t.data(), t.size() * 4, cudaMemcpyHostToDevice));
        }
        d.ready = true;
    }
    *out = &d;
    return 0;
}

const char* status_message(int code) {
    switch (code) {
        case kErrTimeoutProducer: return "device wait timed out in a TMA producer";
        case kErrTimeoutMma: return "device wait timed out in an MMA issuer";
        case kErrTimeoutEpilogue: return "device wait timed out in an epilogue/softmax warp";
        case kErrTimeoutDrain: return "device wait timed out while draining after an error";
        case kErrTimeoutProbe: return "device wait timed out in the wait-timeout self-test";
    }
    return "unknown device error";
}

// ------------------------------------------------------------------ GGUF ---

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;
};

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (end - p < int64_t(sizeof(T))) {
            ok = false;
            return v;
        }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || uint64_t(end - p) < n) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p), n);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if (uint64_t(end - p) < n) ok = false;
        else p += n;
    }
};

// Size of one GGUF metadata value of the given type (gguf.cpp type table).
bool skip_value(Reader& r, uint32_t type, uint32_t* u32_out) {
    static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (type == 8) {
        r.str();
    } else if (type == 9) {
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        if (et == 8) {
            for (uint64_t i = 0; i < n && r.ok; ++i) r.str();
        } else if (et < 13 && et != 9) {
            r.skip(n * sizes[et]);
        } else {
            return false;
        }
    } else if (type < 13) {
        if (type == 4 && u32_out) *u32_out = r.get<uint32_t>();
        else r.skip(sizes[type]);
    } else {
        return false;
    }
    return r.ok;
}

// Sidecar written by tools/convert_mlx_sam3_to_gguf.py:596-598:
// {"t_<sha1[:12]>": "<original name>", ...}.  Read like
// src/gguf_model.cpp:28-47 (every "a": "b" pair, in either direction).
void load_aliases(const std::string& path, std::unordered_map<std::string, std::string>& orig_to_short) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return;
    std::string text;
    char buf[65536];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) text.append(buf, n);
    fclose(f);
    std::vector<std::string> strs;
    size_t i = 0;
    std::vector<size_t> after;  // position after each string
    while (i < text.size()) {
        if (text[i] == '"') {
            size_t j = i + 1;
            std::string s;
            while (j < text.size() && text[j] != '"') {
                if (text[j] == '\\' && j + 1 < text.size()) ++j;
                s.push_back(text[j++]);
            }
            strs.push_back(s);
            after.push_back(j + 1);
            i = j + 1;
        } else {
            ++i;
        }
    }
    for (size_t k = 0; k + 1 < strs.size(); ++k) {
        size_t q = after[k];
        while (q < text.size() && isspace(static_cast<unsigned char>(text[q]))) ++q;
        if (q < text.size() && text[q] == ':') {
            orig_to_short[strs[k + 1]] = strs[k];
            orig_to_short[strs[k]] = strs[k];
            ++k;
        }
    }
}

// A GGUF file mapped read-only, with its trunk tensors under their original
// names (the converter's hashed names resolved through the sidecar).  Every
// count, size and offset read from the file is checked against the file's
// length before it is used, so a truncated or corrupt file is an error, not
// an out-of-bounds read or a huge allocation.
struct GgufFile {
    void* map = MAP_FAILED;
    size_t size = 0;
    struct Tensor {
        uint32_t type;
        int64_t ne[4];
        uint64_t offset;   // from the start of the file
        uint64_t nbytes;
    };
    std::vector<std::pair<std::string, Tensor>> trunk;
    const uint8_t* base() const { return static_cast<const uint8_t*>(map); }
    ~GgufFile() {
        if (map != MAP_FAILED) munmap(map, size);
    }
};

int open_gguf(const char* path, const char* map_path, GgufFile& f) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(std::string("cannot open ") + path);
    struct stat stt;
    if (fstat(fd, &stt) != 0) {
        close(fd);
        return fail(std::string("cannot stat ") + path);
    }
    f.size = size_t(stt.st_size);
    if (f.size < 24) {
        close(fd);
        return fail(std::string("not a GGUF file (too short): ") + path);
    }
    f.map = mmap(nullptr, f.size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (f.map == MAP_FAILED) return fail(std::string("mmap failed for ") + path);
    const uint8_t* base = f.base();
    Reader r{base, base + f.size};
    if (r.get<uint32_t>() != 0x46554747u) return fail("not a GGUF file");   // "GGUF"
    const uint32_t version = r.get<uint32_t>();
    if (version < 2 || version > 3) return fail("unsupported GGUF version " + std::to_string(version));
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    const uint64_t rest = uint64_t(r.end - r.p);
    // A tensor record takes at least 24 bytes (name length, dims, type,
    // offset) and a key/value pair at least 13 (key length, type, a value).
    if (n_tensors > rest / 24) return fail("corrupt GGUF header: tensor count " + std::to_string(n_tensors));
    if (n_kv > rest / 13) return fail("corrupt GGUF header: metadata count " + std::to_string(n_kv));
    uint32_t alignment = 32;   // gguf.h GGUF_DEFAULT_ALIGNMENT
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t vt = r.get<uint32_t>();
        uint32_t u = 0;
        if (!skip_value(r, vt, key == "general.alignment" ? &u : nullptr)) r.ok = false;
        if (key == "general.alignment" && u) alignment = u;
    }
    if (!r.ok) return fail("truncated GGUF metadata");
    if (alignment & (alignment - 1)) return fail("corrupt GGUF header: alignment " + std::to_string(alignment));
    std::vector<GgufTensor> ts(n_tensors);
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        ts[i].name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (nd > 4) return fail("corrupt GGUF tensor record: " + std::to_string(nd) + " dimensions");
        for (uint32_t d = 0; d < nd; ++d) ts[i].ne[d] = int64_t(r.get<uint64_t>());
        ts[i].type = r.get<uint32_t>();
        ts[i].offset = r.get<uint64_t>();
    }
    if (!r.ok) return fail("truncated GGUF header");
    const uint64_t hdr = uint64_t(r.p - base);
    const uint64_t data = (hdr + alignment - 1) / alignment * alignment;
    std::unordered_map<std::string, std::string> o2s;
    load_aliases(map_path ? std::string(map_path) : std::string(path) + ".tensor_map.json", o2s);
    std::unordered_map<std::string, std::string> s2o;   // hashed name -> original
    for (const auto& kv : o2s)
        if (kv.first != kv.second) s2o[kv.second] = kv.first;
    for (const auto& t : ts) {
        auto al = s2o.find(t.name);
        const std::string& orig = al != s2o.end() ? al->second : t.name;
        if (orig.rfind(kPrefix, 0) != 0 && orig.rfind(kNeckPrefix, 0) != 0) continue;
        int64_t n = 1;
        for (int d = 0; d < 4; ++d) {
            if (t.ne[d] <= 0 || t.ne[d] > (int64_t(1) << 40) / n) return fail("corrupt GGUF shape for " + orig);
            n *= t.ne[d];
        }
        const int64_t nb = type_nbytes(int(t.type), n);
        if (nb < 0) return fail("unsupported tensor type in " + orig);
        if (data > f.size || t.offset > f.size - data || uint64_t(nb) > f.size - data - t.offset)
            return fail("tensor data out of file bounds: " + orig);
        GgufFile::Tensor tt{t.type, {t.ne[0], t.ne[1], t.ne[2], t.ne[3]}, data + t.offset, uint64_t(nb)};
        f.trunk.emplace_back(orig, tt);
    }
    return 0;
}

}  // namespace

// ---------------------------------------------------------------- context ---

struct Staged {
    int type = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    size_t nbytes = 0;
    void* dev = nullptr;          // raw bytes on the device (linears)
    std::vector<uint8_t> host;    // raw bytes on the host (small tensors, patch embed)
};

struct LayerW {
    __half *qkv = nullptr, *proj = nullptr, *fc1 = nullptr, *fc2 = nullptr;
    int qkv_t = 0, proj_t = 0, fc1_t = 0, fc2_t = 0;
    float *n1w, *n1b, *qkv_b, *proj_b, *n2w, *n2b, *fc1_b, *fc2_b;
};

struct GraphKey {
    int batch, n_layers;
    const void* in;
    void* out;
    bool operator<(const GraphKey& o) const {
        return std::tie(batch, n_layers, in, out) < std::tie(o.batch, o.n_layers, o.in, o.out);
    }
};

struct s3t_ctx {
    int device = 0;
    DeviceState* dev = nullptr;
    cudaStream_t stream = nullptr;
    std::unordered_map<std::string, Staged> staged;
    bool finalized = false;
    int n_layers = 0;
    std::vector<void*> allocs;

    __half* patch_w = nullptr;
    float* pos = nullptr;
    float *lnpre_w = nullptr, *lnpre_b = nullptr;
    LayerW layers[kLayers];
    // The first operation of each neck level (s3t_neck_first), when the file
    // holds the neck: fp16 weight rows [rows][1024] and fp32 bias per row.
    struct NeckFirst {
        int oc = 0, rows = 0;     // output channels; GEMM rows (4 * oc for a 2x2 deconv)
        __half* w = nullptr;
        float* bias = nullptr;
        std::string missing;      // why the level is unavailable
    } neck[4];

    int ws_batch = 0;
    std::vector<void*> ws_allocs;
    std::vector<void*> sk_allocs;   // sk_work, sk_flags: independent of the batch
    float* x = nullptr;
    __half *a16 = nullptr, *qkv = nullptr, *attn = nullptr, *h = nullptr, *cols = nullptr;
    float *img = nullptr, *out = nullptr;
    // Stream-K partials and flags of the pair GEMM (one slot per CTA pair).
    float* sk_work = nullptr;
    int* sk_flags = nullptr;
    int sk_slots = 0;
    uint8_t* rgb = nullptr;   // device copy of host uint8 images (s3t_trunk_run_rgb8)
    size_t rgb_cap = 0;

    // Captured trunk graphs by (batch, layers, input, output), at most
    // kMaxGraphs of them; the least recently launched one is dropped beyond
    // that (a caller whose allocator hands out fresh buffers on every call
    // would otherwise capture a new graph per call and never free one).
    struct CachedGraph {
        cudaGraphExec_t exec;
        uint64_t last_use;
    };
    std::map<GraphKey, CachedGraph> graphs;
    uint64_t graph_clock = 0;
    cudaStream_t copy_in = nullptr, copy_out = nullptr;   // host-buffer pipelining
    std::vector<cudaEvent_t> events;
    // Set only during s3t_trunk_profile: an event is recorded after every launch.
    std::vector<std::pair<int, cudaEvent_t>>* prof = nullptr;
};

namespace {

template <typename T>
int dev_alloc(std::vector<void*>& list, T** p, size_t bytes) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, bytes);
    if (e != cudaSuccess) return fail("cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    list.push_back(q);
    *p = static_cast<T*>(q);
    return 0;
}

constexpr size_t kMaxGraphs = 16;

void free_graphs(s3t_ctx* c) {
    for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second.exec);
    c->graphs.clear();
}

void free_workspace(s3t_ctx* c) {
    free_graphs(c);
    for (void* p : c->ws_allocs) cudaFree(p);
    c->ws_allocs.clear();
    c->ws_batch = 0;
}

int ensure_workspace(s3t_ctx* c, int batch) {
    if (batch <= c->ws_batch) return 0;
    free_workspace(c);
    const size_t M = size_t(batch) * kTokens;
    auto& L = c->ws_allocs;
    if (dev_alloc(L, &c->x, M * kDim * 4) || dev_alloc(L, &c->a16, M * kDim * 2) ||
        dev_alloc(L, &c->qkv, 3 * M * kDim * 2) || dev_alloc(L, &c->attn, M * kDim * 2) ||
        dev_alloc(L, &c->h, M * kMlp * 2) || dev_alloc(L, &c->cols, M * kPatchKPad * 2) ||
        dev_alloc(L, &c->img, size_t(batch) * 3 * kImage * kImage * 4) ||
        dev_alloc(L, &c->out, size_t(batch) * kDim * kTokens * 4)) {
        free_workspace(c);
        return -1;
    }
    if (!c->sk_work) {
        const int slots = c->dev->num_sms / 2;
        if (dev_alloc(c->sk_allocs, &c->sk_work, size_t(slots) * kSkSlotFloats * 4) ||
            dev_alloc(c->sk_allocs, &c->sk_flags, size_t(slots) * kSkSlotFlags * 4)) {
            for (void* q : c->sk_allocs) cudaFree(q);
            c->sk_allocs.clear();
            c->sk_work = nullptr;
            c->sk_flags = nullptr;
            free_workspace(c);
            return -1;
        }
        S3T_CUDA(cudaMemset(c->sk_flags, 0, size_t(slots) * kSkSlotFlags * 4));
        c->sk_slots = slots;
    }
    c->ws_batch = batch;
    return 0;
}

void use_stream_k(const s3t_ctx* c, GemmArgs& g) {
    g.sk_work = c->sk_work;
    g.sk_flags = c->sk_flags;
    g.sk_slots = c->sk_slots;
}

// Stream-K flags back to zero (a run that gave up may have left some set).
int reset_stream_k(const s3t_ctx* c, cudaStream_t st) {
    S3T_CUDA(cudaMemsetAsync(c->sk_flags, 0, size_t(c->sk_slots) * kSkSlotFlags * 4, st));
    return 0;
}

// Enqueue the whole trunk on `st` (called under stream capture).
// Kernel classes of the per-launch profile (s3t_trunk_profile).
enum { kProfStem = 0, kProfQkv, kProfAttnWin, kProfAttnGlob, kProfProj, kProfNorm, kProfFc1, kProfFc2, kProfKinds };

int mark(s3t_ctx* c, cudaStream_t st, int kind) {
    if (!c->prof) return 0;
    cudaEvent_t e;
    S3T_CUDA(cudaEventCreate(&e));
    c->prof->emplace_back(kind, e);
    S3T_CUDA(cudaEventRecord(e, st));
    return 0;
}

#define S3T_MARK(kind) \
    do {                                        \
        if (mark(c, st, (kind))) return -1;     \
    } while (0)

// Enqueue block l on the residual c->x, whose norm1 output is already in
// c->a16: QKV GEMM + RoPE + window scatter, attention, proj GEMM + residual,
// LayerNorm, fc1 GEMM + GELU, fc2 GEMM + residual (src/vision_trunk.cpp:377-459).
// out_nchw: also write the block's output as NCHW (last block), or null.
int enqueue_block(s3t_ctx* c, int l, int batch, float* out_nchw, cudaStream_t st) {
    const int M = batch * kTokens;
    const int sms = c->dev->num_sms;
    int* status = c->dev->status;
    const int64_t qkv_stride = int64_t(M) * kDim;
    const LayerW& w = c->layers[l];
    const bool glob = is_global_attention_block(l);

    GemmArgs q{};
    q.M = M; q.N = 3 * kDim; q.K = kDim;
    q.bias = w.qkv_b;
    q.qkv = c->qkv;
    q.qkv_stride = qkv_stride;
    q.windowed = glob ? 0 : 1;
    q.rope_local = c->dev->rope_local;
    q.rope_global = c->dev->rope_global;
    q.rope_local_t = c->dev->rope_local_t;
    q.rope_global_t = c->dev->rope_global_t;
    q.status = status;
    use_stream_k(c, q);
    S3T_CUDA(launch_gemm(c->a16, w.qkv, q, kEpiQkv, sms, st));
    S3T_MARK(kProfQkv);

    AttnArgs at{};
    at.q = c->qkv;
    at.k = c->qkv + qkv_stride;
    at.v = c->qkv + 2 * qkv_stride;
    at.groups = glob ? batch : batch * 9;
    at.L = glob ? kTokens : kWindow * kWindow;
    at.windowed = glob ? 0 : 1;
    at.scale_log2 = 0.125f * 1.4426950408889634f;
    at.bf16 = 0;
    at.q8 = w.proj_t == S3T_TYPE_Q8_0;
    at.out = c->attn;
    at.status = status;
    S3T_CUDA(launch_attention(at, st));
    S3T_MARK(glob ? kProfAttnGlob : kProfAttnWin);

    GemmArgs p{};
    p.M = M; p.N = kDim; p.K = kDim;
    p.bias = w.proj_b;
    p.resid = c->x;
    p.status = status;
    use_stream_k(c, p);
    S3T_CUDA(launch_gemm(c->attn, w.proj, p, kEpiResid, sms, st));
    S3T_MARK(kProfProj);

    S3T_CUDA(launch_layernorm(c->x, M, w.n2w, w.n2b, c->a16, w.fc1_t == S3T_TYPE_Q8_0, st));
    S3T_MARK(kProfNorm);

    GemmArgs f1{};
    f1.M = M; f1.N = kMlp; f1.K = kDim;
    f1.bias = w.fc1_b;
    f1.out16 = c->h;
    f1.gelu = 1;
    f1.q8 = w.fc2_t == S3T_TYPE_Q8_0;
    f1.status = status;
    use_stream_k(c, f1);
    S3T_CUDA(launch_gemm(c->a16, w.fc1, f1, kEpiF16, sms, st));
    S3T_MARK(kProfFc1);

    GemmArgs f2{};
    f2.M = M; f2.N = kDim; f2.K = kMlp;
    f2.bias = w.fc2_b;
    f2.resid = c->x;
    f2.out_nchw = out_nchw;
    f2.status = status;
    use_stream_k(c, f2);
    S3T_CUDA(launch_gemm(c->h, w.fc2, f2, kEpiResid, sms, st));
    S3T_MARK(kProfFc2);

    return 0;
}

int enqueue_trunk(s3t_ctx* c, const float* images, int batch, int n_layers, float* out, cudaStream_t st) {
    const int M = batch * kTokens;
    const int sms = c->dev->num_sms;
    int* status = c->dev->status;
    S3T_CUDA(cudaMemsetAsync(status, 0, sizeof(int), st));
    if (reset_stream_k(c, st)) return -1;
    S3T_MARK(-1);
    S3T_CUDA(launch_im2col(images, batch, c->cols, st));

    GemmArgs g{};
    g.M = M;
    g.N = kDim;
    g.K = kPatchKPad;
    g.resid = c->x;
    g.pos = c->pos;
    g.status = status;
    use_stream_k(c, g);
    S3T_CUDA(launch_gemm(c->cols, c->patch_w, g, kEpiPatch, sms, st));
    S3T_CUDA(launch_layernorm_stem(c->x, M, c->lnpre_w, c->lnpre_b, c->layers[0].n1w, c->layers[0].n1b, c->a16,
                                   c->layers[0].qkv_t == S3T_TYPE_Q8_0, st));
    S3T_MARK(kProfStem);

    for (int l = 0; l < n_layers; ++l) {
        if (enqueue_block(c, l, batch, (l == n_layers - 1) ? out : nullptr, st)) return -1;
        if (l + 1 < n_layers) {
            const LayerW& nx = c->layers[l + 1];
            S3T_CUDA(launch_layernorm(c->x, M, nx.n1w, nx.n1b, c->a16, nx.qkv_t == S3T_TYPE_Q8_0, st));
            S3T_MARK(kProfNorm);
        }
    }
    return 0;
}

// Stem-only run: patch embed + pos + ln_pre; output NCHW through a host-side
// transpose (diagnostic path, not performance relevant).
int run_stem(s3t_ctx* c, const float* images, int batch, float* out_host_or_dev, bool out_dev, cudaStream_t st) {
    const int M = batch * kTokens;
    S3T_CUDA(cudaMemsetAsync(c->dev->status, 0, sizeof(int), st));
    S3T_CUDA(launch_im2col(images, batch, c->cols, st));
    GemmArgs g{};
    g.M = M; g.N = kDim; g.K = kPatchKPad;
    g.resid = c->x;
    g.pos = c->pos;
    g.status = c->dev->status;
    S3T_CUDA(launch_gemm(c->cols, c->patch_w, g, kEpiPatch, c->dev->num_sms, st));
    S3T_CUDA(launch_layernorm_stem(c->x, M, c->lnpre_w, c->lnpre_b, c->lnpre_w, c->lnpre_b, c->a16, 0, st));
    std::vector<float> tok(size_t(M) * kDim), nchw(size_t(M) * kDim);
    S3T_CUDA(cudaMemcpyAsync(tok.data(), c->x, tok.size() * 4, cudaMemcpyDeviceToHost, st));
    S3T_CUDA(cudaStreamSynchronize(st));
    for (int b = 0; b < batch; ++b)
        for (int t = 0; t < kTokens; ++t)
            for (int ch = 0; ch < kDim; ++ch)
                nchw[(size_t(b) * kDim + ch) * kTokens + t] = tok[(size_t(b) * kTokens + t) * kDim + ch];
    S3T_CUDA(cudaMemcpy(out_host_or_dev, nchw.data(), nchw.size() * 4,
                        out_dev ? cudaMemcpyHostToDevice : cudaMemcpyHostToHost));
    return 0;
}

int check_status(s3t_ctx* c, cudaStream_t st) {
    int code = 0;
    S3T_CUDA(cudaMemcpyAsync(&code, c->dev->status, sizeof(int), cudaMemcpyDeviceToHost, st));
    S3T_CUDA(cudaStreamSynchronize(st));
    if (code != 0) return fail(std::string("device error: ") + status_message(code));
    return 0;
}

// The captured CUDA graph of the trunk for (batch, n_layers, input, output),
// captured on first use.
int trunk_graph(s3t_ctx* c, const float* din, int batch, int n_layers, float* dout, cudaGraphExec_t* out) {
    const GraphKey key{batch, n_layers, din, dout};
    auto it = c->graphs.find(key);
    if (it == c->graphs.end() && c->graphs.size() >= kMaxGraphs) {
        auto lru = c->graphs.begin();
        for (auto g = c->graphs.begin(); g != c->graphs.end(); ++g)
            if (g->second.last_use < lru->second.last_use) lru = g;
        S3T_CUDA(cudaDeviceSynchronize());   // the evicted graph may still be running
        S3T_CUDA(cudaGraphExecDestroy(lru->second.exec));
        c->graphs.erase(lru);
    }
    if (it == c->graphs.end()) {
        cudaStream_t cap;
        S3T_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
        S3T_CUDA(cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal));
        int rc;
        {
            PdlScope pdl(true);
            rc = enqueue_trunk(c, din, batch, n_layers, dout, cap);
        }
        cudaGraph_t graph = nullptr;
        const cudaError_t ec = cudaStreamEndCapture(cap, &graph);
        cudaStreamDestroy(cap);
        if (rc) {
            if (graph) cudaGraphDestroy(graph);
            return -1;
        }
        S3T_CUDA(ec);
        cudaGraphExec_t exec = nullptr;
        const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        S3T_CUDA(ei);
        it = c->graphs.emplace(key, s3t_ctx::CachedGraph{exec, 0}).first;
    }
    it->second.last_use = ++c->graph_clock;
    *out = it->second.exec;
    return 0;
}

// Images per pipelined chunk when both buffers are on the host.
constexpr int kHostChunk = 8;

// Images per pipelined chunk for a host-buffer batch: 8, or half the batch
// for 5 to 16 images (the exposed first upload and last download of a whole
// 8-image batch, 270 MB, cost more than running it as two 4-image chunks);
// 0 when the batch runs as one piece.
int host_chunk(int batch) {
    if (batch > 2 * kHostChunk) return kHostChunk;
    if (batch > 4) return (batch + 1) / 2;
    return 0;
}

int ensure_events(s3t_ctx* c, size_t n) {
    while (c->events.size() < n) {
        cudaEvent_t e;
        S3T_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        c->events.push_back(e);
    }
    if (!c->copy_in) S3T_CUDA(cudaStreamCreateWithFlags(&c->copy_in, cudaStreamNonBlocking));
    if (!c->copy_out) S3T_CUDA(cudaStreamCreateWithFlags(&c->copy_out, cudaStreamNonBlocking));
    return 0;
}

// Host images -> host features for several chunks: the upload of chunk k+1
// and the download of chunk k-1 run on their own streams (their own copy
// engines) while the trunk runs chunk k on `st`, so only the first upload
// and the last download are not hidden behind compute.
int run_host_pipelined(s3t_ctx* c, const float* images, int batch, int n_layers, float* out, cudaStream_t st) {
    const int chunk = host_chunk(batch);
    const int nc = (batch + chunk - 1) / chunk;
    if (ensure_events(c, size_t(2 * nc + 1))) return -1;
    const size_t img_elems = size_t(3) * kImage * kImage, out_elems = size_t(kDim) * kTokens;
    cudaEvent_t start = c->events[2 * nc];
    S3T_CUDA(cudaEventRecord(start, st));   // earlier work on st may still use the buffers
    S3T_CUDA(cudaStreamWaitEvent(c->copy_in, start, 0));
    S3T_CUDA(cudaStreamWaitEvent(c->copy_out, start, 0));
    for (int k = 0; k < nc; ++k) {
        const int b0 = k * chunk, nb = std::min(chunk, batch - b0);
        S3T_CUDA(cudaMemcpyAsync(c->img + b0 * img_elems, images + b0 * img_elems, nb * img_elems * 4,
                                 cudaMemcpyHostToDevice, c->copy_in));
        S3T_CUDA(cudaEventRecord(c->events[k], c->copy_in));
    }
    for (int k = 0; k < nc; ++k) {
        const int b0 = k * chunk, nb = std::min(chunk, batch - b0);
        cudaGraphExec_t g = nullptr;
        if (trunk_graph(c, c->img + b0 * img_elems, nb, n_layers, c->out + b0 * out_elems, &g)) return -1;
        S3T_CUDA(cudaStreamWaitEvent(st, c->events[k], 0));
        S3T_CUDA(cudaGraphLaunch(g, st));
        S3T_CUDA(cudaEventRecord(c->events[nc + k], st));
        S3T_CUDA(cudaStreamWaitEvent(c->copy_out, c->events[nc + k], 0));
        S3T_CUDA(cudaMemcpyAsync(out + b0 * out_elems, c->out + b0 * out_elems, nb * out_elems * 4,
                                 cudaMemcpyDeviceToHost, c->copy_out));
    }
    S3T_CUDA(cudaEventRecord(start, c->copy_out));
    S3T_CUDA(cudaStreamWaitEvent(st, start, 0));
    return check_status(c, st);
}

int run_impl(s3t_ctx* c, const float* images, int batch, int n_layers, float* out, int flags, void* stream) {
    if (!c) return fail("ctx is null");
    if (!c->finalized) return fail("weights not finalized (call s3t_finalize_weights)");
    if (!images || !out) return fail("images or out is null");
    if (batch <= 0) return fail("batch must be positive");
    if (n_layers < 0 || n_layers > c->n_layers) return fail("n_layers out of range");
    S3T_CUDA(cudaSetDevice(c->device));
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
    if (ensure_workspace(c, batch)) return -1;

    const bool in_dev = flags & S3T_IMAGES_ON_DEVICE, out_dev = flags & S3T_OUTPUT_ON_DEVICE;
    if (!in_dev && !out_dev && n_layers > 0 && host_chunk(batch) > 0)
        return run_host_pipelined(c, images, batch, n_layers, out, st);

    const size_t in_bytes = size_t(batch) * 3 * kImage * kImage * 4;
    const size_t out_bytes = size_t(batch) * kDim * kTokens * 4;
    const float* din = in_dev ? images : c->img;
    float* dout = out_dev ? out : c->out;
    if (!in_dev) S3T_CUDA(cudaMemcpyAsync(c->img, images, in_bytes, cudaMemcpyHostToDevice, st));

    if (n_layers == 0) {
        if (run_stem(c, din, batch, out, out_dev, st)) return -1;
        return check_status(c, st);
    }

    cudaGraphExec_t g = nullptr;
    if (trunk_graph(c, din, batch, n_layers, dout, &g)) return -1;
    S3T_CUDA(cudaGraphLaunch(g, st));
    if (!out_dev) {
        S3T_CUDA(cudaMemcpyAsync(out, c->out, out_bytes, cudaMemcpyDeviceToHost, st));
        return check_status(c, st);
    }
    return 0;
}

// Upload helpers used by finalize.
int upload_f32_vec(s3t_ctx* c, const Staged& s, int64_t n, float** dst) {
    std::vector<float> v(n);
    if (s.type == S3T_TYPE_F32) {
        memcpy(v.data(), s.host.data(), n * 4);
    } else if (s.type == S3T_TYPE_F16) {
        const __half* h = reinterpret_cast<const __half*>(s.host.data());
        for (int64_t i = 0; i < n; ++i) v[i] = __half2float(h[i]);
    } else {
        return fail("unsupported type for a vector tensor");
    }
    if (dev_alloc(c->allocs, dst, n * 4)) return -1;
    S3T_CUDA(cudaMemcpy(*dst, v.data(), n * 4, cudaMemcpyHostToDevice));
    return 0;
}

// The neck's first operations as GEMM weight rows (src/vision_neck.cpp:262-345):
// level 0 convs.0.dconv_2x2_0 and level 1 convs.1.dconv_2x2 (2x2 stride-2
// transposed convs, ggml ne [IC, KW, KH, OC]: row r = oc + OC * (kw + 2 kh), the
// row order of deconv2d_bias's mul_mat, :91-93); levels 2 and 3 convs.N.conv_1x1
// (ne [IC, 1, 1, OC]: row = oc).  F16 values are kept, F32 ones rounded to fp16.
// A level whose tensors the file does not hold is left unavailable.
int prepare_neck(s3t_ctx* c) {
    const std::string P(kNeckPrefix);
    const char* names[4] = {"0.dconv_2x2_0", "1.dconv_2x2", "2.conv_1x1", "3.conv_1x1"};
    for (int lvl = 0; lvl < 4; ++lvl) {
        auto& nf = c->neck[lvl];
        const std::string wn = P + names[lvl] + ".weight", bn = P + names[lvl] + ".bias";
        auto wi = c->staged.find(wn), bi = c->staged.find(bn);
        if (wi == c->staged.end() || bi == c->staged.end()) {
            nf.missing = "missing tensor: " + (wi == c->staged.end() ? wn : bn);
            continue;
        }
        const Staged& ws = wi->second;
        const Staged& bs = bi->second;
        const int k = lvl < 2 ? 2 : 1;
        const int64_t oc = ws.ne[3];
        if (ws.ne[0] != kDim || ws.ne[1] != k || ws.ne[2] != k || oc <= 0 || oc % 32 || oc > kMlp / 4 ||
            bs.ne[0] != oc || bs.ne[1] * bs.ne[2] * bs.ne[3] != 1)
            return fail("unexpected shape for " + wn);
        if ((ws.type != S3T_TYPE_F16 && ws.type != S3T_TYPE_F32) || (bs.type != S3T_TYPE_F32 && bs.type != S3T_TYPE_F16))
            return fail("unsupported type for " + wn);
        const int rows = int(oc) * k * k;
        std::vector<__half> wr(size_t(rows) * kDim);
        std::vector<float> br(rows);
        auto wval = [&](size_t i) -> float {
            if (ws.type == S3T_TYPE_F32) {
                float v;
                memcpy(&v, ws.host.data() + i * 4, 4);
                return v;
            }
            return __half2float(reinterpret_cast<const __half*>(ws.host.data())[i]);
        };
        for (int o = 0; o < oc; ++o) {
            const float bv = bs.type == S3T_TYPE_F32 ? reinterpret_cast<const float*>(bs.host.data())[o]
                                                      : __half2float(reinterpret_cast<const __half*>(bs.host.data())[o]);
            for (int kh = 0; kh < k; ++kh)
                for (int kw = 0; kw < k; ++kw) {
                    const int r = o + int(oc) * (kw + k * kh);
                    br[r] = bv;
                    for (int ic = 0; ic < kDim; ++ic)
                        wr[size_t(r) * kDim + ic] = __float2half_rn(wval(size_t(ic) + kDim * (kw + k * (kh + size_t(k) * o))));
                }
        }
        if (dev_alloc(c->allocs, &nf.w, wr.size() * 2) || dev_alloc(c->allocs, &nf.bias, br.size() * 4)) return -1;
        S3T_CUDA(cudaMemcpy(nf.w, wr.data(), wr.size() * 2, cudaMemcpyHostToDevice));
        S3T_CUDA(cudaMemcpy(nf.bias, br.data(), br.size() * 4, cudaMemcpyHostToDevice));
        nf.oc = int(oc);
        nf.rows = rows;
    }
    return 0;
}

}  // namespace

int s3t::set_last_error(const char* msg) { return fail(msg); }

cudaStream_t s3t::ctx_stream(const s3t_ctx* c) { return c ? c->stream : nullptr; }

bool s3t::ctx_stem_view(const s3t_ctx* c, StemView* out) {
    if (!c || !c->finalized || !out) return false;
    out->device = c->device;
    out->num_sms = c->dev->num_sms;
    out->patch_w = c->patch_w;
    out->pos = c->pos;
    out->ln_w = c->lnpre_w;
    out->ln_b = c->lnpre_b;
    out->status = c->dev->status;
    out->stream = c->stream;
    return true;
}

// Nothing may throw across the C ABI (std::bad_alloc from a host buffer, a
// std::length_error from a container): every entry point's body runs inside
// a try block whose handlers turn an exception into the -1 / last-error
// convention (NULL for s3t_create; s3t_destroy swallows it).
#define S3T_CATCH_INT                                                              \
    catch (const std::bad_alloc&) {                                                \
        return fail("out of host memory");                                         \
    }                                                                              \
    catch (const std::exception& e) {                                              \
        return fail(std::string("internal error: ") + e.what());                   \
    }                                                                              \
    catch (...) {                                                                  \
        return fail("internal error");                                             \
    }
#define S3T_CATCH_PTR                                                              \
    catch (const std::exception& e) {                                              \
        fail(std::string("internal error: ") + e.what());                          \
        return nullptr;                                                            \
    }                                                                              \
    catch (...) {                                                                  \
        fail("internal error");                                                    \
        return nullptr;                                                            \
    }
#define S3T_CATCH_VOID \
    catch (...) {      \
    }

extern "C" {

const char* s3t_last_error(void) { return g_last_error.c_str(); }

s3t_ctx* s3t_create(int device) {
    try {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
            fail("no CUDA device " + std::to_string(device));
            return nullptr;
        }
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return nullptr;
        s3t_ctx* c = new s3t_ctx();
        c->device = device;
        c->dev = ds;
        if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
            fail("stream creation failed");
            delete c;
            return nullptr;
        }
        return c;
    } S3T_CATCH_PTR
}

void s3t_destroy(s3t_ctx* c) {
    try {
        if (!c) return;
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        free_workspace(c);
        for (void* p : c->sk_allocs) cudaFree(p);
        for (auto& kv : c->staged)
            if (kv.second.dev) cudaFree(kv.second.dev);
        for (void* p : c->allocs) cudaFree(p);
        if (c->rgb) cudaFree(c->rgb);
        for (cudaEvent_t e : c->events) cudaEventDestroy(e);
        if (c->copy_in) cudaStreamDestroy(c->copy_in);
        if (c->copy_out) cudaStreamDestroy(c->copy_out);
        cudaStreamDestroy(c->stream);
        delete c;
    } S3T_CATCH_VOID
}

int s3t_set_weight(s3t_ctx* c, const char* name, int type, const int64_t ne[4], const void* bytes, size_t nbytes) {
    try {
        if (!c || !name || !ne || !bytes) return fail("null argument to s3t_set_weight");
        if (c->finalized) return fail("weights already finalized");
        int64_t n = 1;
        for (int i = 0; i < 4; ++i) {
            if (ne[i] <= 0) return fail(std::string("bad shape for ") + name);
            n *= ne[i];
        }
        const int64_t need = type_nbytes(type, n);
        if (need < 0) return fail(std::string("unsupported ggml type ") + std::to_string(type) + " for " + name);
        if (int64_t(nbytes) != need) return fail(std::string("size mismatch for ") + name);
        Staged s;
        s.type = type;
        for (int i = 0; i < 4; ++i) s.ne[i] = ne[i];
        s.nbytes = nbytes;
        const std::string nm(name);
        const bool linear = nm.find(".weight") != std::string::npos &&
                            (nm.find(".attn.") != std::string::npos || nm.find(".mlp.") != std::string::npos);
        if (cudaSetDevice(c->device) != cudaSuccess) return fail("cudaSetDevice failed");
        if (linear) {
            if (cudaMalloc(&s.dev, nbytes) != cudaSuccess) return fail("cudaMalloc failed for " + nm);
            cudaError_t e = cudaMemcpy(s.dev, bytes, nbytes, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) {
                cudaFree(s.dev);
                return fail(std::string("upload failed: ") + cudaGetErrorString(e));
            }
        } else {
            s.host.assign(static_cast<const uint8_t*>(bytes), static_cast<const uint8_t*>(bytes) + nbytes);
        }
        auto it = c->staged.find(nm);
        if (it != c->staged.end() && it->second.dev) cudaFree(it->second.dev);
        c->staged[nm] = std::move(s);
        return 0;
    } S3T_CATCH_INT
}

int s3t_load_gguf(s3t_ctx* c, const char* path, const char* map_path) {
    try {
        if (!c || !path) return fail("null argument to s3t_load_gguf");
        GgufFile f;
        if (open_gguf(path, map_path, f)) return -1;
        for (const auto& t : f.trunk)
            if (s3t_set_weight(c, t.first.c_str(), int(t.second.type), t.second.ne, f.base() + t.second.offset,
                               size_t(t.second.nbytes)))
                return -1;
        return 0;
    } S3T_CATCH_INT
}

int s3t_gguf_inspect(const char* path, const char* map_path, int* n_trunk_tensors, int* n_layers) {
    try {
        if (!path) return fail("null argument to s3t_gguf_inspect");
        GgufFile f;
        if (open_gguf(path, map_path, f)) return -1;
        int layers = 0;
        const std::string P(kPrefix);
        for (bool found = true; found && layers < kLayers;) {
            found = false;
            const std::string q = P + ".blocks." + std::to_string(layers) + ".attn.qkv.weight";
            for (const auto& t : f.trunk) found = found || t.first == q;
            if (found) ++layers;
        }
        if (n_trunk_tensors) *n_trunk_tensors = int(f.trunk.size());
        if (n_layers) *n_layers = layers;
        return 0;
    } S3T_CATCH_INT
}

int s3t_finalize_weights(s3t_ctx* c) {
    try {
        if (!c) return fail("ctx is null");
        if (c->finalized) return 0;
        if (cudaSetDevice(c->device) != cudaSuccess) return fail("cudaSetDevice failed");
        auto req = [&](const std::string& nm, int64_t e0, int64_t e1, int64_t e2, int64_t e3) -> const Staged* {
            auto it = c->staged.find(nm);
            if (it == c->staged.end()) {
                fail("missing tensor: " + nm);   // src/vision_trunk.cpp:27-33
                return nullptr;
            }
            const Staged& s = it->second;
            if (s.ne[0] != e0 || s.ne[1] != e1 || s.ne[2] != e2 || s.ne[3] != e3) {
                fail("unexpected shape for " + nm);
                return nullptr;
            }
            return &s;
        };
        const std::string P(kPrefix);
        int nl = 0;
        while (nl < kLayers && c->staged.count(P + ".blocks." + std::to_string(nl) + ".attn.qkv.weight")) ++nl;
        if (nl == 0) return fail("missing tensor: " + P + ".blocks.0.attn.qkv.weight");

        const Staged* pw = req(P + ".patch_embed.proj.weight", 3, 14, 14, 1024);
        const Staged* pe = req(P + ".pos_embed", 1024, 577, 1, 1);
        const Staged* lw = req(P + ".ln_pre.weight", 1024, 1, 1, 1);
        const Staged* lb = req(P + ".ln_pre.bias", 1024, 1, 1, 1);
        if (!pw || !pe || !lw || !lb) return -1;
        if (pw->type != S3T_TYPE_F32 && pw->type != S3T_TYPE_F16) return fail("patch_embed must be F32 or F16");

        // Patch-embed weight: GGUF [O][KH][KW][I] -> [O][ic*196 + kh*14 + kw] fp16,
        // zero padded to 640 columns.
        {
            std::vector<__half> wp(size_t(kDim) * kPatchKPad, __float2half(0.f));
            for (int o = 0; o < kDim; ++o)
                for (int kh = 0; kh < 14; ++kh)
                    for (int kw = 0; kw < 14; ++kw)
                        for (int ic = 0; ic < 3; ++ic) {
                            const size_t src = ((size_t(o) * 14 + kh) * 14 + kw) * 3 + ic;
                            float v;
                            if (pw->type == S3T_TYPE_F32) memcpy(&v, pw->host.data() + src * 4, 4);
                            else v = __half2float(reinterpret_cast<const __half*>(pw->host.data())[src]);
                            wp[size_t(o) * kPatchKPad + ic * 196 + kh * 14 + kw] = __float2half_rn(v);
                        }
            if (dev_alloc(c->allocs, &c->patch_w, wp.size() * 2)) return -1;
            S3T_CUDA(cudaMemcpy(c->patch_w, wp.data(), wp.size() * 2, cudaMemcpyHostToDevice));
        }
        if (upload_f32_vec(c, *pe, 577 * 1024, &c->pos) || upload_f32_vec(c, *lw, 1024, &c->lnpre_w) ||
            upload_f32_vec(c, *lb, 1024, &c->lnpre_b))
            return -1;

        for (int l = 0; l < nl; ++l) {
            const std::string b = P + ".blocks." + std::to_string(l);
            LayerW& w = c->layers[l];
            struct Lin { const char* nm; int64_t k, n; __half** dst; int* t; } lins[4] = {
                {".attn.qkv.weight", kDim, 3 * kDim, &w.qkv, &w.qkv_t},
                {".attn.proj.weight", kDim, kDim, &w.proj, &w.proj_t},
                {".mlp.fc1.weight", kDim, kMlp, &w.fc1, &w.fc1_t},
                {".mlp.fc2.weight", kMlp, kDim, &w.fc2, &w.fc2_t},
            };
            for (auto& li : lins) {
                const Staged* s = req(b + li.nm, li.k, li.n, 1, 1);
                if (!s) return -1;
                *li.t = s->type;
                const int64_t n = li.k * li.n;
                if (s->type == S3T_TYPE_F16) {
                    *li.dst = static_cast<__half*>(s->dev);   // already the GEMM operand [N][K]
                    c->allocs.push_back(s->dev);
                    c->staged[b + li.nm].dev = nullptr;
                } else {
                    if (dev_alloc(c->allocs, li.dst, n * 2)) return -1;
                    if (s->type == S3T_TYPE_Q8_0) S3T_CUDA(launch_dequant_q8_0_to_f16(static_cast<const uint8_t*>(s->dev), n, *li.dst, c->stream));
                    else S3T_CUDA(launch_f32_to_f16(static_cast<const float*>(s->dev), n, *li.dst, c->stream));
                }
            }
            struct Vec { const char* nm; int64_t n; float** dst; } vecs[8] = {
                {".norm1.weight", kDim, &w.n1w}, {".norm1.bias", kDim, &w.n1b},
                {".attn.qkv.bias", 3 * kDim, &w.qkv_b}, {".attn.proj.bias", kDim, &w.proj_b},
                {".norm2.weight", kDim, &w.n2w}, {".norm2.bias", kDim, &w.n2b},
                {".mlp.fc1.bias", kMlp, &w.fc1_b}, {".mlp.fc2.bias", kDim, &w.fc2_b},
            };
            for (auto& v : vecs) {
                const Staged* s = req(b + v.nm, v.n, 1, 1, 1);
                if (!s || upload_f32_vec(c, *s, v.n, v.dst)) return -1;
            }
        }
        if (prepare_neck(c)) return -1;
        S3T_CUDA(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->staged)
            if (kv.second.dev) cudaFree(kv.second.dev);
        c->staged.clear();
        c->n_layers = nl;
        c->finalized = true;
        return 0;
    } S3T_CATCH_INT
}

int s3t_num_layers(const s3t_ctx* c) { return c ? c->n_layers : 0; }

int s3t_trunk_run(s3t_ctx* c, const float* images, int batch, float* out, int flags, void* stream) {
    try {
        return run_impl(c, images, batch, c ? c->n_layers : 0, out, flags, stream);
    } S3T_CATCH_INT
}

int s3t_trunk_run_layers(s3t_ctx* c, const float* images, int batch, int n_layers, float* out, int flags,
                         void* stream) {
    try {
        return run_impl(c, images, batch, n_layers, out, flags, stream);
    } S3T_CATCH_INT
}

int s3t_trunk_run_block(s3t_ctx* c, int layer, const float* x_dev, int batch, float* out_dev, void* stream) {
    try {
        if (!c) return fail("ctx is null");
        if (!c->finalized) return fail("weights not finalized (call s3t_finalize_weights)");
        if (!x_dev || !out_dev) return fail("x or out is null");
        if (batch <= 0) return fail("batch must be positive");
        if (layer < 0 || layer >= c->n_layers) return fail("layer out of range");
        S3T_CUDA(cudaSetDevice(c->device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
        if (ensure_workspace(c, batch)) return -1;
        const int M = batch * kTokens;
        const LayerW& w = c->layers[layer];
        S3T_CUDA(cudaMemsetAsync(c->dev->status, 0, sizeof(int), st));
        if (reset_stream_k(c, st)) return -1;
        S3T_CUDA(cudaMemcpyAsync(c->x, x_dev, size_t(M) * kDim * 4, cudaMemcpyDeviceToDevice, st));
        S3T_CUDA(launch_layernorm(c->x, M, w.n1w, w.n1b, c->a16, w.qkv_t == S3T_TYPE_Q8_0, st));
        if (enqueue_block(c, layer, batch, nullptr, st)) return -1;
        S3T_CUDA(cudaMemcpyAsync(out_dev, c->x, size_t(M) * kDim * 4, cudaMemcpyDeviceToDevice, st));
        return check_status(c, st);
    } S3T_CATCH_INT
}

int s3t_trunk_run_rgb8(s3t_ctx* c, const uint8_t* rgb, int width, int height, int batch, float* out, int flags,
                       void* stream) {
    try {
        if (!c) return fail("ctx is null");
        if (!c->finalized) return fail("weights not finalized (call s3t_finalize_weights)");
        if (!rgb || !out) return fail("rgb or out is null");
        if (batch <= 0 || batch > 65535) return fail("batch must be in [1, 65535]");
        if (width <= 0 || height <= 0 || width > kMaxSourceSide || height > kMaxSourceSide)
            return fail("image width and height must be in [1, 32768]");
        S3T_CUDA(cudaSetDevice(c->device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
        if (ensure_workspace(c, batch)) return -1;
        const uint8_t* src = rgb;
        if (!(flags & S3T_IMAGES_ON_DEVICE)) {
            const size_t bytes = size_t(batch) * size_t(height) * size_t(width) * 3;
            if (bytes > c->rgb_cap) {
                if (c->rgb) {
                    S3T_CUDA(cudaStreamSynchronize(st));
                    S3T_CUDA(cudaFree(c->rgb));
                    c->rgb = nullptr;
                    c->rgb_cap = 0;
                }
                void* q = nullptr;
                const cudaError_t e = cudaMalloc(&q, bytes);
                if (e != cudaSuccess) return fail("cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
                c->rgb = static_cast<uint8_t*>(q);
                c->rgb_cap = bytes;
            }
            S3T_CUDA(cudaMemcpyAsync(c->rgb, rgb, bytes, cudaMemcpyHostToDevice, st));
            src = c->rgb;
        }
        S3T_CUDA(launch_resize_rgb8(src, width, height, batch, c->img, st));
        return run_impl(c, c->img, batch, c->n_layers, out, flags | S3T_IMAGES_ON_DEVICE, stream);
    } S3T_CATCH_INT
}

int s3t_trunk_profile(s3t_ctx* c, const float* images_dev, int batch, float* out_dev, void* stream, double* kind_ms,
                      int* kind_launches) {
    try {
        if (!c) return fail("ctx is null");
        if (!c->finalized) return fail("weights not finalized (call s3t_finalize_weights)");
        if (!images_dev || !out_dev || !kind_ms || !kind_launches) return fail("null argument to s3t_trunk_profile");
        if (batch <= 0) return fail("batch must be positive");
        S3T_CUDA(cudaSetDevice(c->device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
        if (ensure_workspace(c, batch)) return -1;
        std::vector<std::pair<int, cudaEvent_t>> ev;
        c->prof = &ev;
        const int rc = enqueue_trunk(c, images_dev, batch, c->n_layers, out_dev, st);
        c->prof = nullptr;
        const cudaError_t se = cudaStreamSynchronize(st);
        for (int k = 0; k < kProfKinds; ++k) {
            kind_ms[k] = 0.0;
            kind_launches[k] = 0;
        }
        for (size_t i = 1; rc == 0 && se == cudaSuccess && i < ev.size(); ++i) {
            float ms = 0.f;
            if (cudaEventElapsedTime(&ms, ev[i - 1].second, ev[i].second) == cudaSuccess && ev[i].first >= 0) {
                kind_ms[ev[i].first] += ms;
                kind_launches[ev[i].first] += 1;
            }
        }
        for (auto& e : ev) cudaEventDestroy(e.second);
        if (rc) return rc;
        S3T_CUDA(se);
        return check_status(c, st);
    } S3T_CATCH_INT
}

int s3t_neck_first_shape(const s3t_ctx* c, int level, int64_t shape[4]) {
    try {
        if (!c || !shape) return fail("null argument to s3t_neck_first_shape");
        if (!c->finalized) return fail("weights not finalized (call s3t_finalize_weights)");
        if (level < 0 || level > 3) return fail("neck level must be in [0, 3]");
        const auto& nf = c->neck[level];
        if (!nf.w) return fail(nf.missing);
        const int side = level < 2 ? 2 * kGrid : level == 2 ? kGrid : kGrid / 2;
        shape[0] = 1;
        shape[1] = nf.oc;
        shape[2] = shape[3] = side;
        return 0;
    } S3T_CATCH_INT
}

int s3t_neck_first(s3t_ctx* c, int level, const float* trunk_dev, int batch, float* out_dev, void* stream) {
    try {
        if (!c) return fail("ctx is null");
        if (!c->finalized) return fail("weights not finalized (call s3t_finalize_weights)");
        if (!trunk_dev || !out_dev) return fail("trunk or out is null");
        if (batch <= 0) return fail("batch must be positive");
        if (level < 0 || level > 3) return fail("neck level must be in [0, 3]");
        const auto& nf = c->neck[level];
        if (!nf.w) return fail(nf.missing);
        S3T_CUDA(cudaSetDevice(c->device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : c->stream;
        if (ensure_workspace(c, batch)) return -1;   // a16 holds the A operand, h the GEMM result
        const int T = level == 3 ? (kGrid / 2) * (kGrid / 2) : kTokens;
        S3T_CUDA(launch_neck_tokens(trunk_dev, batch, level, c->a16, st));
        GemmArgs g{};
        g.M = batch * T;
        g.N = nf.rows;
        g.K = kDim;
        g.bias = nf.bias;
        g.out16 = c->h;
        g.gelu = level == 0;
        g.status = c->dev->status;
        S3T_CUDA(launch_gemm(c->a16, nf.w, g, kEpiF16, c->dev->num_sms, st));
        S3T_CUDA(launch_neck_out(c->h, batch, level, nf.oc, out_dev, st));
        return 0;
    } S3T_CATCH_INT
}

int s3t_sync(s3t_ctx* c, void* stream) {
    try {
        if (!c) return fail("ctx is null");
        S3T_CUDA(cudaSetDevice(c->device));
        return check_status(c, stream ? static_cast<cudaStream_t>(stream) : c->stream);
    } S3T_CATCH_INT
}

// ---------------------------------------------------------- op level ---

int s3t_dequantize(int type, const void* src, int64_t n, float* dst, void* stream) {
    try {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (type == S3T_TYPE_Q8_0) {
            if (n % 32) return fail("Q8_0 length must be a multiple of 32");
            S3T_CUDA(launch_dequant_q8_0_to_f32(static_cast<const uint8_t*>(src), n, dst, st));
        } else if (type == S3T_TYPE_F16) {
            S3T_CUDA(launch_f16_to_f32(static_cast<const __half*>(src), n, dst, st));
        } else if (type == S3T_TYPE_F32) {
            S3T_CUDA(cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDeviceToDevice, st));
        } else {
            return fail("unsupported type");
        }
        return 0;
    } S3T_CATCH_INT
}

int s3t_weight_operand(int type, const void* src, int64_t n, void* dst16, void* stream) {
    try {
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        if (!src || !dst16 || n <= 0) return fail("weight_operand: null buffer or empty length");
        if (type == S3T_TYPE_Q8_0) {
            if (n % 32) return fail("Q8_0 length must be a multiple of 32");
            S3T_CUDA(launch_dequant_q8_0_to_f16(static_cast<const uint8_t*>(src), n, static_cast<__half*>(dst16), st));
        } else if (type == S3T_TYPE_F32) {
            S3T_CUDA(launch_f32_to_f16(static_cast<const float*>(src), n, static_cast<__half*>(dst16), st));
        } else if (type == S3T_TYPE_F16) {
            S3T_CUDA(cudaMemcpyAsync(dst16, src, size_t(n) * 2, cudaMemcpyDeviceToDevice, st));
        } else {
            return fail("unsupported type");
        }
        return 0;
    } S3T_CATCH_INT
}

int s3t_gemm_f16(int device, const void* x16, const void* w16, const float* bias, int M, int N, int K, int act, int q8,
                 void* y16, void* stream) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        S3T_CUDA(cudaSetDevice(device));
        if (K % 64 || N % 32 || M <= 0) return fail("gemm needs K % 64 == 0, N % 32 == 0, M > 0");
        GemmArgs g{};
        g.M = M; g.N = N; g.K = K;
        g.bias = bias;
        g.out16 = static_cast<__half*>(y16);
        g.gelu = act == 1;
        g.q8 = q8;
        g.status = ds->status;
        S3T_CUDA(launch_gemm(static_cast<const __half*>(x16), static_cast<const __half*>(w16), g, kEpiF16, ds->num_sms,
                             static_cast<cudaStream_t>(stream)));
        return 0;
    } S3T_CATCH_INT
}

int s3t_attention(int device, const void* q, const void* k, const void* v, int groups, int L, int windowed, int bf16,
                  void* out, void* stream) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        S3T_CUDA(cudaSetDevice(device));
        if (L % 64 || groups <= 0) return fail("attention needs L % 64 == 0 and groups > 0");
        if (windowed ? (L != kWindow * kWindow || groups % 9) : (L != kTokens))
            return fail("attention output mapping needs L = 576 (windowed, groups = 9*images) or 5184 (global)");
        AttnArgs a{};
        a.q = q; a.k = k; a.v = v;
        a.groups = groups; a.L = L; a.windowed = windowed;
        a.scale_log2 = 0.125f * 1.4426950408889634f;
        a.bf16 = bf16;
        a.out = out;
        a.status = ds->status;
        S3T_CUDA(launch_attention(a, static_cast<cudaStream_t>(stream)));
        return 0;
    } S3T_CATCH_INT
}

int s3t_mha_d32(int device, const void* q, const void* k, const void* v, int batch, int q_len, int kv_len,
                const float* key_mask, void* out, int flags, void* stream) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        S3T_CUDA(cudaSetDevice(device));
        if (!q || !k || !v || !out) return fail("mha_d32: q, k, v and out must be device pointers");
        if (batch <= 0 || q_len <= 0 || kv_len <= 0) return fail("mha_d32 needs batch, q_len and kv_len > 0");
        if (int64_t(batch) * (q_len + 127) / 128 * 8 > (int64_t(1) << 30)) return fail("mha_d32: batch * q_len too large");
        if (flags & ~(S3T_MHA_BF16 | S3T_MHA_OUT_F16 | S3T_MHA_BIAS)) return fail("mha_d32: unknown flags");
        if ((flags & S3T_MHA_BIAS) && !key_mask) return fail("mha_d32: S3T_MHA_BIAS needs the bias array");
        if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
             reinterpret_cast<uintptr_t>(out)) & 15)
            return fail("mha_d32: q, k, v and out must be 16-byte aligned");
        MhaArgs a{};
        a.q = q; a.k = k; a.v = v;
        a.key_mask = key_mask;
        a.batch = batch;
        a.q_len = q_len; a.kv_len = kv_len;
        // The reference's scale, 1.0f / std::sqrt(float(kHeadDim)), in the log2 domain.
        a.scale_log2 = (1.0f / std::sqrt(32.0f)) * 1.4426950408889634f;
        a.bf16 = (flags & S3T_MHA_BF16) != 0;
        a.out_f16 = (flags & S3T_MHA_OUT_F16) != 0;
        a.bias = (flags & S3T_MHA_BIAS) != 0;
        a.out = out;
        a.status = ds->status;
        S3T_CUDA(launch_mha32(a, static_cast<cudaStream_t>(stream)));
        return 0;
    } S3T_CATCH_INT
}

int s3t_rope(int device, void* x, int groups, int L, int windowed, int bf16, void* stream) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        S3T_CUDA(cudaSetDevice(device));
        S3T_CUDA(launch_rope_inplace(x, groups, L, windowed, bf16, ds->rope_local, ds->rope_global,
                                     static_cast<cudaStream_t>(stream)));
        return 0;
    } S3T_CATCH_INT
}

int s3t_layernorm(int device, const float* x, int rows, const float* gamma, const float* beta, void* y16, int q8,
                  void* stream) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        S3T_CUDA(cudaSetDevice(device));
        S3T_CUDA(launch_layernorm(x, rows, gamma, beta, static_cast<__half*>(y16), q8, static_cast<cudaStream_t>(stream)));
        return 0;
    } S3T_CATCH_INT
}

int s3t_preprocess_rgb8(int device, const uint8_t* rgb, int width, int height, int batch, float* out, void* stream) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        if (!rgb || !out) return fail("rgb or out is null");
        if (batch <= 0 || batch > 65535) return fail("batch must be in [1, 65535]");
        if (width <= 0 || height <= 0 || width > kMaxSourceSide || height > kMaxSourceSide)
            return fail("image width and height must be in [1, 32768]");
        S3T_CUDA(cudaSetDevice(device));
        S3T_CUDA(launch_resize_rgb8(rgb, width, height, batch, out, static_cast<cudaStream_t>(stream)));
        return 0;
    } S3T_CATCH_INT
}

int s3t_selftest_wait_timeout(int device, int limit_ms) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        if (limit_ms < 1 || limit_ms > 2000) return fail("limit_ms must be in [1, 2000]");
        S3T_CUDA(cudaSetDevice(device));
        int* gave_up = nullptr;
        S3T_CUDA(cudaMalloc(&gave_up, sizeof(int)));
        S3T_CUDA(cudaMemset(gave_up, 0, sizeof(int)));
        cudaError_t e = launch_wait_timeout_probe(ds->status, uint64_t(limit_ms) * 1000000ull, gave_up, nullptr);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        int h = 0;
        if (e == cudaSuccess) e = cudaMemcpy(&h, gave_up, sizeof(int), cudaMemcpyDeviceToHost);
        cudaFree(gave_up);
        S3T_CUDA(e);
        if (!h) return fail("self-test: the bounded wait did not give up");
        return 0;   // the timeout is now in the device status word (s3t_device_status reports it)
    } S3T_CATCH_INT
}

int s3t_device_status(int device) {
    try {
        DeviceState* ds = nullptr;
        if (device_state(device, &ds)) return -1;
        S3T_CUDA(cudaSetDevice(device));
        S3T_CUDA(cudaDeviceSynchronize());
        int code = 0;
        S3T_CUDA(cudaMemcpy(&code, ds->status, sizeof(int), cudaMemcpyDeviceToHost));
        S3T_CUDA(cudaMemset(ds->status, 0, sizeof(int)));
        if (code) return fail(std::string("device error: ") + status_message(code));
        return 0;
    } S3T_CATCH_INT
}

}  // extern "C"
