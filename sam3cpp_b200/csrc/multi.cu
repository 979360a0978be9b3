// Several GPUs of one node behind one handle: s3t_multi_* (include/s3t.h).
//
// The trunk is per image (src/vision_trunk.cpp:301 takes one image; nothing
// couples two images), so a batch is split into contiguous shards, one per
// GPU, each GPU holding its own copy of the weights in its own s3t_ctx.  One
// host thread drives each GPU.  The only exchange is moving images in and
// feature maps out:
//
// * host buffers: every GPU copies its own slice of the host images in and
//   its own slice of the features out (the context's chunked host pipeline
//   overlaps those copies with compute), so nothing is gathered on a device;
// * device buffers on the first GPU (S3T_IMAGES_ON_DEVICE /
//   S3T_OUTPUT_ON_DEVICE): the first GPU computes its shard in place on the
//   caller's stream; every other GPU works through its shard in chunks of
//   kChunk images with two staging buffers, so the peer copy of chunk k's
//   features into the first GPU's output (and of chunk k+2's images in)
//   overlaps the trunk on chunk k+1.  The other GPUs start after the work
//   already queued on the caller's stream (an event), and the caller's
//   stream waits for their last copies (events), so the call is asynchronous
//   like s3t_trunk_run with device buffers.  Copies are plain
//   cudaMemcpyPeerAsync over NVLink; no kernel reads another GPU's memory.
#include "s3t.h"
#include "kernels.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <exception>
#include <string>
#include <thread>
#include <vector>

using namespace s3t;

namespace {

constexpr int kChunk = 4;   // images per staged chunk on the GPUs that are not the first

struct Staging {
    float* in[2] = {nullptr, nullptr};
    float* out[2] = {nullptr, nullptr};
    cudaEvent_t computed[2] = {nullptr, nullptr};   // trunk of the chunk in buffer b finished
    cudaEvent_t drained[2] = {nullptr, nullptr};    // buffer b's features copied out
    cudaStream_t copy = nullptr;
    cudaStream_t compute = nullptr;
    cudaEvent_t finished = nullptr;                 // this GPU's last copy of a run
};

std::string cuda_msg(const char* what, cudaError_t e) { return std::string(what) + ": " + cudaGetErrorString(e); }

}  // namespace

struct s3t_multi {
    std::vector<int> devices;
    std::vector<s3t_ctx*> ctx;
    std::vector<Staging> stage;   // index 0 unused (the first GPU needs no staging)
    cudaEvent_t start = nullptr;  // on the first GPU: the caller's queued work before a run
};

namespace {

void free_staging(int device, Staging& s) {
    cudaSetDevice(device);
    for (int b = 0; b < 2; ++b) {
        if (s.in[b]) cudaFree(s.in[b]);
        if (s.out[b]) cudaFree(s.out[b]);
        if (s.computed[b]) cudaEventDestroy(s.computed[b]);
        if (s.drained[b]) cudaEventDestroy(s.drained[b]);
    }
    if (s.copy) cudaStreamDestroy(s.copy);
    if (s.compute) cudaStreamDestroy(s.compute);
    if (s.finished) cudaEventDestroy(s.finished);
    s = Staging{};
}

std::string make_staging(int device, Staging& s) {
    cudaError_t e = cudaSetDevice(device);
    const size_t in_bytes = size_t(kChunk) * 3 * kImage * kImage * 4, out_bytes = size_t(kChunk) * kDim * kTokens * 4;
    for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
        void* p = nullptr;
        if ((e = cudaMalloc(&p, in_bytes)) != cudaSuccess) break;
        s.in[b] = static_cast<float*>(p);
        if ((e = cudaMalloc(&p, out_bytes)) != cudaSuccess) break;
        s.out[b] = static_cast<float*>(p);
        if ((e = cudaEventCreateWithFlags(&s.computed[b], cudaEventDisableTiming)) != cudaSuccess) break;
        e = cudaEventCreateWithFlags(&s.drained[b], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.copy, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.compute, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.finished, cudaEventDisableTiming);
    if (e != cudaSuccess) {
        free_staging(device, s);
        return cuda_msg("staging buffers", e);
    }
    return {};
}

// Shard of GPU k (k >= 1) through its staging buffers, enqueued after
// `start` (an event of the first GPU); s.finished is recorded after the last
// copy.  images / out point at this shard's first image; images_dev /
// out_dev say whether they are memory of the first GPU (dev0) or host memory.
std::string run_staged(s3t_ctx* ctx, int device, int dev0, Staging& s, cudaEvent_t start, const float* images, int n,
                       float* out, bool images_dev, bool out_dev) {
    const size_t img_elems = size_t(3) * kImage * kImage, out_elems = size_t(kDim) * kTokens;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_msg("cudaSetDevice", e);
    if ((e = cudaStreamWaitEvent(s.compute, start, 0)) != cudaSuccess) return cuda_msg("cudaStreamWaitEvent", e);
    if ((e = cudaStreamWaitEvent(s.copy, start, 0)) != cudaSuccess) return cuda_msg("cudaStreamWaitEvent", e);
    const int chunks = (n + kChunk - 1) / kChunk;
    for (int k = 0; k < chunks; ++k) {
        const int b = k & 1, i0 = k * kChunk, nb = std::min(kChunk, n - i0);
        // buffer b's previous features must have left before the trunk overwrites them
        if (k >= 2 && (e = cudaStreamWaitEvent(s.compute, s.drained[b], 0)) != cudaSuccess)
            return cuda_msg("cudaStreamWaitEvent", e);
        const float* src = images + i0 * img_elems;
        e = images_dev ? cudaMemcpyPeerAsync(s.in[b], device, src, dev0, nb * img_elems * 4, s.compute)
                       : cudaMemcpyAsync(s.in[b], src, nb * img_elems * 4, cudaMemcpyHostToDevice, s.compute);
        if (e != cudaSuccess) return cuda_msg("image copy", e);
        if (s3t_trunk_run(ctx, s.in[b], nb, s.out[b], S3T_IMAGES_ON_DEVICE | S3T_OUTPUT_ON_DEVICE, s.compute))
            return s3t_last_error();
        if ((e = cudaEventRecord(s.computed[b], s.compute)) != cudaSuccess) return cuda_msg("cudaEventRecord", e);
        if ((e = cudaStreamWaitEvent(s.copy, s.computed[b], 0)) != cudaSuccess) return cuda_msg("cudaStreamWaitEvent", e);
        float* dst = out + i0 * out_elems;
        e = out_dev ? cudaMemcpyPeerAsync(dst, dev0, s.out[b], device, nb * out_elems * 4, s.copy)
                    : cudaMemcpyAsync(dst, s.out[b], nb * out_elems * 4, cudaMemcpyDeviceToHost, s.copy);
        if (e != cudaSuccess) return cuda_msg("feature copy", e);
        if ((e = cudaEventRecord(s.drained[b], s.copy)) != cudaSuccess) return cuda_msg("cudaEventRecord", e);
    }
    if ((e = cudaEventRecord(s.finished, s.copy)) != cudaSuccess) return cuda_msg("cudaEventRecord", e);
    return {};
}

// Runs fn(k) for every GPU k on its own host thread; returns the first error.
template <typename F>
std::string on_every_gpu(size_t n, F fn) {
    std::vector<std::string> err(n);
    std::vector<std::thread> th;
    for (size_t k = 0; k < n; ++k)
        th.emplace_back([&, k] {
            try {
                err[k] = fn(k);
            } catch (const std::exception& ex) {
                err[k] = std::string("internal error: ") + ex.what();
            } catch (...) {
                err[k] = "internal error";
            }
        });
    for (auto& t : th) t.join();
    for (size_t k = 0; k < n; ++k)
        if (!err[k].empty()) return "GPU " + std::to_string(k) + ": " + err[k];
    return {};
}

}  // namespace

extern "C" {

s3t_multi* s3t_multi_create(const int* devices, int n_devices, const char* gguf_path, const char* tensor_map_path) {
    try {
        if (!devices || n_devices < 1 || !gguf_path) {
            set_last_error("s3t_multi_create: need 1 or more devices and a GGUF path");
            return nullptr;
        }
        for (int i = 0; i < n_devices; ++i)
            for (int j = 0; j < i; ++j)
                if (devices[i] == devices[j]) {
                    set_last_error(("s3t_multi_create: device " + std::to_string(devices[i]) + " listed twice").c_str());
                    return nullptr;
                }
        s3t_multi* m = new s3t_multi();
        m->devices.assign(devices, devices + n_devices);
        m->ctx.assign(n_devices, nullptr);
        m->stage.resize(n_devices);
        std::string err = on_every_gpu(n_devices, [&](size_t k) -> std::string {
            s3t_ctx* c = s3t_create(m->devices[k]);
            if (!c) return s3t_last_error();
            m->ctx[k] = c;
            if (s3t_load_gguf(c, gguf_path, tensor_map_path) || s3t_finalize_weights(c)) return s3t_last_error();
            if (k > 0) {
                // Peer access both ways where the topology allows it (NVLink);
                // cudaMemcpyPeerAsync also works without it.
                int can = 0;
                if (cudaDeviceCanAccessPeer(&can, m->devices[k], m->devices[0]) == cudaSuccess && can) {
                    cudaSetDevice(m->devices[k]);
                    if (cudaDeviceEnablePeerAccess(m->devices[0], 0) != cudaSuccess) cudaGetLastError();
                }
                return make_staging(m->devices[k], m->stage[k]);
            }
            return {};
        });
        if (err.empty() && (cudaSetDevice(m->devices[0]) != cudaSuccess ||
                            cudaEventCreateWithFlags(&m->start, cudaEventDisableTiming) != cudaSuccess))
            err = "s3t_multi_create: event creation failed";
        if (err.empty()) {
            for (int k = 1; k < n_devices; ++k) {
                int can = 0;
                if (cudaDeviceCanAccessPeer(&can, m->devices[0], m->devices[k]) == cudaSuccess && can &&
                    cudaDeviceEnablePeerAccess(m->devices[k], 0) != cudaSuccess)
                    cudaGetLastError();
            }
        }
        if (!err.empty()) {
            s3t_multi_destroy(m);
            set_last_error(err.c_str());
            return nullptr;
        }
        return m;
    } catch (...) {
        set_last_error("s3t_multi_create: internal error");
        return nullptr;
    }
}

void s3t_multi_destroy(s3t_multi* m) {
    if (!m) return;
    try {
        for (size_t k = 0; k < m->devices.size(); ++k) {
            if (k > 0) {
                cudaSetDevice(m->devices[k]);
                if (m->stage[k].copy) cudaStreamSynchronize(m->stage[k].copy);
                if (m->stage[k].compute) cudaStreamSynchronize(m->stage[k].compute);
                free_staging(m->devices[k], m->stage[k]);
            }
            if (m->ctx[k]) s3t_destroy(m->ctx[k]);
        }
        if (m->start) {
            cudaSetDevice(m->devices[0]);
            cudaEventDestroy(m->start);
        }
        delete m;
    } catch (...) {
    }
}

int s3t_multi_num_devices(const s3t_multi* m) { return m ? int(m->devices.size()) : 0; }

int s3t_multi_run(s3t_multi* m, const float* images, int batch, float* out, int flags, void* stream) {
    try {
        if (!m) return set_last_error("s3t_multi_run: handle is null");
        if (!images || !out) return set_last_error("s3t_multi_run: images or out is null");
        if (batch <= 0) return set_last_error("s3t_multi_run: batch must be positive");
        if (flags & ~(S3T_IMAGES_ON_DEVICE | S3T_OUTPUT_ON_DEVICE)) return set_last_error("s3t_multi_run: unknown flags");
        const bool in_dev = flags & S3T_IMAGES_ON_DEVICE, out_dev = flags & S3T_OUTPUT_ON_DEVICE;
        const size_t n = m->devices.size();
        const int per = int((size_t(batch) + n - 1) / n);
        const size_t img_elems = size_t(3) * kImage * kImage, out_elems = size_t(kDim) * kTokens;
        const int dev0 = m->devices[0];
        cudaStream_t st0 = stream ? static_cast<cudaStream_t>(stream) : ctx_stream(m->ctx[0]);
        if (!in_dev && !out_dev) {
            // Host buffers: every GPU copies its own slices (its context
            // pipelines the host copies with compute); synchronous.
            const std::string err = on_every_gpu(n, [&](size_t k) -> std::string {
                const int i0 = int(k) * per, nb = std::min(per, batch - i0);
                if (nb <= 0) return {};
                cudaStream_t st = k ? nullptr : st0;
                if (s3t_trunk_run(m->ctx[k], images + i0 * img_elems, nb, out + i0 * out_elems, 0, st) ||
                    s3t_sync(m->ctx[k], st))
                    return s3t_last_error();
                return {};
            });
            return err.empty() ? 0 : set_last_error(err.c_str());
        }
        cudaError_t e = cudaSetDevice(dev0);
        if (e == cudaSuccess) e = cudaEventRecord(m->start, st0);
        if (e != cudaSuccess) return set_last_error(cuda_msg("s3t_multi_run", e).c_str());
        std::vector<char> used(n, 0);
        const std::string err = on_every_gpu(n, [&](size_t k) -> std::string {
            const int i0 = int(k) * per, nb = std::min(per, batch - i0);
            if (nb <= 0) return {};
            used[k] = 1;
            const float* src = images + i0 * img_elems;
            float* dst = out + i0 * out_elems;
            if (k == 0) {
                // The first GPU works on its shard in place, on the caller's stream.
                if (s3t_trunk_run(m->ctx[0], src, nb, dst, flags, st0)) return s3t_last_error();
                return {};
            }
            return run_staged(m->ctx[k], m->devices[k], dev0, m->stage[k], m->start, src, nb, dst, in_dev, out_dev);
        });
        if (!err.empty()) return set_last_error(err.c_str());
        // The caller's stream waits for every other GPU's last copy.
        if ((e = cudaSetDevice(dev0)) != cudaSuccess) return set_last_error(cuda_msg("s3t_multi_run", e).c_str());
        for (size_t k = 1; k < n; ++k)
            if (used[k] && (e = cudaStreamWaitEvent(st0, m->stage[k].finished, 0)) != cudaSuccess)
                return set_last_error(cuda_msg("cudaStreamWaitEvent", e).c_str());
        return 0;
    } catch (...) {
        return set_last_error("s3t_multi_run: internal error");
    }
}

int s3t_multi_sync(s3t_multi* m, void* stream) {
    try {
        if (!m) return set_last_error("s3t_multi_sync: handle is null");
        const std::string err = on_every_gpu(m->devices.size(), [&](size_t k) -> std::string {
            if (k > 0) {
                cudaError_t e = cudaSetDevice(m->devices[k]);
                if (e == cudaSuccess) e = cudaStreamSynchronize(m->stage[k].copy);
                if (e != cudaSuccess) return cuda_msg("cudaStreamSynchronize", e);
            }
            return s3t_sync(m->ctx[k], k ? m->stage[k].compute : stream) ? std::string(s3t_last_error())
                                                                          : std::string();
        });
        return err.empty() ? 0 : set_last_error(err.c_str());
    } catch (...) {
        return set_last_error("s3t_multi_sync: internal error");
    }
}

}  // extern "C"
