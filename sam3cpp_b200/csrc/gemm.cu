// Persistent, warp-specialized tcgen05 GEMM for the trunk's linears:
//   C[M,N] = A[M,K] * B[N,K]^T,  A = activations fp16, B = weights fp16,
// fp32 accumulation in TMEM, operands staged by TMA (128-byte swizzle) in a
// STAGES-deep mbarrier ring, accumulators double-buffered in TMEM so the
// epilogue of tile i overlaps the mainloop of tile i+1.
//
// Roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + UMMA
// issuer, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
//
// The epilogues fuse what the reference runs as separate ggml ops after each
// mul_mat (src/vision_trunk.cpp:50-62 linear + bias, :451 gelu_erf, :439/:458
// residual adds, :417-425 RoPE, :364-374 patch-embed + abs-pos, :461 NCHW
// permute) and the activation rounding ggml's CPU mul_mat applies to the next
// GEMM's input (fp16 for F16 weights, Q8_0 blocks for Q8_0 weights).
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_runtime.h>
#include <stdio.h>

namespace s3t {

namespace {

constexpr int kBM = 128, kBK = 64;

template <int BN>
struct GemmCfg {
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr uint32_t A_BYTES = kBM * kBK * 2;
    static constexpr uint32_t B_BYTES = BN * kBK * 2;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr size_t SMEM = size_t(STAGES) * (A_BYTES + B_BYTES) + 1024 + 256;
};

__device__ __forceinline__ void load_bias32(const float* bias, int n, float (&b)[32]) {
    if (bias) {
        const float4* p = reinterpret_cast<const float4*>(bias + n);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float4 t = __ldg(p + i);
            b[4 * i] = t.x; b[4 * i + 1] = t.y; b[4 * i + 2] = t.z; b[4 * i + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) b[i] = 0.f;
    }
}

__device__ __forceinline__ void store_half32(__half* dst, const float (&v)[32]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 u;
        u.x = pack_half2(v[8 * i + 0], v[8 * i + 1]);
        u.y = pack_half2(v[8 * i + 2], v[8 * i + 3]);
        u.z = pack_half2(v[8 * i + 4], v[8 * i + 5]);
        u.w = pack_half2(v[8 * i + 6], v[8 * i + 7]);
        d[i] = u;
    }
}

// Bias, GELU and Q8_0 rounding of one 32-column chunk, packed to fp16 pairs.
__device__ __forceinline__ void f16_chunk(const GemmArgs& a, int n, const uint32_t (&r)[32], uint32_t (&pk)[16]) {
    float2 v[16];
    if (a.bias) {
        const float4* p = reinterpret_cast<const float4*>(a.bias + n);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = __ldg(p + i);
            v[2 * i] = __fadd2_rn(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])),
                                  make_float2(b.x, b.y));
            v[2 * i + 1] = __fadd2_rn(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])),
                                      make_float2(b.z, b.w));
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    }
    if (a.gelu) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = gelu_erf_as2(v[i]);
    }
    if (a.q8) {
        float f[32];
#pragma unroll
        for (int i = 0; i < 16; ++i) { f[2 * i] = v[i].x; f[2 * i + 1] = v[i].y; }
        q8_0_fake_quant32(f);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = make_float2(f[2 * i], f[2 * i + 1]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_half2(v[i].x, v[i].y);
}

// Token m of the QKV GEMM: its (window or image) group g and index i in that
// group, and its RoPE row/column positions.
struct QkvPos {
    int g, i, px, py;
};

__device__ __forceinline__ QkvPos qkv_pos(int m, int windowed) {
    const int img = m / kTokens, t = m - img * kTokens;
    const int y = t / kGrid, x = t - y * kGrid;
    QkvPos p;
    if (windowed) {
        p.g = img * 9 + (y / kWindow) * 3 + (x / kWindow);
        p.py = y % kWindow;
        p.px = x % kWindow;
        p.i = p.py * kWindow + p.px;
    } else {
        p.g = img;
        p.i = t;
        p.px = x;
        p.py = y;
    }
    return p;
}

// Bias and axial RoPE (q and k; columns n..n+31 are one half of a head) of one
// 32-column chunk of row m, packed to fp16 pairs.
__device__ __forceinline__ void qkv_chunk(const GemmArgs& a, int m, int n, const uint32_t (&r)[32],
                                          uint32_t (&pk)[16]) {
    float2 v[16];
    {
        const float4* p = reinterpret_cast<const float4*>(a.bias + n);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = __ldg(p + i);
            v[2 * i] = __fadd2_rn(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])),
                                  make_float2(b.x, b.y));
            v[2 * i + 1] = __fadd2_rn(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])),
                                      make_float2(b.z, b.w));
        }
    }
    if ((n >> 10) < 2) {
        const QkvPos p = qkv_pos(m, a.windowed);
        const int half = (n >> 5) & 1;
        float c[16], s[16];
        if (half) {
            // y position: the same for (nearly) every row of a warp, so the
            // row-major table is read as broadcasts
            const float* tab = a.windowed ? a.rope_local : a.rope_global;
            const float4* cs = reinterpret_cast<const float4*>(tab + p.py * 32);   // [pos][cos16 | sin16]
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 c4 = __ldg(cs + q), s4 = __ldg(cs + 4 + q);
                c[4 * q] = c4.x; c[4 * q + 1] = c4.y; c[4 * q + 2] = c4.z; c[4 * q + 3] = c4.w;
                s[4 * q] = s4.x; s[4 * q + 1] = s4.y; s[4 * q + 2] = s4.z; s[4 * q + 3] = s4.w;
            }
        } else {
            // x position: consecutive rows of a warp have consecutive positions,
            // so the transposed table gives one contiguous 4-byte load per lane
            const float* tt = a.windowed ? a.rope_local_t : a.rope_global_t;
            const int P = a.windowed ? kWindow : kGrid;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                c[j] = __ldg(tt + j * P + p.px);
                s[j] = __ldg(tt + (16 + j) * P + p.px);
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // (x0, x1) -> (x0 c - x1 s, x0 s + x1 c)
            v[j] = __ffma2_rn(make_float2(v[j].x, v[j].x), make_float2(c[j], s[j]),
                              __fmul2_rn(make_float2(v[j].y, v[j].y), make_float2(-s[j], c[j])));
        }
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_half2(v[i].x, v[i].y);
}

template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, int m, int n, const uint32_t (&r)[32]) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);

    if constexpr (EPI == kEpiF16) {
        float b[32];
        load_bias32(a.bias, n, b);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += b[i];
        if (a.gelu) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = gelu_erf_as(v[i]);
        }
        if (a.q8) q8_0_fake_quant32(v);
        store_half32(a.out16 + int64_t(m) * a.N + n, v);
    } else if constexpr (EPI == kEpiQkv) {
        float b[32];
        load_bias32(a.bias, n, b);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += b[i];
        const int img = m / kTokens, t = m - img * kTokens;
        const int y = t / kGrid, x = t - y * kGrid;
        const int which = n >> 10, head = (n & 1023) >> 6, half = (n >> 5) & 1;
        int g, i, L, px, py;
        const float* tab;
        if (a.windowed) {
            g = img * 9 + (y / kWindow) * 3 + (x / kWindow);
            py = y % kWindow; px = x % kWindow;
            i = py * kWindow + px;
            L = kWindow * kWindow;
            tab = a.rope_local;
        } else {
            g = img; i = t; L = kTokens; px = x; py = y;
            tab = a.rope_global;
        }
        if (which < 2) {
            const float4* cs = reinterpret_cast<const float4*>(tab + (half ? py : px) * 32);   // [pos][cos16 | sin16]
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 c4 = __ldg(cs + q), s4 = __ldg(cs + 4 + q);
                const float c[4] = {c4.x, c4.y, c4.z, c4.w}, s[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = 4 * q + u;
                    const float x0 = v[2 * j], x1 = v[2 * j + 1];
                    v[2 * j] = x0 * c[u] - x1 * s[u];
                    v[2 * j + 1] = x0 * s[u] + x1 * c[u];
                }
            }
        }
        __half* dst = a.qkv + which * a.qkv_stride + (int64_t(g * kHeads + head) * L + i) * kHeadDim + half * 32;
        store_half32(dst, v);
    } else if constexpr (EPI == kEpiResid) {
        float b[32];
        load_bias32(a.bias, n, b);
        float4* xr = reinterpret_cast<float4*>(a.resid + int64_t(m) * a.N + n);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            float4 t = xr[q];
            t.x = t.x + (v[4 * q + 0] + b[4 * q + 0]);
            t.y = t.y + (v[4 * q + 1] + b[4 * q + 1]);
            t.z = t.z + (v[4 * q + 2] + b[4 * q + 2]);
            t.w = t.w + (v[4 * q + 3] + b[4 * q + 3]);
            xr[q] = t;
            v[4 * q + 0] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
        }
        if (a.out_nchw) {
            const int img = m / kTokens, t = m - img * kTokens;
            float* o = a.out_nchw + (int64_t(img) * a.N + n) * kTokens + t;
#pragma unroll
            for (int i = 0; i < 32; ++i) o[int64_t(i) * kTokens] = v[i];
        }
    } else {  // kEpiPatch
        const int t = m % kTokens;
        const int y = t / kGrid, x = t - y * kGrid;
        const float4* p = reinterpret_cast<const float4*>(a.pos + int64_t(1 + (y % 24) * 24 + (x % 24)) * kDim + n);
        float4* xr = reinterpret_cast<float4*>(a.resid + int64_t(m) * a.N + n);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 pp = __ldg(p + q);
            xr[q] = make_float4(v[4 * q] + pp.x, v[4 * q + 1] + pp.y, v[4 * q + 2] + pp.z, v[4 * q + 3] + pp.w);
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmArgs args) {
    using Cfg = GemmCfg<BN>;
    constexpr int STAGES = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles_n = (args.N + BN - 1) / BN;
    const int n_tiles = ((args.M + kBM - 1) / kBM) * n_tiles_n;
    const int num_kb = args.K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(tfull + i, 1);
            mbar_init(tempty + i, 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t armed = 0, armed_parity = 0;  // per-stage: armed at least once / parity of last arm
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int m0 = (tile / n_tiles_n) * kBM, n0 = (tile % n_tiles_n) * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(empty + s, ph ^ 1, args.status, kErrTimeoutProducer, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full + s, Cfg::A_BYTES + Cfg::B_BYTES);
                    tma_load_2d(sA + s * Cfg::A_BYTES, &tmA, full + s, kb * kBK, m0);
                    tma_load_2d(sB + s * Cfg::B_BYTES, &tmB, full + s, kb * kBK, n0);
                    armed |= 1u << s;
                    armed_parity = (armed_parity & ~(1u << s)) | (ph << s);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            if (!ok) {
                // Gave up: wait (bounded) for the copies this thread started.
                for (int i = 0; i < STAGES; ++i)
                    if (armed & (1u << i))
                        mbar_wait(full + i, (armed_parity >> i) & 1u, args.status, kErrTimeoutDrain, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(kBM, BN, 0, 0);
            int s = 0;
            uint32_t ph = 0;
            bool ok = true, issued = false;
            int local = 0;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(tempty + acc, aph ^ 1, args.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full + s, ph, args.status, kErrTimeoutMma, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        umma_f16_ss(d_tmem, umma_desc_sw128(a0 + k * 32, 16, 1024), umma_desc_sw128(b0 + k * 32, 16, 1024),
                                    idesc, (kb | k) != 0);
                    }
                    issued = true;
                    umma_commit(empty + s);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(tfull + acc);
            }
            if (!ok && issued) {
                umma_commit(drain);
                mbar_wait(drain, 0, args.status, kErrTimeoutDrain, nullptr);
            }
        }
    } else {
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        int local = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            if (!mbar_wait(tfull + acc, aph, args.status, kErrTimeoutEpilogue, abort_flag)) break;
            tc_fence_after();
            const int m0 = (tile / n_tiles_n) * kBM, n0 = (tile % n_tiles_n) * BN;
            const int m = m0 + row;
            const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + acc * BN;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                const int n = n0 + c * 32;
                if (n >= args.N) break;
                uint32_t r[32];
                tmem_ld32(tbase + c * 32, r);
                tmem_wait_ld();
                if (m < args.M) epilogue_chunk<EPI>(args, m, n, r);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty + acc);
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// Two-SM version: a CTA pair (cluster of 2) owns a 256 x 256 output tile
// (320 threads per CTA: producer warp, MMA warp, 8 epilogue warps).
// CTA r stages rows [128r, 128r+128) of the A tile and rows [128r, 128r+128)
// of the B tile (half of N); the leader (rank 0) issues
// tcgen05.mma.cta_group::2 (M=256, N=256), which reads both CTAs' halves and
// leaves rows [128r, +128) x 256 of the accumulator in CTA r's TMEM.  Each
// UMMA therefore reads 8 KB of a CTA's shared memory per 128 x 256 x 16 of
// work instead of 12 KB.  Loads of both CTAs complete on the leader's full
// barrier; the leader's commits arrive on both CTAs' barriers (multicast
// commit); both CTAs' epilogue warps release an accumulator buffer on the
// leader's barrier.  No TMA load uses cluster multicast.
//
// The epilogue warps sit on the same SM sub-partitions as the single
// producer and UMMA threads, so every instruction they issue can delay the
// mainloop: the UMMA loop uses descriptors built once, the fp32 epilogue
// math runs as packed f32x2 operations (two columns per instruction), and the
// outputs (fp16 for kEpiF16 / kEpiQkv, the fp32 residual for kEpiResid) leave
// through shared memory and one TMA store per 32 x 32 chunk instead of 32
// scattered row stores.
template <int BK_, int RBUF_ = 1>
struct PairCfgT {
    static constexpr int BN = 256;
    // A stage holds BK K-columns as 64-column (128-byte) swizzle atoms.  With
    // BK = 128 the lone UMMA thread waits, issues and commits once per 8
    // UMMAs (K = 1024 GEMMs); the long-K fc2 keeps 64-column stages, 6 deep.
    static constexpr int BK = BK_;
    static constexpr int STAGES = BK_ == 128 ? 3 : 6;
    static constexpr uint32_t ATOM_A = kBM * 64 * 2;            // 128 rows x 64 K-columns
    static constexpr uint32_t ATOM_B = (BN / 2) * 64 * 2;
    static constexpr uint32_t A_BYTES = ATOM_A * (BK / 64);     // this CTA's 128 rows of A
    static constexpr uint32_t B_BYTES = ATOM_B * (BK / 64);     // this CTA's 128 rows of B
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr int EPI_WARPS = 8;
    static constexpr int COL_GROUPS = EPI_WARPS / 4;            // warps per TMEM lane quarter
    static constexpr int WARP_COLS = BN / COL_GROUPS;           // accumulator columns per warp
    // kEpiF16 stages each 32x32 output chunk in shared memory (2 KB buffers,
    // 64-byte swizzle) and stores it with TMA.
    static constexpr int OUT_BUFS = EPI_WARPS <= 8 ? 2 : 1;
    __host__ __device__ static constexpr bool staged_out(int EPI) {
        return EPI == kEpiF16 || EPI == kEpiQkv || EPI == kEpiResid;
    }
    static constexpr uint32_t OUT_BYTES = OUT_BUFS * 2048;
    // The residual epilogue (kEpiResid, 64-column stages) keeps RBUF 32 x 32
    // fp32 chunks per warp in flight.  Two (proj: its epilogue is as long as
    // its K = 1024 mainloop, and exposed at one or two images) cost 32 KB,
    // paid for with a 5-deep ring; the long-K fc2 keeps one and 6 stages.
    static constexpr uint32_t kResidBuf = 32 * 32 * 4;
    __host__ __device__ static constexpr int stages(int EPI) {
        return EPI == kEpiResid && RBUF_ == 2 ? 5 : STAGES;
    }
    __host__ __device__ static constexpr uint32_t out_bytes(int EPI) {
        return EPI == kEpiResid ? RBUF_ * kResidBuf : (staged_out(EPI) ? OUT_BYTES : 0);
    }
    template <int EPI>
    static constexpr size_t smem() {
        return size_t(stages(EPI)) * (A_BYTES + B_BYTES) + EPI_WARPS * out_bytes(EPI) + 1024 + 512;
    }
    static constexpr int THREADS = 64 + 32 * EPI_WARPS;
};
using PairCfg = PairCfgT<128>;

// The work of one CTA pair, as segments of (tile, K blocks [k0, k1)).
// Whole tiles: tile = pair, pair + n_pairs, ... with all K blocks.  Stream-K
// (SK): the n_tiles x num_kb K-block units split into one contiguous range
// per pair, each at least num_kb long, so a tile is shared by at most two
// pairs.  A pair walks its range as: the head of the tile its range ends in
// (K blocks [0, k1): kSegOut, first), its whole tiles, then the tail of the
// tile its range starts in ([k0, num_kb): kSegIn, last).  The kSegOut
// epilogue writes the raw accumulator to the pair's workspace slot and
// raises one flag per epilogue warp; before the kSegIn mainloop, the
// epilogue warps wait for the previous pair's flags and load that
// accumulator into tensor memory, and the UMMAs continue on it.  Every
// output is therefore the same sequential K accumulation as an unsplit
// tile: results do not depend on stream-K, the batch or the timing.
enum : int { kSegFull = 0, kSegOut = 1, kSegIn = 2 };
struct Seg {
    int tile, k0, k1, role;
};
struct SegWalk {
    int num_kb, t, t_end, stride;
    int head_tile, head_k1, tail_tile, tail_k0;
    int phase;
    __device__ SegWalk(int pair, int n_pairs, int n_tiles, int num_kb_, bool sk) : num_kb(num_kb_) {
        if (!sk) {
            t = pair; t_end = n_tiles; stride = n_pairs;
            head_tile = tail_tile = -1;
            head_k1 = tail_k0 = 0;
            phase = 1;
            return;
        }
        const int64_t units = int64_t(n_tiles) * num_kb;
        const int u0 = int(units * pair / n_pairs), u1 = int(units * (pair + 1) / n_pairs);
        head_k1 = u1 % num_kb;
        head_tile = head_k1 ? u1 / num_kb : -1;
        tail_k0 = u0 % num_kb;
        tail_tile = tail_k0 ? u0 / num_kb : -1;
        t = (u0 + num_kb - 1) / num_kb;
        t_end = u1 / num_kb;
        stride = 1;
        phase = 0;
    }
    __device__ bool next(Seg& g) {
        if (phase == 0) {
            phase = 1;
            if (head_tile >= 0) {
                g.tile = head_tile; g.k0 = 0; g.k1 = head_k1; g.role = kSegOut;
                return true;
            }
        }
        if (phase == 1) {
            if (t < t_end) {
                g.tile = t; g.k0 = 0; g.k1 = num_kb; g.role = kSegFull;
                t += stride;
                return true;
            }
            phase = 2;
        }
        if (phase == 2) {
            phase = 3;
            if (tail_tile >= 0) {
                g.tile = tail_tile; g.k0 = tail_k0; g.k1 = num_kb; g.role = kSegIn;
                return true;
            }
        }
        return false;
    }
};

template <int EPI, int BK, bool SK, int RB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfgT<BK, RB>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
    using Cfg = PairCfgT<BK, RB>;
    static_assert(RB == 1 || (EPI == kEpiResid && BK == 64), "two residual buffers fit beside 64-column stages only");
    constexpr int STAGES = Cfg::stages(EPI), BN = Cfg::BN;
    constexpr uint32_t OUTB = Cfg::out_bytes(EPI);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
    uint8_t* sOut = sB + STAGES * Cfg::B_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sOut + Cfg::EPI_WARPS * OUTB);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* rload = drain + 1;                     // [EPI_WARPS][2]: residual chunk loads (kEpiResid)
    uint64_t* tpre = rload + 2 * Cfg::EPI_WARPS;     // stream-K: the kSegIn accumulator is loaded
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tpre + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int n_tiles_n = (args.N + BN - 1) / BN;
    const int n_tiles = ((args.M + 2 * kBM - 1) / (2 * kBM)) * n_tiles_n;
    const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const int num_kb = args.K / Cfg::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(tfull + i, 1);
            mbar_init(tempty + i, 2 * Cfg::EPI_WARPS);   // every epilogue warp of the pair
        }
        mbar_init(drain, 1);
        for (int i = 0; i < 2 * Cfg::EPI_WARPS; ++i) mbar_init(rload + i, 1);
        mbar_init(tpre, 2 * Cfg::EPI_WARPS);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();   // both CTAs' barriers exist before any cross-CTA arrive
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            uint32_t armed = 0, armed_parity = 0;
            bool ok = true;
            // The weights do not depend on the previous kernel: the first
            // segment's B tiles of the first stages are requested before
            // griddep_wait, so they arrive while the predecessor drains.
            SegWalk walk(pair, n_pairs, n_tiles, num_kb, SK);
            int pre = 0;
            {
                SegWalk peek = walk;
                Seg g0;
                if (peek.next(g0)) {
                    const int n0 = (g0.tile % n_tiles_n) * BN + int(rank) * (BN / 2);
                    pre = g0.k1 - g0.k0 < STAGES ? g0.k1 - g0.k0 : STAGES;
                    for (int i = 0; i < pre; ++i) {
                        const uint32_t lfull = mapa_shared(smem_u32(full + i), 0);
                        if (leader) {
                            mbar_arrive_expect_tx(full + i, 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
                            armed |= 1u << i;   // phase 0
                        }
#pragma unroll
                        for (int at = 0; at < Cfg::BK / 64; ++at)
                            tma_load_2d_pair(sB + i * Cfg::B_BYTES + at * Cfg::ATOM_B, &tmB, lfull,
                                             (g0.k0 + i) * Cfg::BK + at * 64, n0);
                    }
                }
            }
            griddep_wait();
            Seg g;
            for (bool first = true; ok && walk.next(g); first = false) {
                const int m0 = (g.tile / n_tiles_n) * 2 * kBM + int(rank) * kBM;
                const int n0 = (g.tile % n_tiles_n) * BN + int(rank) * (BN / 2);
                for (int kb = g.k0; kb < g.k1; ++kb) {
                    // Stages 0..pre-1 of the first segment: armed and B requested above.
                    const bool prefetched = first && kb - g.k0 < pre;
                    if (!prefetched && !mbar_wait(empty + s, ph ^ 1, args.status, kErrTimeoutProducer, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t lfull = mapa_shared(smem_u32(full + s), 0);
                    if (leader && !prefetched) {
                        mbar_arrive_expect_tx(full + s, 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
                        armed |= 1u << s;
                        armed_parity = (armed_parity & ~(1u << s)) | (ph << s);
                    }
#pragma unroll
                    for (int at = 0; at < Cfg::BK / 64; ++at) {
                        tma_load_2d_pair(sA + s * Cfg::A_BYTES + at * Cfg::ATOM_A, &tmA, lfull, kb * Cfg::BK + at * 64, m0);
                        if (!prefetched)
                            tma_load_2d_pair(sB + s * Cfg::B_BYTES + at * Cfg::ATOM_B, &tmB, lfull,
                                             kb * Cfg::BK + at * 64, n0);
                    }
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
            }
            if (!ok && leader) {
                // Gave up: wait (bounded) for the pair's copies counted on these barriers.
                for (int i = 0; i < STAGES; ++i)
                    if (armed & (1u << i))
                        mbar_wait(full + i, (armed_parity >> i) & 1u, args.status, kErrTimeoutDrain, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = umma_idesc_f16(2 * kBM, BN, 0, 0);
            // Descriptors are built once; a stage advances the start address
            // field by its byte size / 16, a K step of 16 by 32 bytes (2).
            const uint64_t dA0 = umma_desc_sw128(smem_u32(sA), 16, 1024);
            const uint64_t dB0 = umma_desc_sw128(smem_u32(sB), 16, 1024);
            int s = 0;
            uint32_t ph = 0;
            bool ok = true, issued = false;
            int local = 0;
            SegWalk walk(pair, n_pairs, n_tiles, num_kb, SK);
            Seg g;
            for (; ok && walk.next(g); ++local) {
                const int acc = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!mbar_wait(tempty + acc, aph ^ 1, args.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                // A kSegIn accumulator starts from the previous pair's partial,
                // which the epilogue warps load into tensor memory.
                if (SK && g.role == kSegIn && !mbar_wait(tpre, 0, args.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                const bool cont = SK && g.role == kSegIn;
                for (int kb = g.k0; kb < g.k1; ++kb) {
                    if (!mbar_wait(full + s, ph, args.status, kErrTimeoutMma, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = dA0 + uint64_t(s) * (Cfg::A_BYTES >> 4);
                    const uint64_t db = dB0 + uint64_t(s) * (Cfg::B_BYTES >> 4);
#pragma unroll
                    for (int k = 0; k < Cfg::BK / 16; ++k)
                        umma_f16_ss_pair(d_tmem, da + (k / 4) * (Cfg::ATOM_A >> 4) + 2 * (k % 4),
                                         db + (k / 4) * (Cfg::ATOM_B >> 4) + 2 * (k % 4), idesc,
                                         cont || (kb != g.k0) || (k != 0));
                    issued = true;
                    umma_commit_pair(empty + s, 0x3);
                    if (++s == STAGES) {
                        s = 0;
                        ph ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit_pair(tfull + acc, 0x3);
            }
            if (!ok && issued) {
                umma_commit_pair(drain, 0x1);
                mbar_wait(drain, 0, args.status, kErrTimeoutDrain, nullptr);
            }
        }
    } else {
        // Epilogue warps 2..EPI_WARPS+1: warp w reads TMEM lane quarter w % 4
        // (rows 32*(w%4)..+31 of this CTA's half) and WARP_COLS of the 256 columns.
        griddep_wait();   // the residual is the previous kernels' output
        const int quarter = warp & 3;
        const int col_grp = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        uint32_t rphase = 0;     // bit b: parity of the next residual load into buffer b
        uint32_t rpending = 0;   // bit b: a residual load into buffer b is in flight
        int local = 0;
        const int ew = warp - 2;
        // This warp's 32 rows x WARP_COLS of a pair's stream-K slot: float4 i
        // of chunk c of every lane at [(c * 8 + i) * 32 + lane], so each warp
        // access is 512 contiguous bytes.
        auto sk_slot = [&](int slot_pair) {
            return args.sk_work + size_t(slot_pair) * kSkSlotFloats + int(rank) * (kSkSlotFloats / 2) +
                   ew * (32 * Cfg::WARP_COLS) + lane * 4;
        };
        // Stream-K: the previous pair's head accumulator of the kSegIn tile
        // into accumulator buffer `buf` (free: its last user's epilogue is done).
        auto preload = [&](int buf) -> bool {
            int* fl = args.sk_flags + ((pair - 1) * 2 + int(rank)) * 8 + ew;
            int got = 1;
            if (lane == 0) {
                got = flag_wait(fl, args.status, kErrTimeoutEpilogue, abort_flag);
                if (got) *fl = 0;   // consumed: zero again for the next launch
            }
            if (!__shfl_sync(0xffffffffu, got, 0)) return false;
            const float* src = sk_slot(pair - 1);
            const uint32_t tb = tmem_base + (uint32_t(quarter * 32) << 16) + buf * BN + col_grp * Cfg::WARP_COLS;
#pragma unroll 1
            for (int c = 0; c < Cfg::WARP_COLS / 32; ++c) {
                uint32_t r[32];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (c * 8 + i) * 128));
                    r[4 * i] = __float_as_uint(v.x); r[4 * i + 1] = __float_as_uint(v.y);
                    r[4 * i + 2] = __float_as_uint(v.z); r[4 * i + 3] = __float_as_uint(v.w);
                }
                tmem_st32(tb + c * 32, r);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(tpre), 0));
            return true;
        };
        SegWalk walk(pair, n_pairs, n_tiles, num_kb, SK);
        Seg g, gnext;
        bool have = walk.next(g);
        if (SK && have && g.role == kSegIn && !preload(0)) have = false;
        for (; have; g = gnext, ++local) {
            const bool have_next = walk.next(gnext);
            // The accumulator of a following kSegIn is loaded now, so its
            // mainloop can overlap this segment's epilogue; after a kSegOut
            // only once that segment's partial is out (pairs whose head is
            // followed straight by their tail would otherwise wait in a chain).
            const bool preload_next = SK && have_next && gnext.role == kSegIn;
            if (preload_next && g.role != kSegOut && !preload((local + 1) & 1)) break;
            const int tile = g.tile;
            const int acc = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            const int m = (tile / n_tiles_n) * 2 * kBM + int(rank) * kBM + row;
            const int n0 = (tile % n_tiles_n) * BN + col_grp * Cfg::WARP_COLS;
            const bool row_ok = m < args.M;
            if (SK && g.role == kSegOut) {
                // The tile's first K blocks: raw accumulator to this pair's slot.
                if (!mbar_wait(tfull + acc, aph, args.status, kErrTimeoutEpilogue, abort_flag)) break;
                tc_fence_after();
                const uint32_t tb = tmem_base + (uint32_t(quarter * 32) << 16) + acc * BN + col_grp * Cfg::WARP_COLS;
                float* dst = sk_slot(pair);
#pragma unroll 1
                for (int c = 0; c < Cfg::WARP_COLS / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(tb + c * 32, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        __stcg(reinterpret_cast<float4*>(dst + (c * 8 + i) * 128), make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                                   __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) flag_release(args.sk_flags + (pair * 2 + int(rank)) * 8 + ew, 1);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(tempty + acc), 0));
                if (preload_next && !preload((local + 1) & 1)) break;
                have = have_next;
                continue;
            }
            if constexpr (EPI == kEpiResid) {
                // The fp32 residual comes in by TMA, 32 x 32 chunks into this
                // warp's RB store stages: the first RB chunks while the tile's
                // mainloop still runs, the others pulled into L2 now and loaded
                // into a stage as soon as its store has read it, RB chunks
                // ahead (the residual is not written by anyone else before this
                // epilogue).
                const int row0 = m - lane;
                if (*abort_flag) break;
                if (row0 < args.M) {
                    if (lane == 0) {
                        bulk_wait_group_read<0>();   // the previous tile's stores have read both stages
#pragma unroll
                        for (int b = 0; b < RB; ++b) {
                            mbar_arrive_expect_tx(rload + 2 * ew + b, Cfg::kResidBuf);
                            tma_load_2d(sOut + ew * OUTB + b * Cfg::kResidBuf, &tmC, rload + 2 * ew + b, n0 + 32 * b,
                                        row0);
                        }
#pragma unroll
                        for (int q = RB; q < Cfg::WARP_COLS / 32; ++q) tma_prefetch_l2_2d(&tmC, n0 + 32 * q, row0);
                    }
                    rpending = (1u << RB) - 1;
                }
            }
            if (!mbar_wait(tfull + acc, aph, args.status, kErrTimeoutEpilogue, abort_flag)) break;
            tc_fence_after();
            const uint32_t tbase = tmem_base + (uint32_t(quarter * 32) << 16) + acc * BN + col_grp * Cfg::WARP_COLS;
            if constexpr (EPI == kEpiF16) {
                // Rows row0..row0+31 of the chunk go out through shared memory
                // and one TMA store per warp (rows past M are not written).
                uint8_t* stage = sOut + (warp - 2) * OUTB;
                const int row0 = m - lane;
#pragma unroll 1
                for (int c = 0; c < Cfg::WARP_COLS / 32; ++c) {
                    const int n = n0 + c * 32;
                    if (n >= args.N) break;
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_wait_ld();
                    uint32_t pk[16];
                    f16_chunk(args, n, r, pk);
                    uint8_t* buf = stage + (c % Cfg::OUT_BUFS) * 2048;
                    if (lane == 0) bulk_wait_group_read<Cfg::OUT_BUFS - 1>();   // earlier store has read buf
                    __syncwarp();
                    uint8_t* rowp = buf + lane * 64;
                    const int sw = (lane >> 1) & 3;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        *reinterpret_cast<uint4*>(rowp + ((q ^ sw) << 4)) =
                            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (row0 < args.M) tma_store_2d(&tmC, buf, n, row0);
                        bulk_commit_group();
                    }
                }
            } else if constexpr (EPI == kEpiQkv) {
                // As above, but a 32-row chunk is stored as four 8-row boxes
                // into the [which][group][head][token][64] layout: 8 tokens in
                // a row of the grid never straddle a window or an image.
                uint8_t* stage = sOut + (warp - 2) * OUTB;
                const int row0 = m - lane;
                const int L = args.windowed ? kWindow * kWindow : kTokens;
                const int planes = int(args.qkv_stride / (int64_t(L) * kHeadDim));   // group x head planes per q/k/v
#pragma unroll 1
                for (int c = 0; c < Cfg::WARP_COLS / 32; ++c) {
                    const int n = n0 + c * 32;
                    if (n >= args.N) break;
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_wait_ld();
                    uint32_t pk[16];
                    qkv_chunk(args, m, n, r, pk);
                    uint8_t* buf = stage + (c % Cfg::OUT_BUFS) * 2048;
                    if (lane == 0) bulk_wait_group_read<Cfg::OUT_BUFS - 1>();
                    __syncwarp();
                    uint8_t* rowp = buf + lane * 64;
                    const int sw = (lane >> 1) & 3;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        *reinterpret_cast<uint4*>(rowp + ((q ^ sw) << 4)) =
                            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        const int which = n >> 10, head = (n & 1023) >> 6, half = (n >> 5) & 1;
#pragma unroll
                        for (int r8 = 0; r8 < 4; ++r8) {
                            const int mm = row0 + 8 * r8;
                            if (mm < args.M) {
                                const QkvPos p = qkv_pos(mm, args.windowed);
                                tma_store_3d(&tmC, buf + r8 * 512, half * 32, p.i,
                                             which * planes + p.g * kHeads + head);
                            }
                        }
                        bulk_commit_group();
                    }
                }
            } else if constexpr (EPI == kEpiResid) {
                // Stage c % RB (32 rows x 128 B, 128-byte swizzle, the layout TMA
                // writes) holds chunk c of the residual; each lane adds its row's
                // accumulator and bias in place, and one TMA store writes the
                // chunk back.  Rows past M are zero-filled by the load and not
                // written by the store.
                const int row0 = m - lane;
                const bool chunk_rows = row0 < args.M;   // warp-uniform
                // A warp whose 32 rows all lie past M has nothing to add or store;
                // it must not touch the stage, which its previous tile's last
                // store may still be reading.
#pragma unroll
                for (int c = 0; c < Cfg::WARP_COLS / 32 && chunk_rows; ++c) {
                    const int n = n0 + c * 32;
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_wait_ld();
                    const int b = c % RB;
                    uint8_t* stage = sOut + ew * OUTB + b * Cfg::kResidBuf;
                    if (!mbar_wait(rload + 2 * ew + b, (rphase >> b) & 1u, args.status, kErrTimeoutEpilogue, abort_flag))
                        break;
                    rphase ^= 1u << b;
                    rpending &= ~(1u << b);
                    uint8_t* rowp = stage + lane * 128;
                    // x = x + (acc + bias), two columns per packed operation
                    const float4* bp = reinterpret_cast<const float4*>(args.bias + n);
                    float v[32];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 xq = *reinterpret_cast<const float4*>(rowp + ((q ^ (lane & 7)) << 4));
                        const float4 bb = args.bias ? __ldg(bp + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                        const float2 s0 = __fadd2_rn(
                            make_float2(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1])),
                            make_float2(bb.x, bb.y));
                        const float2 s1 = __fadd2_rn(
                            make_float2(__uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])),
                            make_float2(bb.z, bb.w));
                        const float2 t0 = __fadd2_rn(make_float2(xq.x, xq.y), s0);
                        const float2 t1 = __fadd2_rn(make_float2(xq.z, xq.w), s1);
                        v[4 * q] = t0.x; v[4 * q + 1] = t0.y; v[4 * q + 2] = t1.x; v[4 * q + 3] = t1.y;
                        *reinterpret_cast<float4*>(rowp + ((q ^ (lane & 7)) << 4)) = make_float4(t0.x, t0.y, t1.x, t1.y);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmC, stage, n, row0);
                        bulk_commit_group();
                        if (c + RB < Cfg::WARP_COLS / 32) {
                            bulk_wait_group_read<0>();   // the store has read the stage
                            mbar_arrive_expect_tx(rload + 2 * ew + b, Cfg::kResidBuf);
                            tma_load_2d(stage, &tmC, rload + 2 * ew + b, n + 32 * RB, row0);
                        }
                    }
                    if (c + RB < Cfg::WARP_COLS / 32) rpending |= 1u << b;
                    if (row_ok && args.out_nchw) {
                        const int img = m / kTokens, t = m - img * kTokens;
                        float* o = args.out_nchw + (int64_t(img) * args.N + n) * kTokens + t;
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[int64_t(i) * kTokens] = v[i];
                    }
                }
            } else {
#pragma unroll 1
                for (int c = 0; c < Cfg::WARP_COLS / 32; ++c) {
                    const int n = n0 + c * 32;
                    if (n >= args.N) break;
                    uint32_t r[32];
                    tmem_ld32(tbase + c * 32, r);
                    tmem_wait_ld();
                    if (m < args.M) epilogue_chunk<EPI>(args, m, n, r);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(tempty + acc), 0));
            have = have_next;
        }
        if constexpr (EPI == kEpiResid) {
            // Gave up mid-tile: let the residual loads in flight land before the CTA exits.
            for (int b = 0; b < 2; ++b)
                if (rpending & (1u << b))
                    mbar_wait(rload + 2 * ew + b, (rphase >> b) & 1u, args.status, kErrTimeoutDrain, nullptr);
        }
        if constexpr (Cfg::staged_out(EPI)) {
            if (lane == 0) bulk_wait_group_all();
        }
    }

    tc_fence_before();
    cluster_sync();   // no CTA leaves while its pair may still signal or read it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

template <int BN, int EPI>
cudaError_t launch_bn(const __half* A, const __half* B, const GemmArgs& args, int num_sms, cudaStream_t stream) {
    using Cfg = GemmCfg<BN>;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.K, args.M, kBK, kBM)) return cudaErrorInvalidValue;
    if (!make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.K, args.N, kBK, BN)) return cudaErrorInvalidValue;
    auto kern = gemm_tn_kernel<BN, EPI>;
    const int n_tiles = ((args.M + kBM - 1) / kBM) * ((args.N + BN - 1) / BN);
    const int grid = n_tiles < num_sms ? n_tiles : num_sms;
    kern<<<grid, 192, Cfg::SMEM, stream>>>(ta, tb, args);
    return cudaGetLastError();
}

// Co-resident CTA pairs of the pair kernel on the current device (set by
// gemm_prepare; one process drives one device at a time in this library).
int g_pair_capacity = 0;

template <int EPI, int BK, int RB = 1>
cudaError_t launch_pair_bk(const __half* A, const __half* B, const GemmArgs& args, int num_sms, cudaStream_t stream) {
    using Cfg = PairCfgT<BK, RB>;
    CUtensorMap ta, tb;
    if (!make_tmap_2d(&ta, A, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.K, args.M, kBK, kBM)) return cudaErrorInvalidValue;
    if (!make_tmap_2d(&tb, B, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.K, args.N, kBK, PairCfg::BN / 2))
        return cudaErrorInvalidValue;
    const int n_tiles = ((args.M + 2 * kBM - 1) / (2 * kBM)) * ((args.N + PairCfg::BN - 1) / PairCfg::BN);
    // Persistent grid: only as many pairs as can be resident at once.
    const int max_pairs = g_pair_capacity > 0 ? g_pair_capacity : num_sms / 2;
    int pairs = n_tiles < max_pairs ? n_tiles : max_pairs;
    // Stream-K when whole tiles would leave the last of at most three waves
    // mostly idle (one or two images: 84 or 164 fc2 tiles on 74 pairs) and
    // the K loop is long enough to pay for the hand-over of a tile's
    // accumulator (a K = 1024 tile's epilogue takes as long as its mainloop;
    // at four images the hand-over costs more than the last wave's idle
    // time); needs every pair resident, which the persistent grid of
    // max_pairs is.
    GemmArgs ka = args;
    ka.sk = 0;
    if (args.sk_work && args.sk_flags && args.sk_slots >= max_pairs && n_tiles >= max_pairs && args.K >= 2048) {
        const int waves = (n_tiles + max_pairs - 1) / max_pairs;
        if (waves <= 3 && int64_t(n_tiles) * 100 < int64_t(92) * waves * max_pairs) {
            ka.sk = 1;
            pairs = max_pairs;
        }
    }
    CUtensorMap tc = ta;
    if (EPI == kEpiF16 &&
        !make_tmap_2d(&tc, args.out16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, args.N, args.M, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    if (EPI == kEpiResid &&
        !make_tmap_2d(&tc, args.resid, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, args.N, args.M, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    if (EPI == kEpiQkv) {
        // q, k, v: qkv_stride elements each, contiguous; one plane per (group, head).
        const uint64_t L = args.windowed ? kWindow * kWindow : kTokens;
        if (args.N != 3 * kDim || args.qkv_stride % int64_t(L * kHeadDim) != 0 ||
            !make_tmap_3d(&tc, args.qkv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kHeadDim, L,
                          3 * uint64_t(args.qkv_stride) / (L * kHeadDim), 32, 8, CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
    }
    if (ka.sk)
        return launch_kernel(gemm_pair_kernel<EPI, BK, true, RB>, dim3(2 * pairs), dim3(Cfg::THREADS),
                             Cfg::template smem<EPI>(), stream, ta, tb, tc, ka);
    return launch_kernel(gemm_pair_kernel<EPI, BK, false, RB>, dim3(2 * pairs), dim3(Cfg::THREADS),
                         Cfg::template smem<EPI>(), stream, ta, tb, tc, ka);
}

template <int EPI>
cudaError_t launch_pair(const __half* A, const __half* B, const GemmArgs& args, int num_sms, cudaStream_t stream) {
    if constexpr (EPI == kEpiResid)
        return args.K >= 2048 ? launch_pair_bk<EPI, 64, 1>(A, B, args, num_sms, stream)
                              : launch_pair_bk<EPI, 64, 2>(A, B, args, num_sms, stream);
    else
        return args.K >= 2048 ? launch_pair_bk<EPI, 64>(A, B, args, num_sms, stream)
                              : launch_pair_bk<EPI, 128>(A, B, args, num_sms, stream);
}

template <int EPI, bool SK>
cudaError_t prepare_pair_sk() {
    if constexpr (EPI == kEpiResid) {
        const cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<EPI, 64, SK, 2>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   int(PairCfgT<64, 2>::smem<EPI>()));
        if (e != cudaSuccess) return e;
    } else {
        const cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<EPI, 128, SK, 1>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   int(PairCfgT<128>::smem<EPI>()));
        if (e != cudaSuccess) return e;
    }
    return cudaFuncSetAttribute(gemm_pair_kernel<EPI, 64, SK, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(PairCfgT<64>::smem<EPI>()));
}

template <int EPI>
cudaError_t prepare_pair() {
    const cudaError_t e = prepare_pair_sk<EPI, false>();
    return e != cudaSuccess ? e : prepare_pair_sk<EPI, true>();
}

template <int BN, int EPI>
cudaError_t prepare_bn() {
    return cudaFuncSetAttribute(gemm_tn_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(GemmCfg<BN>::SMEM));
}

}  // namespace

cudaError_t gemm_prepare() {
    cudaError_t e;
    if ((e = prepare_bn<256, kEpiF16>()) != cudaSuccess) return e;
    if ((e = prepare_bn<128, kEpiF16>()) != cudaSuccess) return e;
    if ((e = prepare_bn<256, kEpiQkv>()) != cudaSuccess) return e;
    if ((e = prepare_bn<256, kEpiResid>()) != cudaSuccess) return e;
    if ((e = prepare_bn<128, kEpiResid>()) != cudaSuccess) return e;
    if ((e = prepare_bn<256, kEpiPatch>()) != cudaSuccess) return e;
    if ((e = prepare_pair<kEpiF16>()) != cudaSuccess) return e;
    {
        int dev = 0, sms = 0, clusters = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(sms, 1, 1);
        cfg.blockDim = dim3(PairCfg::THREADS, 1, 1);
        cfg.dynamicSmemBytes = PairCfg::smem<kEpiF16>();
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = 2;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm_pair_kernel<kEpiF16, 128, false, 1>, &cfg) == cudaSuccess &&
            clusters > 0)
            g_pair_capacity = clusters;
        else
            g_pair_capacity = sms / 2;
    }
    if ((e = prepare_pair<kEpiQkv>()) != cudaSuccess) return e;
    if ((e = prepare_pair<kEpiResid>()) != cudaSuccess) return e;
    return prepare_pair<kEpiPatch>();
}

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {inner * uint64_t(elem_bytes)};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t d0,
                  uint64_t d1, uint64_t d2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {d0 * uint64_t(elem_bytes), d0 * d1 * uint64_t(elem_bytes)};
    cuuint32_t box[3] = {b0, b1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_gemm(const __half* A, const __half* B, const GemmArgs& args, int epi, int num_sms,
                        cudaStream_t stream) {
    if (args.K % kBK != 0 || args.N % 32 != 0 || args.M <= 0) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return cudaErrorInvalidValue;
    // N = 1024 / 3072 / 4736: CTA-pair 256 x 256 tiles (4736 leaves one half
    // tile); narrow problems use single-CTA 128 x 128 tiles.
    const bool wide = args.N >= 1024;
    if (wide && num_sms >= 2 && args.K % (args.K >= 2048 ? 64 : 128) == 0) {
        switch (epi) {
            case kEpiF16: return launch_pair<kEpiF16>(A, B, args, num_sms, stream);
            case kEpiQkv: return launch_pair<kEpiQkv>(A, B, args, num_sms, stream);
            case kEpiResid: return launch_pair<kEpiResid>(A, B, args, num_sms, stream);
            case kEpiPatch: return launch_pair<kEpiPatch>(A, B, args, num_sms, stream);
        }
        return cudaErrorInvalidValue;
    }
    switch (epi) {
        case kEpiF16:
            return wide ? launch_bn<256, kEpiF16>(A, B, args, num_sms, stream)
                        : launch_bn<128, kEpiF16>(A, B, args, num_sms, stream);
        case kEpiQkv:
            return launch_bn<256, kEpiQkv>(A, B, args, num_sms, stream);
        case kEpiResid:
            return wide ? launch_bn<256, kEpiResid>(A, B, args, num_sms, stream)
                        : launch_bn<128, kEpiResid>(A, B, args, num_sms, stream);
        case kEpiPatch:
            return launch_bn<256, kEpiPatch>(A, B, args, num_sms, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace s3t
