// Flash attention for the trunk (d = 64, 16 heads, no mask), tcgen05 based.
//
// Semantics: ggml_flash_attn_ext with scale 1/8 and F32 precision as used by
// apply_attention (src/vision_trunk.cpp:207-228): out = softmax(q k^T / 8) v.
// Windowed layers attend within each 24x24 window (L = 576 keys), global
// layers over the 72x72 grid (L = 5184).  RoPE was already applied by the QKV
// GEMM epilogue; window partition/unpartition (:235-282) is pure addressing:
// q/k/v arrive grouped per (window, head) and the output is written back to
// natural token order, so no permute copy exists.
//
// Persistent kernel: each CTA walks a static list of work items (128-query
// tile, head, group).  Roles (192 threads): warp 0 TMA producer, warp 1 TMEM
// owner + UMMA issuer, warps 2..5 softmax + epilogue (one query row per
// thread).  Per 64-key block b of an item:
//   S = Q K^T   : UMMA M=128 N=64 K=64, A = Q read from TMEM Q[item & 1],
//                 K from shared memory, accumulator in TMEM cols [0,64)
//   P = 2^(S*scale*log2e - m) as fp16/bf16 into TMEM P[b & 1] (32 columns)
//   O += P V    : UMMA M=128 N=64 K=64, A = P read from TMEM, V MN-major from
//                 shared memory, into TMEM O
// Both UMMA kinds take A from tensor memory, so each reads only its B tile
// (2 KB per K step) from shared memory: an SS 128x64x16 UMMA, which also
// reads the 4 KB Q slice every step, is bound by shared-memory bandwidth.
// The softmax warps copy each item's Q tile from shared memory (TMA) into
// Q[item & 1], the next item's while the current item's last block is
// processed.  The UMMA issuer runs one block ahead (S_{b+1} is issued as soon
// as S_b has been read), across item boundaries too; P is double-buffered, so
// the softmax of block b never waits for the PV of block b-1.  O is single:
// the next item's first PV needs P from the same warps, after their epilogue
// has read O.  P never touches shared memory (no proxy fence on the critical
// path).  The row max used for P is raised only when a block
// exceeds it by more than 2^8 (O is then rescaled in TMEM).  Shared memory
// (80 KB) and registers are sized for two CTAs per SM; a 3-deep K/V ring
// keeps S_{b+1} from waiting on loads.
// L is a multiple of 64 for both layer kinds, so keys are never masked; query
// rows past L (last tile of a group) are computed on zero-filled Q rows and
// not stored.
#include "kernels.h"
#include "ptx.cuh"

namespace s3t {

namespace {

constexpr int kBQ = 128, kBKV = 64, kD = 64, kKVStages = 3;
constexpr int kQBufs = 2;                       // shared-memory Q tiles (TMA targets)
constexpr uint32_t kQBytes = kBQ * kD * 2;      // 16 KB
constexpr uint32_t kKVBytes = kBKV * kD * 2;    // 8 KB (each of K, V)
constexpr size_t kAttnSmem = kQBufs * kQBytes + 2 * kKVStages * kKVBytes + 1024 + 256;
constexpr uint32_t kAttnTmemCols = 256;         // S [0,64), O [64,128), P0/P1 [128,192), Q0/Q1 [192,256)
constexpr uint32_t kTmemO = 64;
constexpr uint32_t kTmemP = 128;                // P[x] at kTmemP + 32 x (64 fp16 keys per row)
constexpr uint32_t kTmemQ = 192;                // Q[x] at kTmemQ + 32 x (64 fp16 dims per row)
constexpr int kCtasPerSm = 2;

template <int BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) return pack_bf162(a, b);
    else return pack_half2(a, b);
}

struct Item {
    int qt, head, grp;
};

__device__ __forceinline__ Item item_of(int w, int n_qt) {
    Item it;
    it.qt = w % n_qt;
    const int r = w / n_qt;
    it.head = r % kHeads;
    it.grp = r / kHeads;
    return it;
}

template <int BF16>
__global__ void __launch_bounds__(192, kCtasPerSm)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                              // kQBufs buffers
    uint8_t* sK = sQ + kQBufs * kQBytes;
    uint8_t* sV = sK + kKVStages * kKVBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kKVStages * kKVBytes);
    uint64_t* q_full = bars;                         // [2]
    uint64_t* q_empty = q_full + 2;                  // [2]
    uint64_t* kv_full = q_empty + 2;                 // [S]
    uint64_t* kv_empty = kv_full + kKVStages;        // [S]
    uint64_t* s_full = kv_empty + kKVStages;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_free + 1;                   // [2]: P of blocks with that parity
    uint64_t* o_done = p_full + 2;                   // [2]: PV of blocks with that parity
    uint64_t* o_free = o_done + 2;                   // O read by the item epilogue
    uint64_t* drain = o_free + 1;
    uint64_t* qt_full = drain + 1;                   // [2]: Q of the item with that parity in TMEM
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qt_full + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkv = a.L / kBKV;
    const int n_qt = (a.L + kBQ - 1) / kBQ;
    const int n_items = n_qt * kHeads * a.groups;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(q_full + i, 1);
            mbar_init(q_empty + i, 4);
            mbar_init(qt_full + i, 4);
            mbar_init(o_done + i, 1);
            mbar_init(p_full + i, 4);
        }
        mbar_init(o_free, 4);
        for (int s = 0; s < kKVStages; ++s) {
            mbar_init(kv_full + s, 1);
            mbar_init(kv_empty + s, 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kAttnTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem;
    griddep_launch_dependents();
    griddep_wait();   // q, k, v are the QKV GEMM's output

    if (warp == 0) {
        if (lane == 0) {
            uint32_t armed = 0, armed_parity = 0, q_armed = 0, q_parity = 0;
            bool ok = true;
            int b = 0;   // global block counter of this CTA
            int li = 0;  // local item counter
            for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++li) {
                const Item it = item_of(w, n_qt);
                const int bh = it.grp * kHeads + it.head;
                const int qb = li % kQBufs;
                const uint32_t qph = (li / kQBufs) & 1;
                if (!mbar_wait(q_empty + qb, qph ^ 1, a.status, kErrTimeoutProducer, abort_flag)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(q_full + qb, kQBytes);
                tma_load_3d(sQ + qb * kQBytes, &tmQ, q_full + qb, 0, it.qt * kBQ, bh);
                q_armed |= 1u << qb;
                q_parity = (q_parity & ~(1u << qb)) | (qph << qb);
                for (int j = 0; j < nkv; ++j, ++b) {
                    const int s = b % kKVStages;
                    const uint32_t ph = (b / kKVStages) & 1;
                    if (!mbar_wait(kv_empty + s, ph ^ 1, a.status, kErrTimeoutProducer, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(kv_full + s, 2 * kKVBytes);
                    tma_load_3d(sK + s * kKVBytes, &tmK, kv_full + s, 0, j * kBKV, bh);
                    tma_load_3d(sV + s * kKVBytes, &tmV, kv_full + s, 0, j * kBKV, bh);
                    armed |= 1u << s;
                    armed_parity = (armed_parity & ~(1u << s)) | (ph << s);
                }
            }
            if (!ok) {
                // Gave up: wait (bounded) for every copy this thread started.
                for (int i = 0; i < 2; ++i)
                    if (q_armed & (1u << i))
                        mbar_wait(q_full + i, (q_parity >> i) & 1u, a.status, kErrTimeoutDrain, nullptr);
                for (int i = 0; i < kKVStages; ++i)
                    if (armed & (1u << i))
                        mbar_wait(kv_full + i, (armed_parity >> i) & 1u, a.status, kErrTimeoutDrain, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idS = umma_idesc_f16(kBQ, kBKV, BF16, 0);
            constexpr uint32_t idO = umma_idesc_f16(kBQ, kD, BF16, 1);
            const int my_items = int(blockIdx.x) < n_items ? (n_items - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;
            const int total = my_items * nkv;
            bool ok = true, issued = false;
            // Descriptors are built once; a K step of 16 advances the start
            // address field by 32 bytes (2) for K-major tiles and by 16 rows
            // of 128 bytes (128) for the MN-major V tile.
            const uint64_t dK0 = umma_desc_sw128(smem_u32(sK), 16, 1024);
            const uint64_t dV0 = umma_desc_sw128(smem_u32(sV), kKVBytes, 1024);
            constexpr uint64_t kStageStep = kKVBytes >> 4;
            // State of the next S block to issue (block counter, key block, item, ring stage/phase).
            int sb = 0, sj = 0, sli = 0, ss = 0;
            uint32_t sph = 0;
            auto issue_s = [&]() -> bool {
                const int qb = sli & 1;
                if (sj == 0 && !mbar_wait(qt_full + qb, (sli >> 1) & 1, a.status, kErrTimeoutMma, abort_flag))
                    return false;
                if (!mbar_wait(kv_full + ss, sph, a.status, kErrTimeoutMma, abort_flag)) return false;
                if (sb > 0 && !mbar_wait(s_free, (sb - 1) & 1, a.status, kErrTimeoutMma, abort_flag)) return false;
                tc_fence_after();
                // S = Q K^T with Q read from tensor memory (TS form): only K
                // comes from shared memory, so each UMMA reads half the bytes.
                const uint32_t tq = tmem + kTmemQ + qb * 32;
                const uint64_t dk = dK0 + uint64_t(ss) * kStageStep;
#pragma unroll
                for (int k = 0; k < kD / 16; ++k) umma_f16_ts(tS, tq + 8 * k, dk + 2 * k, idS, k != 0);
                umma_commit(s_full);
                issued = true;
                ++sb;
                if (++sj == nkv) { sj = 0; ++sli; }
                if (++ss == kKVStages) { ss = 0; sph ^= 1; }
                return true;
            };
            if (total > 0) ok = issue_s();
            int j = 0, li = 0, s = 0;
            for (int b = 0; ok && b < total; ++b) {
                if (b + 1 < total && !issue_s()) {
                    ok = false;
                    break;
                }
                if (!mbar_wait(p_full + (b & 1), (b >> 1) & 1, a.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                if (j == 0 && !mbar_wait(o_free, (li & 1) ^ 1, a.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t dv = dV0 + uint64_t(s) * kStageStep;
                const uint32_t tO = tmem + kTmemO;
                const uint32_t tP = tmem + kTmemP + (b & 1) * 32;
#pragma unroll
                for (int k = 0; k < kBKV / 16; ++k) umma_f16_ts(tO, tP + 8 * k, dv + 128 * k, idO, (j | k) != 0);
                umma_commit(kv_empty + s);
                umma_commit(o_done + (b & 1));
                if (++j == nkv) { j = 0; ++li; }
                if (++s == kKVStages) s = 0;
            }
            if (!ok && issued) {
                umma_commit(drain);
                mbar_wait(drain, 0, a.status, kErrTimeoutDrain, nullptr);
            }
        }
    } else {
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = uint32_t(quarter * 32) << 16;
        const float sl2 = a.scale_log2;
        // m_run is the (log2-domain) max the P values of this row are taken
        // relative to.  It is only raised when a block's max exceeds it by
        // more than kRescaleSlack, so O is rescaled in TMEM rarely; P values
        // stay <= 2^kRescaleSlack, and O / l is unchanged by the choice.
        constexpr float kRescaleSlack = 8.0f;
        bool ok = true;
        int b = 0, li = 0;
        // Q of item i goes from its shared-memory tile (TMA, 128-byte swizzle)
        // into tensor memory Q[i & 1], where the S UMMAs read it; the shared
        // tile is then free for the producer.  Item 0 first, item i + 1 while
        // item i's last block is processed (its S has been read).
        auto copy_q = [&](int i) -> bool {
            const int qb = i & 1, qs = i % kQBufs;
            if (!mbar_wait(q_full + qs, (i / kQBufs) & 1, a.status, kErrTimeoutEpilogue, abort_flag)) return false;
            const uint8_t* rowp = sQ + qs * kQBytes + row * 128;
            uint32_t qr[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 u = *reinterpret_cast<const uint4*>(rowp + ((c ^ (row & 7)) << 4));
                qr[4 * c] = u.x; qr[4 * c + 1] = u.y; qr[4 * c + 2] = u.z; qr[4 * c + 3] = u.w;
            }
            tmem_st32(tmem + kTmemQ + qb * 32 + lane_off, qr);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(qt_full + qb);
                mbar_arrive(q_empty + qs);
            }
            return true;
        };
        if (int(blockIdx.x) < n_items) ok = copy_q(0);
        const uint32_t tO = tmem + kTmemO;
        for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++li) {
            const Item it = item_of(w, n_qt);
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < nkv; ++j, ++b) {
                if (!mbar_wait(s_full, b & 1, a.status, kErrTimeoutEpilogue, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t r[64];
                tmem_ld32(tS + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
                tmem_ld32(tS + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_free);
                if (j == nkv - 1 && w + int(gridDim.x) < n_items && !copy_q(li + 1)) {
                    ok = false;
                    break;
                }

                float acc[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = fmaxf(__uint_as_float(r[i]), __uint_as_float(r[8 + i]));
#pragma unroll
                for (int i = 16; i < 64; i += 16)
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        acc[k] = fmax3(acc[k], __uint_as_float(r[i + k]), __uint_as_float(r[i + 8 + k]));
                const float mx =
                    fmax3(fmax3(acc[0], acc[1], acc[2]), fmax3(acc[3], acc[4], acc[5]), fmaxf(acc[6], acc[7])) * sl2;
                const bool raise = mx > m_run + kRescaleSlack;
                const float m_new = raise ? mx : m_run;
                const float alpha = raise ? ex2_approx(m_run - m_new) : 1.0f;
                // Two scores per packed f32x2 instruction (fewer issue slots).
                uint32_t pk[32];
                float2 sums[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                const float2 sl2x2 = make_float2(sl2, sl2), negm = make_float2(-m_new, -m_new);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float2 t = __ffma2_rn(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                                                sl2x2, negm);
                    const float2 e = make_float2(ex2_approx(t.x), ex2_approx(t.y));
                    sums[i & 1] = __fadd2_rn(sums[i & 1], e);
                    pk[i] = pack2<BF16>(e.x, e.y);
                }
                l_run = l_run * alpha + ((sums[0].x + sums[1].x) + (sums[0].y + sums[1].y));

                // P buffer b & 1 is free once the PV of block b-2 has completed.
                if (b > 1) {
                    if (!mbar_wait(o_done + (b & 1), ((b - 2) >> 1) & 1, a.status, kErrTimeoutEpilogue, abort_flag)) {
                        ok = false;
                        break;
                    }
                }
                // Rescaling O needs the PV of block b-1 (same item) to have completed.
                if (j > 0 && __any_sync(0xffffffffu, raise)) {
                    if (!mbar_wait(o_done + ((b - 1) & 1), ((b - 1) >> 1) & 1, a.status, kErrTimeoutEpilogue,
                                   abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    {
                        uint32_t o0[32], o1[32];
                        tmem_ld32(tO + lane_off, o0);
                        tmem_ld32(tO + lane_off + 32, o1);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            o0[i] = __float_as_uint(__uint_as_float(o0[i]) * alpha);
                            o1[i] = __float_as_uint(__uint_as_float(o1[i]) * alpha);
                        }
                        tmem_st32(tO + lane_off, o0);
                        tmem_st32(tO + lane_off + 32, o1);
                        tmem_wait_st();
                    }
                }
                // P row -> this row's TMEM lane (key 2i in the low half of column i).
                tmem_st32(tmem + kTmemP + (b & 1) * 32 + lane_off, pk);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full + (b & 1));
                m_run = m_new;
            }
            if (!ok || !mbar_wait(o_done + ((b - 1) & 1), ((b - 1) >> 1) & 1, a.status, kErrTimeoutEpilogue, abort_flag)) {
                ok = false;
                break;
            }
            // Item epilogue: O / l, natural token order.
            tc_fence_after();
            uint32_t o0[32], o1[32];
            tmem_ld32(tO + lane_off, o0);
            tmem_ld32(tO + lane_off + 32, o1);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            const int qi = it.qt * kBQ + row;
            if (qi < a.L) {
                const float inv = 1.0f / l_run;
                float v[2][32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    v[0][i] = __uint_as_float(o0[i]) * inv;
                    v[1][i] = __uint_as_float(o1[i]) * inv;
                }
                if (a.q8) {
                    q8_0_fake_quant32(v[0]);
                    q8_0_fake_quant32(v[1]);
                }
                int img, tok;
                if (a.windowed) {
                    img = it.grp / 9;
                    const int wi = it.grp - img * 9, wy = wi / 3, wx = wi - wy * 3;
                    const int ly = qi / kWindow, lx = qi - ly * kWindow;
                    tok = (wy * kWindow + ly) * kGrid + wx * kWindow + lx;
                } else {
                    img = it.grp;
                    tok = qi;
                }
                uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) +
                                                      (int64_t(img) * kTokens + tok) * kDim + it.head * kD);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        dst[h * 4 + c] = make_uint4(pack2<BF16>(v[h][8 * c], v[h][8 * c + 1]),
                                                    pack2<BF16>(v[h][8 * c + 2], v[h][8 * c + 3]),
                                                    pack2<BF16>(v[h][8 * c + 4], v[h][8 * c + 5]),
                                                    pack2<BF16>(v[h][8 * c + 6], v[h][8 * c + 7]));
            }
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kAttnTmemCols);
    }
}

}  // namespace

cudaError_t attention_prepare() {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem));
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_fwd_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kAttnSmem));
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t stream) {
    if (a.L % kBKV != 0 || a.groups <= 0) return cudaErrorInvalidValue;
    const CUtensorMapDataType dt = a.bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t zdim = uint64_t(a.groups) * kHeads;
    CUtensorMap tq, tk, tv;
    if (!make_tmap_3d(&tq, a.q, dt, 2, kD, a.L, zdim, kD, kBQ)) return cudaErrorInvalidValue;
    if (!make_tmap_3d(&tk, a.k, dt, 2, kD, a.L, zdim, kD, kBKV)) return cudaErrorInvalidValue;
    if (!make_tmap_3d(&tv, a.v, dt, 2, kD, a.L, zdim, kD, kBKV)) return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int n_items = ((a.L + kBQ - 1) / kBQ) * kHeads * a.groups;
    const int grid = n_items < sms * kCtasPerSm ? n_items : sms * kCtasPerSm;
    if (a.bf16) return launch_kernel(attn_fwd_kernel<1>, dim3(grid), dim3(192), kAttnSmem, stream, tq, tk, tv, a);
    return launch_kernel(attn_fwd_kernel<0>, dim3(grid), dim3(192), kAttnSmem, stream, tq, tk, tv, a);
}

}  // namespace s3t
