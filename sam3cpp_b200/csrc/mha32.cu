// Multi-head attention of the encoder fusion, tcgen05 based: 8 heads of 32,
// model width 256.
//
// Semantics: ggml_flash_attn_ext with prec F32 as used by mha() in
// src/encoder_fusion.cpp:63-88, scale 1/sqrt(32):
//   out = softmax(q k^T * scale + mask) v   per head,
// the mask being additive per key and broadcast over query rows (the prompt
// mask of :120-133 is the same for every row).  As in the CPU kernel
// (ggml-cpu/ops.cpp:8254-8257, 8353-8354) a key whose mask is -inf takes no
// part at all, and a row with every key masked comes out as 0.  Self attention
// (:266) has no mask and q_len = kv_len = H*W; cross attention to the prompt
// (:299) has a short, ragged kv_len and the mask.
//
// Layout: q/k/v are token-major [len][256] (head h in columns [32h, 32h+32)),
// exactly the rows the projection GEMMs produce, for `batch` sequences back
// to back; a 3-D tensor map per operand cuts [rows][32] tiles of one head of
// one sequence with 64-byte swizzle (rows past the sequence's end read as 0).
// Output [batch][q_len][256] fp32 (or fp16/bf16), the layout the output
// projection reads.
//
// Persistent kernel, same pipeline as the trunk's attention (attention.cu):
// each CTA walks work items (128-query tile, head, sequence, key range).  When
// the query tiles are too few to fill the GPU (the decoder's 201 queries
// against 5184 image tokens make 16 tiles), the key blocks of a tile are split
// into ranges: each item then writes its unnormalised O with its (m, l) to a
// scratch buffer, and mha32_combine merges the ranges per row.  Warp 0 TMA producer,
// warp 1 TMEM owner + UMMA issuer, warps 2..5 softmax + epilogue (one query
// row per thread).  Per 64-key block b:
//   S = Q K^T : UMMA M=128 N=64 K=32 (two K steps), TMEM cols [0,64)
//   P = 2^(S*scale*log2e + mask*log2e - m) -> TMEM P[b & 1] (32 columns)
//   O += P V  : UMMA M=128 N=32 K=64, A = P from TMEM, V MN-major, into
//               O[item & 1] (32 columns)
// The mask may instead be a full additive bias per (sequence, head, query,
// key): the decoder's box relative-position bias on its image cross attention
// (src/decoder.cpp:401-418, :457-465), read row by row by the thread that owns
// the query.  Keys past kv_len (the last, ragged block) are masked like -inf
// mask entries; query rows past q_len run on zero-filled Q rows and are not
// stored.  TMEM: S 64 + O 2x32 + P 2x32 = 192 of the 256 columns allocated,
// two CTAs per SM.
#include <math.h>

#include "kernels.h"
#include "ptx.cuh"

namespace s3t {

namespace {

constexpr int kBQ = 128, kBKV = 64, kD = 32, kHeadsE = 8, kModelE = kHeadsE * kD, kKVStages = 4;
constexpr uint32_t kQBytes = kBQ * kD * 2;      // 8 KB
constexpr uint32_t kKVBytes = kBKV * kD * 2;    // 4 KB (each of K, V)
constexpr size_t kMhaSmem = 2 * kQBytes + 2 * kKVStages * kKVBytes + 1024 + 256;
constexpr uint32_t kMhaTmemCols = 256;          // S [0,64), O0 [64,96), O1 [96,128), P0 [128,160), P1 [160,192)
constexpr uint32_t kTmemO = 64, kTmemP = 128;
constexpr int kCtasPerSm = 2;
constexpr float kLog2e = 1.4426950408889634f;

template <int BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (BF16) return pack_bf162(a, b);
    else return pack_half2(a, b);
}

struct Item {
    int qt, head, seq, split;
    int j0, j1;   // key blocks [j0, j1) of this item
};

__device__ __forceinline__ Item item_of(int w, int n_qt, int splits, int nkv) {
    Item it;
    it.split = w % splits;
    const int w2 = w / splits;
    it.qt = w2 % n_qt;
    const int r = w2 / n_qt;
    it.head = r % kHeadsE;
    it.seq = r / kHeadsE;
    it.j0 = int(int64_t(it.split) * nkv / splits);
    it.j1 = int(int64_t(it.split + 1) * nkv / splits);
    return it;
}

// Index of a row's partial in the scratch buffers (splits > 1).
__device__ __forceinline__ int64_t partial_index(int seq, int head, int qt, int row, int split, int n_qt,
                                                 int splits) {
    return (int64_t((seq * kHeadsE + head) * n_qt + qt) * kBQ + row) * splits + split;
}

// MASK: a mask or bias array was given (compiled apart, so the unmasked
// self attention keeps its registers for the softmax).
template <int BF16, bool MASK>
__global__ void __launch_bounds__(192, kCtasPerSm)
    mha32_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                 const __grid_constant__ CUtensorMap tmV, const MhaArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                              // 2 buffers
    uint8_t* sK = sQ + 2 * kQBytes;
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
    uint64_t* o_free = o_done + 2;                   // [2]
    uint64_t* drain = o_free + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkv = (a.kv_len + kBKV - 1) / kBKV;
    const int n_qt = (a.q_len + kBQ - 1) / kBQ;
    const int splits = a.splits;
    const int n_items = n_qt * kHeadsE * a.batch * splits;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(q_full + i, 1);
            mbar_init(q_empty + i, 1);
            mbar_init(o_free + i, 4);
            mbar_init(o_done + i, 1);
            mbar_init(p_full + i, 4);
        }
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
        tmem_alloc(tmem_slot, kMhaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tS = tmem;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t armed = 0, armed_parity = 0, q_armed = 0, q_parity = 0;
            bool ok = true;
            int b = 0;   // global block counter of this CTA
            int li = 0;  // local item counter
            for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++li) {
                const Item it = item_of(w, n_qt, splits, nkv);
                const int x = it.head * kD;   // column of this head: 64-byte aligned
                const int qb = li & 1;
                const uint32_t qph = (li >> 1) & 1;
                if (!mbar_wait(q_empty + qb, qph ^ 1, a.status, kErrTimeoutProducer, abort_flag)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(q_full + qb, kQBytes);
                tma_load_3d(sQ + qb * kQBytes, &tmQ, q_full + qb, x, it.qt * kBQ, it.seq);
                q_armed |= 1u << qb;
                q_parity = (q_parity & ~(1u << qb)) | (qph << qb);
                for (int j = it.j0; j < it.j1; ++j, ++b) {
                    const int s = b % kKVStages;
                    const uint32_t ph = (b / kKVStages) & 1;
                    if (!mbar_wait(kv_empty + s, ph ^ 1, a.status, kErrTimeoutProducer, abort_flag)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(kv_full + s, 2 * kKVBytes);
                    tma_load_3d(sK + s * kKVBytes, &tmK, kv_full + s, x, j * kBKV, it.seq);
                    tma_load_3d(sV + s * kKVBytes, &tmV, kv_full + s, x, j * kBKV, it.seq);
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
            // Key blocks of this CTA's li-th item, and of all its items.
            auto count_of = [&](int li_) -> int {
                const int w = int(blockIdx.x) + li_ * int(gridDim.x);
                if (w >= n_items) return 0;
                const Item it = item_of(w, n_qt, splits, nkv);
                return it.j1 - it.j0;
            };
            int total = 0;
            for (int w = blockIdx.x, li_ = 0; w < n_items; w += gridDim.x, ++li_) total += count_of(li_);
            bool ok = true, issued = false;
            // Descriptors are built once.  A K step of 16 advances the start
            // address field by 32 bytes (2) for the K-major Q and K tiles, and
            // by 16 key rows of 64 bytes (64) for the MN-major V tile.
            const uint64_t dQ0 = umma_desc_sw64(smem_u32(sQ), 16, 512);
            const uint64_t dQ1 = umma_desc_sw64(smem_u32(sQ + kQBytes), 16, 512);
            const uint64_t dK0 = umma_desc_sw64(smem_u32(sK), 16, 512);
            const uint64_t dV0 = umma_desc_sw64(smem_u32(sV), kKVBytes, 512);
            constexpr uint64_t kStageStep = kKVBytes >> 4;
            // State of the next S block to issue (block counter, key block, item, ring stage/phase).
            int sb = 0, sj = 0, sli = 0, ss = 0, scnt = count_of(0);
            uint32_t sph = 0;
            auto issue_s = [&]() -> bool {
                const int qb = sli & 1;
                if (sj == 0 && !mbar_wait(q_full + qb, (sli >> 1) & 1, a.status, kErrTimeoutMma, abort_flag))
                    return false;
                if (!mbar_wait(kv_full + ss, sph, a.status, kErrTimeoutMma, abort_flag)) return false;
                if (sb > 0 && !mbar_wait(s_free, (sb - 1) & 1, a.status, kErrTimeoutMma, abort_flag)) return false;
                tc_fence_after();
                const uint64_t dq = qb ? dQ1 : dQ0, dk = dK0 + uint64_t(ss) * kStageStep;
#pragma unroll
                for (int k = 0; k < kD / 16; ++k) umma_f16_ss(tS, dq + 2 * k, dk + 2 * k, idS, k != 0);
                umma_commit(s_full);
                if (sj == scnt - 1) umma_commit(q_empty + qb);   // Q buffer reusable once these S complete
                issued = true;
                ++sb;
                if (++sj == scnt) { sj = 0; ++sli; scnt = count_of(sli); }
                if (++ss == kKVStages) { ss = 0; sph ^= 1; }
                return true;
            };
            if (total > 0) ok = issue_s();
            int j = 0, li = 0, s = 0, cnt = count_of(0);
            for (int b = 0; ok && b < total; ++b) {
                if (b + 1 < total && !issue_s()) {
                    ok = false;
                    break;
                }
                const int ob = li & 1;
                if (!mbar_wait(p_full + (b & 1), (b >> 1) & 1, a.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                if (j == 0 && !mbar_wait(o_free + ob, ((li >> 1) & 1) ^ 1, a.status, kErrTimeoutMma, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint64_t dv = dV0 + uint64_t(s) * kStageStep;
                const uint32_t tO = tmem + kTmemO + ob * kD;
                const uint32_t tP = tmem + kTmemP + (b & 1) * 32;
#pragma unroll
                for (int k = 0; k < kBKV / 16; ++k) umma_f16_ts(tO, tP + 8 * k, dv + 64 * k, idO, (j | k) != 0);
                umma_commit(kv_empty + s);
                umma_commit(o_done + (b & 1));
                if (++j == cnt) { j = 0; ++li; cnt = count_of(li); }
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
        constexpr bool any_mask = MASK;
        const bool ragged = (a.kv_len % kBKV) != 0;
        // m_run is the (log2-domain) max the P values of this row are taken
        // relative to.  It is only raised when a block's max exceeds it by
        // more than kRescaleSlack, so O is rescaled in TMEM rarely; P values
        // stay <= 2^kRescaleSlack, and O / l is unchanged by the choice.
        // m_run stays -inf while every key seen so far was masked.
        constexpr float kRescaleSlack = 8.0f;
        bool ok = true;
        int b = 0, li = 0;
        for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x, ++li) {
            const Item it = item_of(w, n_qt, splits, nkv);
            const int ob = li & 1;
            const uint32_t tO = tmem + kTmemO + ob * kD;
            const float* mask_row = nullptr;
            if (any_mask && a.bias) {
                // Query rows past q_len are computed but never stored; they read the last row.
                const int qi = min(it.qt * kBQ + row, a.q_len - 1);
                mask_row = a.key_mask + ((int64_t(it.seq) * kHeadsE + it.head) * a.q_len + qi) * a.kv_len;
            } else if (any_mask) {
                mask_row = a.key_mask + int64_t(it.seq) * a.kv_len;
            }
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = it.j0; j < it.j1; ++j, ++b) {
                // A block with masked keys (a mask was given, or keys past
                // kv_len) reads its 64 mask entries before waiting for S, so
                // the loads overlap the wait; -inf marks a key that takes no
                // part.
                const bool masked_blk = any_mask || (ragged && j == nkv - 1);
                float mv[MASK ? kBKV : 1];
                if constexpr (MASK) {
                    const int k0 = j * kBKV;
                    if (any_mask && k0 + kBKV <= a.kv_len && (reinterpret_cast<uintptr_t>(mask_row + k0) & 15) == 0) {
                        const float4* m4 = reinterpret_cast<const float4*>(mask_row + k0);
#pragma unroll
                        for (int c = 0; c < kBKV / 4; ++c) {
                            const float4 t = __ldg(m4 + c);
                            mv[4 * c] = t.x;
                            mv[4 * c + 1] = t.y;
                            mv[4 * c + 2] = t.z;
                            mv[4 * c + 3] = t.w;
                        }
                    } else {
#pragma unroll
                        for (int c = 0; c < kBKV; ++c) {
                            const int kk = k0 + c;
                            mv[c] = kk < a.kv_len ? __ldg(mask_row + kk) : -INFINITY;
                        }
                    }
                }
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

                // Scores in the log2 domain are r * sc.  A masked block is
                // converted in place first: s*scale*log2e + mask*log2e, or
                // -inf for a key that takes no part; it then uses sc = 1.
                float sc = sl2;
                if constexpr (MASK) {
#pragma unroll
                    for (int c = 0; c < kBKV; ++c)
                        r[c] = __float_as_uint(mv[c] != -INFINITY ? fmaf(__uint_as_float(r[c]), sl2, mv[c] * kLog2e)
                                                                 : -INFINITY);
                    sc = 1.0f;
                } else if (masked_blk) {
                    // No mask: only the keys past kv_len of the last block drop out.
                    const int k0 = j * kBKV;
#pragma unroll
                    for (int c = 0; c < kBKV; ++c)
                        r[c] = __float_as_uint(k0 + c < a.kv_len ? __uint_as_float(r[c]) * sl2 : -INFINITY);
                    sc = 1.0f;
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
                    fmax3(fmax3(acc[0], acc[1], acc[2]), fmax3(acc[3], acc[4], acc[5]), fmaxf(acc[6], acc[7])) * sc;
                const bool raise = mx > m_run + kRescaleSlack;
                const float m_new = raise ? mx : m_run;
                const float alpha = raise ? ex2_approx(m_run - m_new) : 1.0f;
                // While no key of the row has counted yet every P is 0; a
                // finite offset keeps -inf - (-inf) out of the exponent.
                const float m_use = m_new == -INFINITY ? 0.0f : m_new;
                uint32_t pk[32];
                float2 sums[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                const float2 scx2 = make_float2(sc, sc), negm = make_float2(-m_use, -m_use);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float2 t = __ffma2_rn(make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                                                scx2, negm);
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
                if (j > it.j0 && __any_sync(0xffffffffu, raise)) {
                    if (!mbar_wait(o_done + ((b - 1) & 1), ((b - 1) >> 1) & 1, a.status, kErrTimeoutEpilogue,
                                   abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint32_t o[32];
                    tmem_ld32(tO + lane_off, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(tO + lane_off, o);
                    tmem_wait_st();
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
            // Item epilogue: O / l (0 for a row whose keys were all masked).
            tc_fence_after();
            uint32_t o[32];
            tmem_ld32(tO + lane_off, o);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free + ob);
            const int qi = it.qt * kBQ + row;
            if (splits > 1 && qi < a.q_len) {
                // One key range of the row: unnormalised O and (m, l), merged by mha32_combine.
                const int64_t p = partial_index(it.seq, it.head, it.qt, row, it.split, n_qt, splits);
                float4* dst = reinterpret_cast<float4*>(a.ws_o + p * kD);
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    dst[c] = make_float4(__uint_as_float(o[4 * c]), __uint_as_float(o[4 * c + 1]),
                                         __uint_as_float(o[4 * c + 2]), __uint_as_float(o[4 * c + 3]));
                *reinterpret_cast<float2*>(a.ws_ml + 2 * p) = make_float2(m_run, l_run);
            } else if (qi < a.q_len) {
                const float inv = l_run == 0.0f ? 0.0f : 1.0f / l_run;
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(o[i]) * inv;
                const int64_t off = (int64_t(it.seq) * a.q_len + qi) * kModelE + it.head * kD;
                if (a.out_f16) {
                    uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off);
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        dst[c] = make_uint4(pack2<BF16>(v[8 * c], v[8 * c + 1]), pack2<BF16>(v[8 * c + 2], v[8 * c + 3]),
                                            pack2<BF16>(v[8 * c + 4], v[8 * c + 5]),
                                            pack2<BF16>(v[8 * c + 6], v[8 * c + 7]));
                } else {
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
                    for (int c = 0; c < 8; ++c) dst[c] = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
                }
            }
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kMhaTmemCols);
    }
}

// Merges the key-range partials of each (sequence, head, query row):
// O = sum_s O_s 2^(m_s - M) / sum_s l_s 2^(m_s - M), M = max_s m_s; a row
// whose every range saw only masked keys (all m_s = -inf) is 0.  One thread
// per (sequence, row, head), heads fastest, so a warp writes 4 whole rows.
__global__ void __launch_bounds__(256) mha32_combine(const MhaArgs a) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = int64_t(a.batch) * a.q_len * kHeadsE;
    if (t >= total) return;
    const int head = int(t % kHeadsE);
    const int64_t r = t / kHeadsE;
    const int qi = int(r % a.q_len);
    const int seq = int(r / a.q_len);
    const int n_qt = (a.q_len + kBQ - 1) / kBQ;
    const int splits = a.splits;
    const int64_t p0 = partial_index(seq, head, qi / kBQ, qi % kBQ, 0, n_qt, splits);
    float m_max = -INFINITY;
    for (int s = 0; s < splits; ++s) m_max = fmaxf(m_max, a.ws_ml[2 * (p0 + s)]);
    float acc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) acc[d] = 0.0f;
    float l = 0.0f;
    if (m_max != -INFINITY) {
        for (int s = 0; s < splits; ++s) {
            const float m = a.ws_ml[2 * (p0 + s)];
            if (m == -INFINITY) continue;
            const float w = exp2f(m - m_max);
            l = fmaf(w, a.ws_ml[2 * (p0 + s) + 1], l);
            const float4* src = reinterpret_cast<const float4*>(a.ws_o + (p0 + s) * kD);
#pragma unroll
            for (int c = 0; c < kD / 4; ++c) {
                const float4 o = src[c];
                acc[4 * c] = fmaf(w, o.x, acc[4 * c]);
                acc[4 * c + 1] = fmaf(w, o.y, acc[4 * c + 1]);
                acc[4 * c + 2] = fmaf(w, o.z, acc[4 * c + 2]);
                acc[4 * c + 3] = fmaf(w, o.w, acc[4 * c + 3]);
            }
        }
    }
    const float inv = l == 0.0f ? 0.0f : 1.0f / l;
    const int64_t off = (int64_t(seq) * a.q_len + qi) * kModelE + head * kD;
    if (a.out_f16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + off);
        for (int c = 0; c < 4; ++c) {
            uint32_t w4[4];
            for (int i = 0; i < 4; ++i) {
                const float x0 = acc[8 * c + 2 * i] * inv, x1 = acc[8 * c + 2 * i + 1] * inv;
                w4[i] = a.bf16 ? pack_bf162(x0, x1) : pack_half2(x0, x1);
            }
            dst[c] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
    } else {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + off);
#pragma unroll
        for (int c = 0; c < kD / 4; ++c)
            dst[c] = make_float4(acc[4 * c] * inv, acc[4 * c + 1] * inv, acc[4 * c + 2] * inv, acc[4 * c + 3] * inv);
    }
}

}  // namespace

cudaError_t mha32_prepare() {
    const void* fns[4] = {reinterpret_cast<const void*>(mha32_kernel<0, false>),
                          reinterpret_cast<const void*>(mha32_kernel<1, false>),
                          reinterpret_cast<const void*>(mha32_kernel<0, true>),
                          reinterpret_cast<const void*>(mha32_kernel<1, true>)};
    for (const void* f : fns) {
        const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMhaSmem));
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_mha32(const MhaArgs& a, cudaStream_t stream) {
    if (a.batch <= 0 || a.q_len <= 0 || a.kv_len <= 0 || !a.q || !a.k || !a.v || !a.out) return cudaErrorInvalidValue;
    // TMA bases and the vector stores of the epilogue need 16-byte alignment.
    if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
         reinterpret_cast<uintptr_t>(a.out)) & 15)
        return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(a.key_mask) & 3) return cudaErrorInvalidValue;
    const CUtensorMapDataType dt = a.bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    // [batch][len][256]; a box is 32 columns (one head, 64 bytes) by 128 or 64
    // rows of one sequence.
    CUtensorMap tq, tk, tv;
    const uint64_t nb = uint64_t(a.batch);
    if (!make_tmap_3d(&tq, a.q, dt, 2, kModelE, uint64_t(a.q_len), nb, kD, kBQ, CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    if (!make_tmap_3d(&tk, a.k, dt, 2, kModelE, uint64_t(a.kv_len), nb, kD, kBKV, CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    if (!make_tmap_3d(&tv, a.v, dt, 2, kModelE, uint64_t(a.kv_len), nb, kD, kBKV, CU_TENSOR_MAP_SWIZZLE_64B))
        return cudaErrorInvalidValue;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t items64 = int64_t((a.q_len + kBQ - 1) / kBQ) * kHeadsE * a.batch;
    if (items64 > (int64_t(1) << 30)) return cudaErrorInvalidValue;
    // Too few query tiles to fill the GPU (two CTAs per SM) and enough keys to
    // pay for the merge (16 blocks or more): split each tile's key blocks into
    // ranges of at least two blocks, about one wave in all.
    const int slots = sms * kCtasPerSm;
    const int nkv = (a.kv_len + kBKV - 1) / kBKV;
    int splits = 1;
    if (items64 * 2 <= slots && nkv >= 16) {
        const int want = int((slots + items64 - 1) / items64);
        splits = want < nkv / 2 ? want : nkv / 2;
    }
    MhaArgs b = a;
    b.splits = splits;
    b.ws_o = b.ws_ml = nullptr;
    void* ws = nullptr;
    if (splits > 1) {
        // Stream-ordered scratch for the partials, freed after the merge.
        const size_t rows = size_t(items64) * kBQ * splits;
        const size_t bytes_o = rows * kD * sizeof(float);
        cudaError_t e = cudaMallocAsync(&ws, bytes_o + rows * 2 * sizeof(float), stream);
        if (e != cudaSuccess) return e;
        b.ws_o = static_cast<float*>(ws);
        b.ws_ml = reinterpret_cast<float*>(static_cast<char*>(ws) + bytes_o);
    }
    const int n_items = int(items64) * splits;
    const int grid = n_items < slots ? n_items : slots;
    const bool masked = b.key_mask != nullptr;
    if (b.bf16 && masked)
        mha32_kernel<1, true><<<grid, 192, kMhaSmem, stream>>>(tq, tk, tv, b);
    else if (b.bf16)
        mha32_kernel<1, false><<<grid, 192, kMhaSmem, stream>>>(tq, tk, tv, b);
    else if (masked)
        mha32_kernel<0, true><<<grid, 192, kMhaSmem, stream>>>(tq, tk, tv, b);
    else
        mha32_kernel<0, false><<<grid, 192, kMhaSmem, stream>>>(tq, tk, tv, b);
    cudaError_t e = cudaGetLastError();
    if (splits > 1) {
        if (e == cudaSuccess) {
            const int64_t threads = int64_t(a.batch) * a.q_len * kHeadsE;
            mha32_combine<<<unsigned((threads + 255) / 256), 256, 0, stream>>>(b);
            e = cudaGetLastError();
        }
        const cudaError_t f = cudaFreeAsync(ws, stream);
        if (e == cudaSuccess) e = f;
    }
    return e;
}

}  // namespace s3t
