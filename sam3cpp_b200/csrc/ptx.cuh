// Blackwell (sm_100a) primitives used by the trunk kernels: mbarriers with
// bounded waits, TMA tile loads, and tcgen05 (TMEM alloc, UMMA issue/commit,
// TMEM <-> register moves).  Everything is inline PTX written for this project.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define S3T_DEV __device__ __forceinline__

namespace s3t {

// A wait that has not completed after this many nanoseconds is treated as a
// hang: the kernel records the error, drains what it started, and returns.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

S3T_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

S3T_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

S3T_DEV void report_error(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

// ------------------------------------------ programmatic dependent launch ---
// griddep_wait: block until every grid this one depends on has completed and
// its memory operations are visible; returns at once when the grid was
// launched without programmatic stream serialization.  Every trunk kernel
// calls it before its first read of a predecessor's output and before its
// first global write.  griddep_launch_dependents: let the next grid of the
// stream be scheduled (its CTAs run their prologue on free SMs, then wait).
S3T_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
S3T_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------- mbarrier ---

S3T_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

S3T_DEV void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

S3T_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

S3T_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

S3T_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (after
// recording `code` in *status) if the phase did not complete in time, or if
// another role of the CTA already gave up (*abort set).
S3T_DEV bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* status, int code, volatile int* abort,
                             uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (abort && *abort) return false;
            if (globaltimer() - t0 > limit_ns) {
                report_error(status, code);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}

S3T_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code, volatile int* abort) {
    return mbar_wait_limit(bar, parity, status, code, abort, kWaitLimitNs);
}

// ------------------------------------------------------ global flags ---
// A flag in global memory set by one CTA and awaited by another of the same
// grid (both resident): release store / acquire load at GPU scope.

S3T_DEV void flag_release(int* f, int v) {
    asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

S3T_DEV int flag_acquire(const int* f) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    return v;
}

// Bounded wait until *f != 0; false (with `code` recorded and *abort set) on
// timeout, or when another role of the CTA already gave up.
S3T_DEV bool flag_wait(const int* f, int* status, int code, volatile int* abort) {
    if (flag_acquire(f)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (flag_acquire(f)) return true;
        __nanosleep(32);
        if ((i & 63u) == 0) {
            if (abort && *abort) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                report_error(status, code);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------ TMA ---

S3T_DEV void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

S3T_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

S3T_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// ------------------------------------------------- CTA pair (cluster of 2) ---

S3T_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared variable in CTA `rank`.
S3T_DEV uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

S3T_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (possibly the
// peer's), with the default release-at-CTA-scope semantics: enough to order
// this warp's completed TMEM reads (tcgen05.fence::before_thread_sync) before
// the MMA that reuses the accumulator, without waiting for the warp's global
// stores to drain as a cluster-scope release would.
S3T_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

S3T_DEV void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier of the pair's leader CTA (no multicast: one destination).
S3T_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t leader_bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(leader_bar), "r"(x), "r"(y)
        : "memory");
}

// Bring a tile of a tensor map into L2 (no shared-memory destination, no
// completion to wait for).
S3T_DEV void tma_prefetch_l2_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (UMMA).
// Tiled bulk store shared -> global (bulk-group completion).  Rows or
// columns of the box outside the tensor are not written.
S3T_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}

S3T_DEV void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

S3T_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N bulk groups of this thread still read shared memory.
template <int N>
S3T_DEV void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every bulk group of this thread has completed.
S3T_DEV void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

S3T_DEV void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// -------------------------------------------------------------- tcgen05 ---

S3T_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

S3T_DEV void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

S3T_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

S3T_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
S3T_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem) * B(smem)^T, kind::f16 (fp16/bf16 in, fp32 accumulate).
S3T_DEV void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]: A (M x K, K-major) is read from tensor
// memory, row m in lane m, two 16-bit K elements per 32-bit column.
S3T_DEV void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive (once) on an mbarrier when all previously issued UMMAs of this thread complete.
S3T_DEV void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Two-SM variants (cta_group::2): the pair's TMEM is allocated by one warp in
// each CTA; the leader CTA issues the MMA, which reads A and B halves from
// both CTAs' shared memory at the same offsets and writes each CTA's TMEM.
S3T_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

S3T_DEV void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

S3T_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

S3T_DEV void umma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the mbarrier at this offset in every CTA of `cta_mask` when
// the leader's previously issued pair MMAs complete.
S3T_DEV void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(cta_mask)
        : "memory");
}

// Instruction descriptor, kind::f16: D=f32, A/B = f16 (fmt 0) or bf16 (fmt 1),
// A K-major, B K-major (b_mn_major=0) or MN-major (1), shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N, int ab_fmt, int b_mn_major) {
    return (1u << 4)                              // D format: f32
           | (uint32_t(ab_fmt) << 7)              // A format
           | (uint32_t(ab_fmt) << 10)             // B format
           | (0u << 15)                           // A K-major
           | (uint32_t(b_mn_major) << 16)         // B major
           | (uint32_t(N >> 3) << 17)             // N / 8
           | (uint32_t(M >> 4) << 24);            // M / 16
}

// Shared-memory matrix descriptor, 128-byte swizzle (tile base 1024-aligned).
// K-major: rows of 128 B (64 halves), 8-row core groups 1024 B apart (SBO).
// MN-major: rows of 128 B along MN, 8 K-rows per 1024 B group (SBO); LBO is
// the byte distance between 64-element MN chunks.
S3T_DEV uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
    d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= uint64_t(1) << 46;   // descriptor version (sm_100)
    d |= uint64_t(2) << 61;   // SWIZZLE_128B
    return d;
}

// Shared-memory matrix descriptor, 64-byte swizzle (tile base 1024-aligned).
// K-major: rows of 64 B (32 halves), 8-row core groups 512 B apart (SBO).
// MN-major: rows of 64 B along MN, 8 K-rows per 512 B group (SBO); LBO is
// the byte distance between 32-element MN chunks.
S3T_DEV uint64_t umma_desc_sw64(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
    d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= uint64_t(1) << 46;   // descriptor version (sm_100)
    d |= uint64_t(4) << 61;   // SWIZZLE_64B
    return d;
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// row (lane base + i), columns [col, col+32).
S3T_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

S3T_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

S3T_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

S3T_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Three-input max (sm_100).
S3T_DEV float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

S3T_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
S3T_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x on the SFU (hardware approximation; inputs far below -126 flush to 0).
S3T_DEV float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 1/x on the SFU (hardware approximation).
S3T_DEV float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU with the error function of Abramowitz & Stegun, Handbook of
// Mathematical Functions, formula 7.1.26 (|erf error| <= 1.5e-7):
// erf(z) = 1 - (a1 t + ... + a5 t^5) exp(-z^2), t = 1/(1 + p z), z >= 0.
// Same function as ggml_vec_gelu_erf_f32: 0.5 x (1 + erf(x / sqrt 2)).
S3T_DEV float gelu_erf_as(float x) {
    // GELU(x) = relu(x) - |x| Q(x), Q = erfc(|x| / sqrt 2) / 2 = 0.5 poly(t) t exp(-x^2 / 2)
    const float ax = fabsf(x);
    const float t = rcp_approx(fmaf(0.3275911f * 0.70710678118654752f, ax, 1.0f));
    float q = fmaf(0.5f * 1.061405429f, t, 0.5f * -1.453152027f);
    q = fmaf(q, t, 0.5f * 1.421413741f);
    q = fmaf(q, t, 0.5f * -0.284496736f);
    q = fmaf(q, t, 0.5f * 0.254829592f);
    const float e = ex2_approx(x * x * -0.72134752044448170f);   // exp(-x^2 / 2)
    return fmaf(-(ax * t) * q, e, fmaxf(x, 0.f));
}

// Two lanes of gelu_erf_as with packed f32x2 arithmetic (same operations,
// round-to-nearest, so each lane's result equals the scalar one).
S3T_DEV float2 gelu_erf_as2(float2 x) {
    const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
    const float2 d = __ffma2_rn(make_float2(0.3275911f * 0.70710678118654752f, 0.3275911f * 0.70710678118654752f), ax,
                                make_float2(1.0f, 1.0f));
    const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    // -Q(x) / (|x| t exp(-x^2/2)) as a polynomial in t (coefficients negated).
    float2 q = __ffma2_rn(make_float2(-0.5f * 1.061405429f, -0.5f * 1.061405429f), t,
                          make_float2(0.5f * 1.453152027f, 0.5f * 1.453152027f));
    q = __ffma2_rn(q, t, make_float2(-0.5f * 1.421413741f, -0.5f * 1.421413741f));
    q = __ffma2_rn(q, t, make_float2(0.5f * 0.284496736f, 0.5f * 0.284496736f));
    q = __ffma2_rn(q, t, make_float2(-0.5f * 0.254829592f, -0.5f * 0.254829592f));
    const float2 s = __fmul2_rn(__fmul2_rn(x, x), make_float2(-0.72134752044448170f, -0.72134752044448170f));
    const float2 e = make_float2(ex2_approx(s.x), ex2_approx(s.y));
    const float2 u = __fmul2_rn(__fmul2_rn(ax, t), q);
    return __ffma2_rn(u, e, make_float2(fmaxf(x.x, 0.f), fmaxf(x.y, 0.f)));
}

S3T_DEV uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

S3T_DEV uint32_t pack_bf162(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// The Q8_0 activation rounding ggml's CPU mul_mat applies before a Q8_0 dot
// (ggml-cpu/arch/x86/quants.c quantize_row_q8_0): per 32-block, d = amax/127
// kept as fp16, q = round-half-even(x * 127/amax); returns the dequantized
// block value q*d in place.  IEEE division is used (no fast-math).
S3T_DEV void q8_0_fake_quant32(float (&v)[32]) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = __half2float(__float2half_rn(__fdiv_rn(amax, 127.f)));
    const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = rintf(__fmul_rn(v[i], id)) * d;
}

}  // namespace s3t
