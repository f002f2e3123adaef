// qkv_prefill.cu -- kernel D: chunked causal prefill attention over the paged q8_0 cache on the
// 5th-generation tensor cores (tcgen05.mma kind::f16, fp32 accumulators in tensor memory).
//
// Semantics follow ggml's CPU flash_attn_ext with q8_0 K/V (the reference's prefill call,
// src/qwfn_graph.cpp:417-476, with the causal mask of src/qwfn_engine.cpp:1238-1274): every query
// row is quantised to q8_0 (ggml's quantize_row_q8_0 rounding), scores are q.k * scale, softmax
// in fp32, V dequantised.  On the tensor cores the operands are fp16: a query element becomes
// fp16(d_q * q) and a cache element fp16(d * q) (one rounding each; the int8 and fp16 scale are
// exact), products accumulate in fp32.
//
// Tile: 128 rows = (128 / G) query tokens x the G q-heads sharing one KV head, so each K/V tile
// is dequantised once for all of them.  Two tiles of a KV head run on a CTA pair (a cluster of
// two, one CTA per SM) whose MMAs are tcgen05.mma.cta_group::2 with M = 256: each CTA holds its
// query tile and dequantises half of every K tile (64 keys) and V tile (128 dims) into its own
// shared memory.  A pair runs a contiguous run of segments (pair tile, KV range) from a host plan
// that gives every pair the same number of KV tiles; each segment leaves a partial record per
// tile, merged by k_prefill_merge.  17 warps per CTA:
//   warp 0      TMEM allocation; in the leader one thread issues all MMAs, in the follower one
//               thread copies its query tiles and reports them to the leader
//   warps 1-8   softmax in two halves of the S row's 128 keys: thread r owns row r (TMEM lane
//               r): its half's S from TMEM, causal (and kept-block) mask, online softmax with a
//               lazily raised reference max (O rescaled only when the row max grows by more
//               than 2^8), P as fp16 over the half's S columns
//   warps 9-16  K producers (9-12) and V producers (13-16): read q8_0 tiles from the pages and
//               dequantise to fp16 into the 128-byte-swizzled layouts the MMAs read, in a ring
//               of five 32 KiB slots freed by the commits of the MMAs that read them.
// Per KV tile j (S buffer b = j % 2): S_b = Q K_j^T (N = 128), then after the softmax wrote P_j:
// O += P_j V_j.  S_{j+1} is issued before PV_j so the tensor core works while the softmax runs.
// Every wait is bounded (ST_TIMEOUT, then all roles leave their loops, the issuing thread drains
// its MMAs and the CTAs free their TMEM).
#include "qkv.h"
#include "qkv_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

namespace qkv {
namespace pf {

// warps: 0 MMA issue, 1 .. 4 SMX_GROUPS softmax, then 4 NGRP K producers and 4 NGRP V producers
constexpr int SMX_GROUPS = 2;          // softmax warp groups (column halves of S)
constexpr int NGRP       = 1;          // 128-thread producer groups per operand
constexpr int PW_K       = 1 + 4 * SMX_GROUPS;
constexpr int PW_V       = PW_K + 4 * NGRP;
constexpr int NTHR       = 32 * (PW_V + 4 * NGRP);
constexpr int KT   = PF_KT;            // keys per KV tile (N of S, K of PV): two page tiles
static_assert(KT == 2 * TILE_TOK, "a KV tile is two 64-token page tiles");
// shared memory map, offsets from a 1024-byte aligned base
constexpr int SM_Q       = 0;          // A of S: [4 k-atoms][128 rows][128 B]
constexpr int SM_RING    = 65536;      // NSLOT x 32 KiB slots: this CTA's half of a K tile (64 keys x 256 dims) or V tile (128 dims x 128 keys)
constexpr int NSLOT      = 5;
constexpr int SLOT_BYTES = 32768;
constexpr int SM_BAR     = SM_RING + NSLOT * SLOT_BYTES;
constexpr int SM_PMAX    = SM_BAR + 256;   // [2 S buffers][2 softmax halves][128 rows] bf16: the halves' row maxima
constexpr int SMEM_BYTES = SM_PMAX + 2 * 2 * 128 * 2 + 1024;
// tensor memory columns: O, then two S buffers (P of a tile is stored over its S)
constexpr uint32_t TM_O = 0, TM_S = 256, TM_COLS = 512;
constexpr uint64_t WAIT_NS = 200ull * 1000 * 1000;

// Barriers.  The MMAs of a CTA pair are issued by the pair's leader (cluster rank 0); the
// barriers the issuing thread waits on live in the leader and both CTAs arrive on them (the
// follower through its cluster address); the MMAs' commits arrive on the barrier of the same
// name in both CTAs (multicast).
struct Bars {
    uint64_t slot_full[NSLOT];   // leader: producers of both CTAs (2 x 128 NGRP arrivals): the pair's slot u filled
    uint64_t slot_free[NSLOT];   // both: commit after the MMAs reading slot u
    uint64_t s_full[2];          // both: commit after S_j
    uint64_t s_read[2];          // both, local: the CTA's softmax threads (256 arrivals) posted their halves' maxima of S_j
    uint64_t p_full[2];          // leader: softmax of both CTAs (2 x 256 arrivals): P_j stored (and O rescaled)
    uint64_t pv_done[2];         // both: commit after PV_j
    uint64_t q_full;             // both, local: the CTA's query tile landed (expect_tx)
    uint64_t q_peer;             // leader: the follower's query tile landed (1 arrival)
    uint64_t q_empty;            // both: commit after the last S of a segment
    uint64_t drain;              // leader: commit before exit
    uint32_t tmem;
    int32_t  abort;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase completes (or ~20 us
// pass) instead of spinning on issue slots the working warps need.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Phase timestamps for latency analysis, compiled only with -DQKV_TIMELINE (the product build
// never defines it): g_pf_tl[CTA][role][tile][phase], written on every launch by one thread of
// each role for the first PF_TL_TILES KV tiles of the CTA.  Roles: 0 / 1 softmax halves (warps 1
// and 5), 2 MMA issue (leader), 3 K producers (warp 9), 4 V producers (warp 13).
// qkv_pf_tl_read copies the table out.
#ifdef QKV_TIMELINE
constexpr int PF_TL_CTAS = 160, PF_TL_TILES = 16, PF_TL_PH = 6;
__device__ unsigned long long g_pf_tl[PF_TL_CTAS][5][PF_TL_TILES][PF_TL_PH];
#define PF_TL(cond, role, idx, ph)                                                                   \
    do {                                                                                             \
        if ((cond) && (idx) >= 0 && (idx) < PF_TL_TILES && blockIdx.x < PF_TL_CTAS)                  \
            g_pf_tl[blockIdx.x][role][idx][ph] = global_ns();                                        \
    } while (0)
#else
#define PF_TL(cond, role, idx, ph) do { } while (0)
#endif
// Non-blocking test of the phase of `parity`.
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of `parity` to complete.  Returns false when another role aborted or the
// wait ran past WAIT_NS (then it raises the abort flag and ST_TIMEOUT itself).
__device__ __noinline__ bool wait_bar_slow(uint64_t *bar, uint32_t parity, Bars *B, int32_t *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
#pragma unroll 1
        for (int i = 0; i < 4; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (*(volatile int32_t *)&B->abort) return false;
        if (global_ns() - t0 > WAIT_NS) {
            *(volatile int32_t *)&B->abort = 1;
            atomicOr(status, ST_TIMEOUT);
            return false;
        }
    }
}
// A phase that already completed is seen inline, without the call.
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, Bars *B, int32_t *status) {
    return mbar_test(bar, parity) || wait_bar_slow(bar, parity, B, status);
}
// Bounded wait that ignores the abort flag (draining in-flight asynchronous work before exit).
__device__ __noinline__ void drain_bar(uint64_t *bar, uint32_t parity, int32_t *status) {
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > WAIT_NS) {
            atomicOr(status, ST_TIMEOUT);
            return;
        }
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes apart.
// Fields: start address >> 4 [0,14), leading offset >> 4 [16,30) (unused by swizzled K-major),
// stride offset >> 4 [32,46), fixed 0b001 [46,49), base offset 0, swizzle mode 2 (128 B) [61,64).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: D f32 (bit 4), A/B f16 (format 0), both K-major, N >> 3 at
// bit 17, M >> 4 at bit 24.  The pair's MMAs are M = 256: rows 0-127 in the leader, 128-255 in
// the follower; B is split along N (the leader holds rows 0 .. N/2-1 of B, the follower the rest).
constexpr uint32_t idesc_f16(int M, int N) { return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24); }
constexpr uint32_t IDESC_S  = idesc_f16(2 * PF_ROWS, KT);
constexpr uint32_t IDESC_PV = idesc_f16(2 * PF_ROWS, HD);

// The pair's D[tmem] (+)= A x B^T, A from tensor memory (each CTA's 128 rows in its lanes, K
// packed two per column), B from shared memory (each CTA its half of B's rows)
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The pair's D[tmem] (+)= A x B^T, both from shared memory (each CTA its 128 rows of A and its
// half of B's rows)
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Commit of the pair's MMAs issued so far by this thread: one arrival on `bar` (the same shared
// offset) in both CTAs of the pair.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                     smem_u32(bar)),
                 "h"((uint16_t)3)
                 : "memory");
}
// ... one arrival on `bar` of the issuing CTA only.
__device__ __forceinline__ void mma_commit_own(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of both CTAs of the pair.
__device__ __forceinline__ void pair_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrival on the leader's (cluster rank 0) copy of barrier `bar`.  From the follower: through
// the barrier's cluster address, release at cluster scope, so that the follower's shared and
// tensor memory stores before it are visible to the MMAs the leader issues after it.  The
// leader's own threads arrive locally (CTA scope, the single-CTA pattern).
__device__ __forceinline__ void mbar_arrive_leader(uint64_t *bar, int rank) {
    if (rank == 0) {
        mbar_arrive(bar);
        return;
    }
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(a) : "r"(smem_u32(bar)));
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(a) : "memory");
}
#define PF_R32(v)                                                                                                   \
    "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),     \
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),      \
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),     \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
#define PF_W32(v)                                                                                                   \
    "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),   \
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), \
        "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), \
        "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
// 32 consecutive columns of the warp's 32 lanes: thread i gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : PF_R32(v)
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        PF_W32(v)
        : "memory");
}
// 2^x on the SFU (ex2.approx: relative error ~2^-22; 2^-inf = +0)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// Key i of a 128-key tile is visible to the row if i < nvis (causal) and its 4-cell block's bit
// is set in the row's kept-block word (all ones without a sparse selection).
__device__ __forceinline__ bool key_vis(int i, int nvis, uint32_t word) {
    return i < nvis && ((word >> (i >> 2)) & 1u);
}
// A row max as bf16 rounded toward +inf (never below the max; +-inf and 0 exact), and back: the
// two softmax halves exchange their maxima this way and both use the larger rounded value, so they
// hold the same reference (the softmax does not depend on which reference, beyond P's rounding).
__device__ __forceinline__ uint16_t max_up_bf16(float x) {
    const uint32_t u = __float_as_uint(x);
    return (uint16_t)((x > 0.0f ? u + 0xFFFFu : u) >> 16);
}
__device__ __forceinline__ float bf16_bits(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
// Max of this half's 64 keys (64 half .. 64 half + 63) of the thread's S row (two loads, one wait;
// tree of 3-input max); invisible keys count as -inf unless FULL.
template <bool FULL>
__device__ __forceinline__ float half_max(uint32_t scol, int half, int nvis, uint32_t word) {
    uint32_t v[2][32];
    tmem_ld32(scol + 64 * half, v[0]);
    tmem_ld32(scol + 64 * half + 32, v[1]);
    tmem_wait_ld();
    float m = -INFINITY;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float x[32];
#pragma unroll
        for (int e = 0; e < 32; e++) x[e] = (FULL || key_vis(64 * half + 32 * h + e, nvis, word)) ? __uint_as_float(v[h][e]) : -INFINITY;
#pragma unroll
        for (int e = 0; e < 8; e++) x[e] = fmaxf(max3(x[e], x[e + 8], x[e + 16]), x[e + 24]);
        m = max3(m, fmaxf(max3(x[0], x[1], x[2]), x[3]), fmaxf(max3(x[4], x[5], x[6]), x[7]));
    }
    return m;
}
// P = 2^(s * sl2 - mu) of this half's keys (read again: one round trip), stored as fp16 pairs in
// S columns 64 half .. 64 half + 31, inside the columns this half read.  Returns the sum of P.
template <bool FULL>
__device__ __forceinline__ float half_p(uint32_t scol, int half, int nvis, uint32_t word, float sl2, float mu) {
    const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-mu, -mu);
    float2 la = make_float2(0.f, 0.f), lb = make_float2(0.f, 0.f);
    uint32_t v[2][32];
    tmem_ld32(scol + 64 * half, v[0]);
    tmem_ld32(scol + 64 * half + 32, v[1]);
    tmem_wait_ld();
#pragma unroll
    for (int h = 0; h < 2; h++) {
        uint32_t pr[16];
#pragma unroll
        for (int e = 0; e < 16; e++) {
            const int i = 64 * half + 32 * h + 2 * e;
            const float2 y = __ffma2_rn(make_float2(FULL || key_vis(i, nvis, word) ? __uint_as_float(v[h][2 * e]) : -INFINITY,
                                                    FULL || key_vis(i + 1, nvis, word) ? __uint_as_float(v[h][2 * e + 1]) : -INFINITY),
                                        sc2, nm2);
            const float2 p = make_float2(ex2(y.x), ex2(y.y));
            if (e & 1) lb = __fadd2_rn(lb, p);
            else la = __fadd2_rn(la, p);
            const __half2 hp = __floats2half2_rn(p.x, p.y);
            pr[e] = *reinterpret_cast<const uint32_t *>(&hp);
        }
        tmem_st16(scol + 64 * half + 16 * h, pr);
    }
    return (la.x + lb.x) + (la.y + lb.y);
}

__device__ __forceinline__ uint4 ldg_nc16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ void sts16(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
// int8 x4 (two's complement) -> two f16x2 holding the exact values: bytes 0,1 -> lo, 2,3 -> hi.
__device__ __forceinline__ void s8x4_to_f16(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;                      // x + 128 as unsigned bytes
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);  // f16 1024 + u (exact)
    const uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), bias);
    lo = *reinterpret_cast<uint32_t *>(&ha);
    hi = *reinterpret_cast<uint32_t *>(&hb);
}
// 128-byte-swizzled address of 16-byte chunk c (0..7) of row r in a [rows][128 B] block.
__device__ __forceinline__ uint32_t swz(uint32_t base, int r, int c) { return base + r * 128 + ((c ^ (r & 7)) << 4); }

// ---------------------------------------------------------------------------------------------
// Query preparation: bf16 rows -> q8_0 (ggml quantize_row_q8_0 rounding) -> fp16(d * q), written
// as the 64 KiB A-operand image of each tile.  One warp per row; lane l holds elements 8l..8l+7.
__global__ void __launch_bounds__(256) k_prefill_q(const PrefillParams P) {
    // This grid may have started early: the queries may come from the kernel before it, and the
    // previous call's k_prefill reads the query tiles this grid rewrites.  k_prefill may become
    // resident only once this wait has returned: its producers read the KV pages without a wait
    // of their own, and an earlier kernel of the chain may still be writing them until then (the
    // decode kernel appends its new rows into the pages and lets its dependents start at entry;
    // its merge does the same).  k_prefill waits for this grid before reading the query tiles.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= P.n_tiles * PF_ROWS) return;
    const int tile = warp / PF_ROWS, r = warp % PF_ROWS;
    const int kvh = tile / P.n_groups, g = tile % P.n_groups;
    const int tok = g * P.tpt + r / P.G, head = kvh * P.G + r % P.G;
    uint4 o = make_uint4(0, 0, 0, 0);
    if (tok < P.Tc) {
        const uint4 raw = ldg_nc16(P.Q + ((int64_t)tok * P.n_head + head) * HD + lane * 8);
        const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
        float x[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            x[2 * i]     = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) amax = fmaxf(amax, fabsf(x[i]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d  = div127_rn(amax);
        const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
        const __half dh = __float2half_rn(d);
        uint32_t h[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const __half a = __hmul(__float2half_rn(round_half_away_f(__fmul_rn(x[2 * i], id))), dh);
            const __half b = __hmul(__float2half_rn(round_half_away_f(__fmul_rn(x[2 * i + 1], id))), dh);
            h[i] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
        }
        o = make_uint4(h[0], h[1], h[2], h[3]);
    }
    uint8_t *dst = P.qtiles + (int64_t)tile * PF_QTILE + (lane >> 3) * (PF_ROWS * 128) + r * 128 + (((lane & 7) ^ (r & 7)) << 4);
    *reinterpret_cast<uint4 *>(dst) = o;
}

// ---------------------------------------------------------------------------------------------
struct Seg {
    int tile, kt0, nk, part;
};
__device__ __forceinline__ Seg seg_of(const int4 *segs, int i) {
    const int4 s = segs[i];
    return Seg{s.x, s.y, s.z - s.y, s.w};
}

// Source of 64-token page tile kt of KV head kvh; nvalid = its keys below n_kv (<= 0: none, no
// loads).  A block-table entry outside the pool is reported in the status word.
struct TileSrc {
    const uint8_t *src;
    int nvalid;
};
// Page-table entry of page tile kt (-1 past the table).
__device__ __forceinline__ int32_t page_of(const PrefillParams &P, int kt) {
    const int pi = kt >> 2;
    return pi < P.max_pages ? __ldg(P.bt + pi) : -1;
}
// Page tile kt of KV head kvh, whose page-table entry is `page`.
__device__ __forceinline__ TileSrc tile_src(const PrefillParams &P, int kvh, int kt, int32_t page, bool report) {
    const int nvalid = min(TILE_TOK, P.n_kv - kt * TILE_TOK);
    if (nvalid <= 0) return TileSrc{nullptr, 0};
    if (page < 0 || page >= P.n_pages) {
        if (report) atomicOr(P.status, ST_BAD_PAGE);
        return TileSrc{nullptr, 0};
    }
    return TileSrc{P.pool + (int64_t)page * P.page_bytes + (int64_t)(kvh * TILES_PER_PAGE + (kt & 3)) * TILE_BYTES,
                   nvalid};
}

// This CTA's half of K tile T: keys 64 rank .. +63 (page tile 2T + rank), all 256 dims; the slot
// holds [4 atoms of 64 dims][64 keys][128 B], 128-byte swizzled.  K-producer thread t (0..127):
// 16-dim chunk kc = 4 ((t >> 3) & 3) + (t & 3) for keys 2 (t >> 5) + ((t >> 2) & 1) + 8 i,
// i = 0..7.  A warp reads 2 keys x 256 contiguous bytes per i; the 8 lanes of a shared-store phase
// cover 2 keys (different swizzle rows) x 4 chunks of one atom: no bank conflicts.
constexpr int KPT = 8;   // K chunks per producer thread and tile
struct KLoad {
    uint4    q[KPT];
    uint32_t d[KPT];
    int      nvalid;
};
__device__ __forceinline__ int k_chunk(int t) { return 4 * ((t >> 3) & 3) + (t & 3); }
__device__ __forceinline__ int k_key0(int t) { return 2 * (t >> 5) + ((t >> 2) & 1); }
__device__ __forceinline__ void k_load(const PrefillParams &P, int t, int kvh, int T, int rank, int32_t page, KLoad &L) {
    const int kc = k_chunk(t), kb = k_key0(t);
    const TileSrc ts = tile_src(P, kvh, 2 * T + rank, page, t == 0);
    L.nvalid = ts.nvalid;
#pragma unroll
    for (int i = 0; i < KPT; i++) {
        const int tk = kb + 8 * i;
        if (ts.src) {
            L.q[i] = ldg_nc16(ts.src + TILE_KQ + tk * HD + ((kc ^ kswz(tk)) << 4));
            L.d[i] = *reinterpret_cast<const uint16_t *>(ts.src + kd_off(tk, kc >> 1));
        } else {
            L.q[i] = make_uint4(0, 0, 0, 0);
            L.d[i] = 0;
        }
    }
}
__device__ __forceinline__ void k_store(uint32_t slot, int t, const KLoad &L) {
    const int kc = k_chunk(t), kb = k_key0(t);
    const uint32_t atom = slot + (kc >> 2) * (64 * 128);
#pragma unroll
    for (int i = 0; i < KPT; i++) {
        const int key = kb + 8 * i;
        const uint32_t d2 = key < L.nvalid ? (L.d[i] | (L.d[i] << 16)) : 0u;
        const uint32_t w[4] = {L.q[i].x, L.q[i].y, L.q[i].z, L.q[i].w};
        uint32_t hh[8];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            uint32_t lo, hi;
            s8x4_to_f16(w[e], lo, hi);
            hh[2 * e]     = hmul2(lo, d2);
            hh[2 * e + 1] = hmul2(hi, d2);
        }
        sts16(swz(atom, key, (kc & 3) * 2), make_uint4(hh[0], hh[1], hh[2], hh[3]));
        sts16(swz(atom, key, (kc & 3) * 2 + 1), make_uint4(hh[4], hh[5], hh[6], hh[7]));
    }
}

// This CTA's half of V tile T: dims 128 rank .. +127, keys 0..127 (page tiles 2T, 2T+1); the slot
// holds [2 atoms of 64 keys][128 dims][128 B], 128-byte swizzled.  V-producer thread t (0..127):
// tokens 16 vc .. +15 (vc = t & 3) of page tile 2T + a (a = (t >> 3) & 1) for the 8 dims
// 32 bl + dd + 4 i (bl = t >> 5, dd = ((t >> 2) & 1) | ((t >> 4) & 1) << 1, i = 0..7), all in
// q8_0 block bl of the half, so they share one set of scales.  Per i a warp reads 4 consecutive
// dims x 64 bytes of each page tile; a shared-store phase covers 2 adjacent dims (rows of
// different swizzle parity) x 4 chunks: no bank conflicts.
constexpr int VPT = 8;   // V dims per producer thread and tile
struct VLoad {
    uint4 q[VPT];
    uint4 d0, d1;
    int   nvalid;
};
__device__ __forceinline__ int v_dim0(int t) { return 32 * (t >> 5) + (((t >> 2) & 1) | (((t >> 4) & 1) << 1)); }
__device__ __forceinline__ void v_load(const PrefillParams &P, int t, int kvh, int T, int rank, int32_t page, VLoad &L) {
    const int vc = t & 3, a = (t >> 3) & 1, d0 = 128 * rank + v_dim0(t);
    const TileSrc ts = tile_src(P, kvh, 2 * T + a, page, false);
    L.nvalid = ts.nvalid;
    if (ts.src) {
#pragma unroll
        for (int i = 0; i < VPT; i++) {
            const int dim = d0 + 4 * i;
            L.q[i] = ldg_nc16(ts.src + TILE_VQ + dim * TILE_TOK + ((vc ^ ((dim >> 1) & 3)) << 4));
        }
        const uint8_t *vd = ts.src + vd_off(d0 >> 5, vc * 16);
        L.d0 = ldg_nc16(vd);
        L.d1 = ldg_nc16(vd + 16);
    } else {
#pragma unroll
        for (int i = 0; i < VPT; i++) L.q[i] = make_uint4(0, 0, 0, 0);
        L.d0 = L.d1 = make_uint4(0, 0, 0, 0);
    }
}
__device__ __forceinline__ void v_store(uint32_t slot, int t, const VLoad &L) {
    const int vc = t & 3, a = (t >> 3) & 1, d0 = v_dim0(t);
    const uint32_t atom = slot + a * (128 * 128);
    uint32_t dv[8] = {L.d0.x, L.d0.y, L.d0.z, L.d0.w, L.d1.x, L.d1.y, L.d1.z, L.d1.w};
#pragma unroll
    for (int e = 0; e < 8; e++) {   // tokens 16 vc + 2e, +1: zero scales past n_kv
        const int t0 = vc * 16 + 2 * e;
        dv[e] &= t0 + 1 < L.nvalid ? 0xffffffffu : (t0 < L.nvalid ? 0x0000ffffu : 0u);
    }
#pragma unroll
    for (int i = 0; i < VPT; i++) {
        const int dim = d0 + 4 * i;
        const uint32_t w[4] = {L.q[i].x, L.q[i].y, L.q[i].z, L.q[i].w};
        uint32_t hh[8];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            uint32_t lo, hi;
            s8x4_to_f16(w[e], lo, hi);
            hh[2 * e]     = hmul2(lo, dv[2 * e]);
            hh[2 * e + 1] = hmul2(hi, dv[2 * e + 1]);
        }
        sts16(swz(atom, dim, vc * 2), make_uint4(hh[0], hh[1], hh[2], hh[3]));
        sts16(swz(atom, dim, vc * 2 + 1), make_uint4(hh[4], hh[5], hh[6], hh[7]));
    }
}

// Ring order of a segment's K/V ops (each one slot): K_0, then (K_k, V_{k-1}) for k = 1 .. nk-1,
// then V_{nk-1} (the MMA issue order S_0, S_1, PV_0, S_2, PV_1, ...).
__device__ __forceinline__ uint32_t op_k(int k) { return k == 0 ? 0u : (uint32_t)(2 * k - 1); }
__device__ __forceinline__ uint32_t op_v(int k, int nk) { return k == nk - 1 ? (uint32_t)(2 * nk - 1) : (uint32_t)(2 * k + 2); }

// One producer group's walk over this CTA's halves of its ops in ring order (K group: the K
// ops, V group: the V ops).  The next op's loads are issued as soon as the last one is stored,
// so they are in flight while its slot is awaited; the page-table entry of the next KV tile is
// loaded one step ahead.  Every store ends with an arrival on the leader's slot_full.
template <bool KGRP>
__device__ __forceinline__ void produce(const PrefillParams &P, const int4 *segs, Bars *B, uint32_t sbase, int t,
                                        int rank, int s0, int s1) {
    using Load = typename std::conditional<KGRP, KLoad, VLoad>::type;
    int si = s0, k = 0;
    uint32_t op0 = 0;
#ifdef QKV_TIMELINE
    int jt = 0;   // operands stored so far (the KV tile of the next store)
#endif
    Seg sg{};
    int32_t page = -1;
    if (si < s1) {
        sg = seg_of(segs, si);
        page = page_of(P, 2 * sg.kt0);
    }
    auto load_next = [&](Load &L, uint32_t &u) -> bool {   // false: walk finished
        if (si >= s1) return false;
        const int kvh = sg.tile / P.n_gpairs;
        if constexpr (KGRP) {
            k_load(P, t, kvh, sg.kt0 + k, rank, page, L);
            u = op0 + op_k(k);
        } else {
            v_load(P, t, kvh, sg.kt0 + k, rank, page, L);
            u = op0 + op_v(k, sg.nk);
        }
        if (++k == sg.nk) {
            k = 0;
            op0 += 2 * sg.nk;
            if (++si < s1) sg = seg_of(segs, si);
        }
        if (si < s1) page = page_of(P, 2 * (sg.kt0 + k));
        return true;
    };
    auto store = [&](const Load &ld, uint32_t u) -> bool {
        const uint32_t sl = u % NSLOT;
        PF_TL(t == 0, KGRP ? 3 : 4, jt, 0);
        if (u >= NSLOT && !__all_sync(0xffffffffu, wait_bar(&B->slot_free[sl], ((u / NSLOT) - 1) & 1, B, P.status)))
            return false;   // warp-uniform: every lane leaves together
        PF_TL(t == 0, KGRP ? 3 : 4, jt, 1);
        const uint32_t slot = sbase + SM_RING + sl * SLOT_BYTES;
        if constexpr (KGRP) k_store(slot, t, ld);
        else v_store(slot, t, ld);
        fence_proxy_async();
        mbar_arrive_leader(&B->slot_full[sl], rank);
        PF_TL(t == 0, KGRP ? 3 : 4, jt, 2);
#ifdef QKV_TIMELINE
        jt++;
#endif
        return true;
    };
    Load A;
    uint32_t uA = 0;
    while (load_next(A, uA))
        if (!store(A, uA)) return;
}

// SPARSE: P.qsa_bits holds each query row's kept-block bitset (qkv_attn_prefill_qsa); the dense
// instantiation has no trace of it.
template <bool SPARSE>
__global__ void __launch_bounds__(NTHR, 1) k_prefill(const __grid_constant__ PrefillParams P,
                                                     const __grid_constant__ PfPlanInline PL) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(sm);
    Bars *B = reinterpret_cast<Bars *>(sm + SM_BAR);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = (int)cluster_rank();   // 0: leader (issues the pair's MMAs), 1: follower
    const int4 *segs = P.plan_inline ? reinterpret_cast<const int4 *>(PL.v) : P.segs;
    const int32_t *cta_seg = P.plan_inline ? PL.v + P.off_cta : P.cta_seg;
    const int pr = blockIdx.x >> 1;   // the pair's run of segments
    const int s0 = cta_seg[pr], s1 = cta_seg[pr + 1];
    // Launched with programmatic stream serialisation after k_prefill_q: everything up to the
    // first query-tile copy (barriers, TMEM, the producers' K/V tiles, which earlier launches
    // wrote) overlaps that kernel; the copying threads wait for it before the copy.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (tid == 0) {
        for (int i = 0; i < NSLOT; i++) {
            mbar_init(&B->slot_full[i], 2 * 128 * NGRP);
            mbar_init(&B->slot_free[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&B->s_full[i], 1);
            mbar_init(&B->s_read[i], 128 * SMX_GROUPS);
            mbar_init(&B->p_full[i], 2 * 128 * SMX_GROUPS);
            mbar_init(&B->pv_done[i], 1);
        }
        mbar_init(&B->q_full, 1);
        mbar_init(&B->q_peer, 1);
        mbar_init(&B->q_empty, 1);
        mbar_init(&B->drain, 1);
        B->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // both CTAs' warp 0: the pair's tensor memory
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B->tmem)),
                     "r"(TM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    pair_sync();   // both CTAs' barriers initialised and TMEM allocated before any cross-CTA arrival
    tc_fence_after();
    const uint32_t tmem = B->tmem;

    if (warp == 0) {
        if (lane == 0 && rank == 0) {
            // -------------------------------------------------------------- MMA issue (leader)
            bool ok = true;
            int q_pending = -1;   // parity of a query copy still in flight after an abort
            uint32_t it = 0, op0 = 0;
            const uint32_t qa = sbase + SM_Q, ra = sbase + SM_RING;
            // wait for ring slot u (the u-th op of the pair); returns its address
            auto slot_wait = [&](uint32_t u, uint32_t &addr) -> bool {
                const uint32_t sl = u % NSLOT;
                addr = ra + sl * SLOT_BYTES;
                return wait_bar(&B->slot_full[sl], (u / NSLOT) & 1, B, P.status);
            };
            auto issue_s = [&](uint32_t j, uint32_t u) -> bool {
                uint32_t kaddr;
                if (!slot_wait(u, kaddr)) return false;
                tc_fence_after();
                const uint32_t d = tmem + TM_S + (j & 1) * KT;
                // descriptor start addresses advance by (bytes >> 4) in the low field
                const uint64_t qd = sdesc(qa), kd = sdesc(kaddr);
#pragma unroll
                for (int kk = 0; kk < HD / 16; kk++)
                    mma_f16_ss(d, qd + (uint64_t)(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4),
                               kd + (uint64_t)(((kk >> 2) * (64 * 128) + (kk & 3) * 32) >> 4), IDESC_S, kk ? 1u : 0u);
                mma_commit_pair(&B->slot_free[u % NSLOT]);
                mma_commit_pair(&B->s_full[j & 1]);
                return true;
            };
            auto issue_pv = [&](uint32_t j, uint32_t u, bool first) -> bool {
                const uint32_t b = j & 1;
                if (!wait_bar(&B->p_full[b], (j >> 1) & 1, B, P.status)) return false;
                uint32_t vaddr;
                if (!slot_wait(u, vaddr)) return false;
                tc_fence_after();
                const uint64_t vd = sdesc(vaddr);
#pragma unroll
                for (int kk = 0; kk < KT / 16; kk++)   // P of keys 16 kk..: columns 64 (kk >> 2) + 8 (kk & 3)
                    mma_f16_ts(tmem + TM_O, tmem + TM_S + b * KT + 64 * (kk >> 2) + 8 * (kk & 3),
                               vd + (uint64_t)(((kk >> 2) * (128 * 128) + (kk & 3) * 32) >> 4), IDESC_PV,
                               (first && kk == 0) ? 0u : 1u);
                mma_commit_pair(&B->slot_free[u % NSLOT]);
                mma_commit_pair(&B->pv_done[b]);
                return true;
            };
            asm volatile("griddepcontrol.wait;" ::: "memory");   // query tiles of k_prefill_q
            for (int si = s0; si < s1 && ok; si++) {
                const Seg sg = seg_of(segs, si);
                if (si > s0 && !(ok = wait_bar(&B->q_empty, (si - s0 - 1) & 1, B, P.status))) break;
                // the leader's tile of the pair (2 gp) always exists
                const int tile = (sg.tile / P.n_gpairs) * P.n_groups + 2 * (sg.tile % P.n_gpairs);
                mbar_expect_tx(&B->q_full, PF_QTILE);
                const uint8_t *qsrc = P.qtiles + (int64_t)tile * PF_QTILE;
#pragma unroll
                for (int c = 0; c < 4; c++) bulk_load(sm + SM_Q + c * 16384, qsrc + c * 16384, 16384, &B->q_full);
                if (!(ok = wait_bar(&B->q_full, (si - s0) & 1, B, P.status))) {
                    q_pending = (si - s0) & 1;
                    break;
                }
                if (!(ok = wait_bar(&B->q_peer, (si - s0) & 1, B, P.status))) break;
                tc_fence_after();
                for (int k = 0; k < sg.nk && ok; k++) {
                    PF_TL(true, 2, (int)(it + k), 0);
                    ok = issue_s(it + k, op0 + op_k(k));
                    PF_TL(true, 2, (int)(it + k), 1);
                    if (ok && k == sg.nk - 1) mma_commit_pair(&B->q_empty);
                    if (ok && k >= 1) ok = issue_pv(it + k - 1, op0 + op_v(k - 1, sg.nk), k == 1);
                    PF_TL(true, 2, (int)(it + k), 2);
                }
                if (ok) ok = issue_pv(it + sg.nk - 1, op0 + op_v(sg.nk - 1, sg.nk), sg.nk == 1);
                it += sg.nk;
                op0 += 2 * sg.nk;
            }
            if (q_pending >= 0) drain_bar(&B->q_full, (uint32_t)q_pending, P.status);
            mma_commit_own(&B->drain);
            drain_bar(&B->drain, 0, P.status);
        } else if (lane == 0) {
            // -------------------------------------------------------------- follower: its query tiles
            // For each segment: once the pair's previous S MMAs are done with the query buffer,
            // copy this CTA's query tile (rows 128-255 of the pair's MMAs) and tell the leader.
            bool ok = true;
            int q_pending = -1;
            asm volatile("griddepcontrol.wait;" ::: "memory");   // query tiles of k_prefill_q
            for (int si = s0; si < s1 && ok; si++) {
                const Seg sg = seg_of(segs, si);
                if (si > s0 && !(ok = wait_bar(&B->q_empty, (si - s0 - 1) & 1, B, P.status))) break;
                const int g = 2 * (sg.tile % P.n_gpairs) + 1;
                if (g < P.n_groups) {
                    mbar_expect_tx(&B->q_full, PF_QTILE);
                    const uint8_t *qsrc = P.qtiles + ((int64_t)(sg.tile / P.n_gpairs) * P.n_groups + g) * PF_QTILE;
#pragma unroll
                    for (int c = 0; c < 4; c++) bulk_load(sm + SM_Q + c * 16384, qsrc + c * 16384, 16384, &B->q_full);
                } else {
                    mbar_arrive(&B->q_full);   // no second tile in this pair: rows fully masked
                }
                if (!(ok = wait_bar(&B->q_full, (si - s0) & 1, B, P.status))) {
                    q_pending = (si - s0) & 1;
                    break;
                }
                mbar_arrive_leader(&B->q_peer, rank);
            }
            if (q_pending >= 0) drain_bar(&B->q_full, (uint32_t)q_pending, P.status);
        }
        __syncwarp();
    } else if (warp < 1 + 4 * SMX_GROUPS) {
        // ------------------------------------------------------------------ softmax
        // Warps 1-4 (half 0) and 5-8 (half 1): warp w reads TMEM lanes 32 (w & 3) .. +31, so
        // thread r owns row r of this CTA's tile in both halves.  Control flow is warp-uniform
        // (tcgen05.ld/st are warp-collective): every wait's result is agreed with __all_sync.  Per
        // 128-key tile half h reads only its keys 64h .. 64h+63, posts their max (bf16, rounded
        // up) in shared memory and meets the other half at s_read; both take the larger posted
        // value, so both raise the lazily raised reference the same way.  Half h then reads its
        // keys again, turns them into P (fp16 pairs) and stores them over S columns
        // 64h .. 64h+31.  If the row max grows by more than 2^8 over the reference, the
        // reference moves up and l and O (half h rescales O columns 128h .. 128h+127) are scaled.
        const int half = (warp - 1) >> 2, r = (warp & 3) * 32 + lane;
        uint16_t *pmax = reinterpret_cast<uint16_t *>(sm + SM_PMAX);
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        auto wait_all = [&](uint64_t *bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, wait_bar(bar, parity, B, P.status));
        };
        uint32_t it = 0;
        bool ok = true;
        for (int si = s0; si < s1 && ok; si++) {
            const Seg sg = seg_of(segs, si);
            const int g = 2 * (sg.tile % P.n_gpairs) + rank;   // this CTA's query group (n_groups: none)
            const int tok = g * P.tpt + r / P.G;
            const int qpos = g < P.n_groups && tok < P.Tc ? P.pos0 + tok : -1;
            float m_ref = -INFINITY, l = 0.f;
            // the row's kept-block word of each KV tile (sparse prefill), one tile ahead
            const uint32_t *wrow = SPARSE && qpos >= 0 ? P.qsa_bits + (int64_t)tok * P.qsa_words : nullptr;
            const int kt_vis = qpos >= 0 ? qpos / KT : -1;   // last KV tile with a visible key
            uint32_t word_next = SPARSE && wrow && sg.kt0 <= kt_vis ? __ldg(wrow + sg.kt0) : ~0u;
            for (int k = 0; k < sg.nk; k++) {
                const uint32_t j = it + k, b = j & 1;
                if (!(ok = wait_all(&B->s_full[b], (j >> 1) & 1))) break;
                PF_TL(lane == 0 && (warp & 3) == 1, half, (int)j, 0);
                tc_fence_after();
                const uint32_t scol = tmem + lane_base + TM_S + b * KT;
                const int nvis = min(max(qpos - (sg.kt0 + k) * KT + 1, 0), KT);
                const uint32_t word = SPARSE ? word_next : ~0u;
                if (SPARSE && wrow) word_next = sg.kt0 + k + 1 <= kt_vis && k + 1 < sg.nk ? __ldg(wrow + sg.kt0 + k + 1) : ~0u;
                const bool full = __all_sync(0xffffffffu, nvis == KT && (!SPARSE || word == ~0u));
                const float hmax = full ? half_max<true>(scol, half, nvis, word) : half_max<false>(scol, half, nvis, word);
                // this half's max (bf16, rounded up) to shared memory; the other half reads it after
                // the meeting.  Slot b is written again for tile j + 2, whose S needs P_j consumed,
                // i.e. both halves past this read.
                PF_TL(lane == 0 && (warp & 3) == 1, half, (int)j, 1);
                pmax[(2 * b + half) * PF_ROWS + r] = max_up_bf16(hmax);
                tc_fence_before();
                mbar_arrive(&B->s_read[b]);
                if (!(ok = wait_all(&B->s_read[b], (j >> 1) & 1))) break;
                PF_TL(lane == 0 && (warp & 3) == 1, half, (int)j, 2);
                tc_fence_after();
                const float smax = fmaxf(bf16_bits(pmax[(2 * b) * PF_ROWS + r]), bf16_bits(pmax[(2 * b + 1) * PF_ROWS + r]));
                // lazily raised reference max: O and l are rescaled only when a row max grows by
                // more than 2^8 over the reference (P stays <= 256, exact enough in fp16)
                const float mx = smax * P.scale_log2;   // scale > 0: max of scaled = scaled max
                const bool need = mx > m_ref + 8.0f;
                const float F = (need && m_ref != -INFINITY) ? ex2(m_ref - mx) : 1.0f;
                if (need) m_ref = mx;
                l *= F;
                const float mu = m_ref == -INFINITY ? 0.f : m_ref;   // fully masked so far: p = 0
                l += full ? half_p<true>(scol, half, nvis, word, P.scale_log2, mu)
                          : half_p<false>(scol, half, nvis, word, P.scale_log2, mu);
                PF_TL(lane == 0 && (warp & 3) == 1, half, (int)j, 3);
                if (k > 0 && __any_sync(0xffffffffu, F != 1.0f)) {
                    // O holds PV of the previous tile: rescale it once that product has landed
                    if (!(ok = wait_all(&B->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1))) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int c8 = 4 * half; c8 < 4 * half + 4; c8++) {
                        uint32_t o[32];
                        tmem_ld32(tmem + lane_base + TM_O + c8 * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; c++) o[c] = __float_as_uint(__uint_as_float(o[c]) * F);
                        tmem_st32(tmem + lane_base + TM_O + c8 * 32, o);
                    }
                }
                tmem_wait_st();
                PF_TL(lane == 0 && (warp & 3) == 1, half, (int)j, 4);
                tc_fence_before();
                mbar_arrive_leader(&B->p_full[b], rank);
                PF_TL(lane == 0 && (warp & 3) == 1, half, (int)j, 5);
            }
            if (!ok) break;
            // ---- epilogue: this half's O columns of the segment's partial record
            const uint32_t jl = it + sg.nk - 1;
            if (!(ok = wait_all(&B->pv_done[jl & 1], (jl >> 1) & 1))) break;
            tc_fence_after();
            if (g < P.n_groups) {   // records 2 part + rank; stores of a warp cover 32 adjacent rows
                float *rec = P.partial + (int64_t)(2 * sg.part + rank) * pf_part_floats();
#pragma unroll 1
                for (int c8 = 4 * half; c8 < 4 * half + 4; c8++) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_base + TM_O + c8 * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int q = 0; q < 8; q++)
                        __stcg(reinterpret_cast<float4 *>(rec) + (int64_t)(c8 * 8 + q) * PF_ROWS + r,
                               make_float4(__uint_as_float(o[4 * q]), __uint_as_float(o[4 * q + 1]),
                                           __uint_as_float(o[4 * q + 2]), __uint_as_float(o[4 * q + 3])));
                }
                if (half == 0) __stcg(rec + PF_ROWS * HD + r, m_ref);
                __stcg(rec + PF_ROWS * HD + (1 + half) * PF_ROWS + r, l);
            }
            tc_fence_before();
            it += sg.nk;
        }
    } else {
        // ------------------------------------------------------------------ producers
        // warps 9-12 fill this CTA's halves of the K tiles, warps 13-16 its halves of the V tiles.
        if (warp < PW_V) produce<true>(P, segs, B, sbase, tid - 32 * PW_K, rank, s0, s1);
        else produce<false>(P, segs, B, sbase, tid - 32 * PW_V, rank, s0, s1);
    }
    tc_fence_before();
    __syncthreads();
    pair_sync();   // the leader's MMAs are drained: neither CTA's tensor or shared memory is in use
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TM_COLS) : "memory");
    }
}

// Merge of the segments' partial records of every tile: O = sum_p 2^(m_p - M) O_p / sum_p
// 2^(m_p - M) l_p, parts in order (batches of MG_PB parts, the running max rescaled between
// batches).  CTA = (tile, MG_ROWS rows), 256 threads.  Thread (row = t % MG_ROWS, column group
// t / MG_ROWS) loads its 4 float4 columns and (m, l) of a whole batch at once -- one round trip to
// L2 for up to MG_PB parts; adjacent threads read adjacent rows (coalesced in the record layout).
// The rows go through shared memory so that the output, rows of 256 contiguous floats, is written
// by threads along each row.
constexpr int MG_ROWS = 16, MG_PB = 4;
__global__ void __launch_bounds__(256) k_prefill_merge(const __grid_constant__ PrefillParams P,
                                                       const __grid_constant__ PfPlanInline PL) {
    __shared__ float4 rows[MG_ROWS][HD / 4 + 1];
    constexpr int QTR = PF_ROWS / MG_ROWS;
    const int tile = blockIdx.x / QTR, r0 = (blockIdx.x % QTR) * MG_ROWS;
    const int t = threadIdx.x, rr = t % MG_ROWS, fg = t / MG_ROWS, row = r0 + rr;
    // the next call's k_prefill_q may become resident now (it waits for this grid)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");   // partial records of k_prefill
    // the tile's pair tile and its CTA in the pair: record of part i = 2 (first + i) + rank
    const int kvh0 = tile / P.n_groups, g0 = tile % P.n_groups;
    const int2 tp = (P.plan_inline ? reinterpret_cast<const int2 *>(PL.v + P.off_tiles)
                                   : P.tile_parts)[kvh0 * P.n_gpairs + (g0 >> 1)];
    const float *base = P.partial + (int64_t)(2 * tp.y + (g0 & 1)) * pf_part_floats();
    float M = -INFINITY, L = 0.f;
    float4 acc[4];
#pragma unroll
    for (int i = 0; i < 4; i++) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p0 = 0; p0 < tp.x; p0 += MG_PB) {
        float m[MG_PB], l[MG_PB];
        float4 v[MG_PB][4];
#pragma unroll
        for (int k = 0; k < MG_PB; k++) {
            const float *rec = base + (int64_t)2 * min(p0 + k, tp.x - 1) * pf_part_floats();   // clamped: weight 0
            m[k] = p0 + k < tp.x ? __ldcg(rec + PF_ROWS * HD + row) : -INFINITY;
            l[k] = __ldcg(rec + PF_ROWS * HD + PF_ROWS + row) + __ldcg(rec + PF_ROWS * HD + 2 * PF_ROWS + row);
#pragma unroll
            for (int i = 0; i < 4; i++)
                v[k][i] = __ldcg(reinterpret_cast<const float4 *>(rec) + (int64_t)(fg * 4 + i) * PF_ROWS + row);
        }
        float Mn = M;
#pragma unroll
        for (int k = 0; k < MG_PB; k++) Mn = fmaxf(Mn, m[k]);
        const float a = M == -INFINITY ? 0.f : ex2(M - Mn);   // rescale of the earlier batches
        L *= a;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            acc[i].x *= a; acc[i].y *= a; acc[i].z *= a; acc[i].w *= a;
        }
#pragma unroll
        for (int k = 0; k < MG_PB; k++) {
            const float w = m[k] == -INFINITY ? 0.f : ex2(m[k] - Mn);
            L = fmaf(w, l[k], L);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                acc[i].x = fmaf(w, v[k][i].x, acc[i].x);
                acc[i].y = fmaf(w, v[k][i].y, acc[i].y);
                acc[i].z = fmaf(w, v[k][i].z, acc[i].z);
                acc[i].w = fmaf(w, v[k][i].w, acc[i].w);
            }
        }
        M = Mn;
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++)
        rows[rr][fg * 4 + i] = make_float4(acc[i].x * inv, acc[i].y * inv, acc[i].z * inv, acc[i].w * inv);
    __syncthreads();
    const int kvh = tile / P.n_groups, g = tile % P.n_groups;
#pragma unroll 1
    for (int e = t; e < MG_ROWS * (HD / 4); e += 256) {
        const int q = e & (HD / 4 - 1), rw = r0 + e / (HD / 4);
        const int tok = g * P.tpt + rw / P.G, head = kvh * P.G + rw % P.G;
        if (tok < P.Tc) reinterpret_cast<float4 *>(P.out + ((int64_t)tok * P.n_head + head) * HD)[q] = rows[e / (HD / 4)][q];
    }
}

}  // namespace pf
#ifdef QKV_TIMELINE
}  // namespace qkv
extern "C" int qkv_pf_tl_read(unsigned long long *host, int reset) {
    const size_t bytes = sizeof(qkv::pf::g_pf_tl);
    if (host && cudaMemcpyFromSymbol(host, qkv::pf::g_pf_tl, bytes) != cudaSuccess) return -1;
    if (reset) {
        void *d = nullptr;
        if (cudaGetSymbolAddress(&d, qkv::pf::g_pf_tl) != cudaSuccess || cudaMemset(d, 0, bytes) != cudaSuccess) return -1;
    }
    return (int)(bytes / 8);
}
namespace qkv {
#endif

// Launch of a kernel that may start while the previous kernel on the stream finishes
// (programmatic dependent launch); it synchronises itself with griddepcontrol.wait.
template <typename K, typename... A>
static cudaError_t launch_pdl(K kernel, unsigned grid, unsigned block, size_t smem, cudaStream_t st, const A &...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The three kernels of a call, each launched behind its predecessor (programmatic dependent
// launch): k_prefill_q waits for whatever precedes it before reading the queries, k_prefill and
// k_prefill_merge wait for the kernel before them (see the kernels).  k_prefill runs as clusters
// of two CTAs (the MMA pairs).
static cudaError_t configure_prefill() {
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && configured[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(pf::k_prefill<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(pf::k_prefill<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM_BYTES);
    if (e == cudaSuccess && dev >= 0 && dev < 64) configured[dev] = true;
    return e;
}

static void prefill_config(cudaLaunchConfig_t &cfg, cudaLaunchAttribute (&attr)[2], unsigned grid, cudaStream_t st) {
    cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(pf::NTHR);
    cfg.dynamicSmemBytes = pf::SMEM_BYTES;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
}

int prefill_max_pairs() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev]) return cached[dev];
    if (configure_prefill() != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    prefill_config(cfg, attr, 2 * 64, nullptr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, pf::k_prefill<false>, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cached[dev] = n;
    return n;
}

cudaError_t launch_prefill(const PrefillParams &p, const PfPlanInline &plan, cudaStream_t st) {
    cudaError_t e = configure_prefill();
    if (e != cudaSuccess) return e;
    const int64_t rows = (int64_t)p.n_tiles * PF_ROWS;
    if ((e = launch_pdl(pf::k_prefill_q, (unsigned)((rows + 7) / 8), 256, 0, st, p)) != cudaSuccess) return e;
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    prefill_config(cfg, attr, (unsigned)p.n_ctas, st);
    if ((e = p.qsa_bits ? cudaLaunchKernelEx(&cfg, pf::k_prefill<true>, p, plan)
                        : cudaLaunchKernelEx(&cfg, pf::k_prefill<false>, p, plan)) != cudaSuccess)
        return e;
    if ((e = launch_pdl(pf::k_prefill_merge, (unsigned)(p.n_tiles * (PF_ROWS / pf::MG_ROWS)), 256, 0, st, p, plan)) !=
        cudaSuccess)
        return e;
    count_launches(3);
    return cudaSuccess;
}

}  // namespace qkv
