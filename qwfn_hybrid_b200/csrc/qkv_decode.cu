// qkv_decode.cu -- kernel C: split-K decode / MTP-verify attention over the paged q8_0 cache.
//
// Work plan (host-built, passed by value).  A pair is (sequence, KV head); its tiles are the
// 64-token tiles of the sequence (dense) or the selected block ids (sparse).  Each pair is cut
// into `units` contiguous tile ranges in proportion to its length, and every CTA runs exactly one
// unit, so a ragged batch balances by tiles.  A pair with one unit writes its output directly;
// otherwise every unit leaves a partial record (running max m, row sum l, unnormalised O) and
// k_decode_merge, launched right behind (programmatic dependent launch, so its CTAs are resident
// before the last units finish), combines each (pair, query row) in a fixed order: results do
// not depend on which unit finishes last.
//
// Per unit, the G*T query rows of the KV head's group are quantised to q8_0 exactly as ggml's
// CPU flash_attn_ext quantises its query row, so every QK value is sum_b isum_b * (d_k * d_q)
// with an exact integer block dot.
//
// CTA = 4 warps, 2-4 CTAs per SM.  Tiles (34816 B: K quants, V quants transposed, scales) stream
// into a 2-stage shared-memory ring with 1-D bulk copies (cp.async.bulk, the TMA engine; no
// multicast) completing on mbarriers.  Per tile:
//   QK  warp w: its 16 tokens x all query rows.  mma.m16n8k32 s8 per q8_0 block, A = K rows
//       (token order permuted by pi16() so that a movmatrix transpose of P lands in the PV B
//       layout), B = quantised Q.  The accumulator input is 0x4B400000 so the int32 dot d comes
//       out as the float 12582912 + d; one packed subtract recovers d exactly, then
//       S += d * (dq * dk) with packed f32x2 arithmetic.
//   softmax: tile max across the 4 warps via shared memory, exp2, P -> f16 -> movmatrix -> smem.
//   PV  warp w: its 64 dims x all query rows over the 64 tokens.  mma.m16n8k16 f16 with
//       A = V^T int8 widened to f16 exactly (byte permute + bias subtract) and B = P * dv.
// Optional fused append (dense only): the unit owning a tile that holds one of the T new
// positions quantises those rows (kernel A's rounding) in its prologue and stores them in the
// page, then starts the bulk copy of that tile, which thus brings the new rows with it.
#include "qkv.h"
#include "qkv_internal.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <cuda_fp16.h>

namespace qkv {
namespace dec {

constexpr int PF_TILES = 2;   // tiles per unit prefetched into L2 before the previous launch ends
constexpr int PSTR   = 80;      // halves per P row in smem (64 tokens + pad: conflict-free LDS.64)
constexpr int QSTR   = 288;     // bytes per quantised query row (256 + pad)
constexpr uint32_t MAGIC_I = 0x4B400000u;
constexpr float    MAGIC_F = 12582912.0f;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Phase timestamps for latency analysis, compiled only with -DQKV_TIMELINE (the product build
// never defines it): thread 0 of every CTA notes %globaltimer at its phases and appends one record
// {kernel, block, t[0..19]} to g_tl_rec; qkv_tl_read copies the records out.
#ifdef QKV_TIMELINE
__device__ unsigned long long g_tl_rec[1 << 16][22];
__device__ unsigned int g_tl_n;
#define TL_DECL unsigned long long tl_[20] = {};
#define TL(i) do { if (threadIdx.x == 0) tl_[i] = global_ns(); } while (0)
#define TL_FLUSH(kid)                                                             \
    do {                                                                          \
        if (threadIdx.x == 0) {                                                   \
            const unsigned k_ = atomicAdd(&g_tl_n, 1u) & 0xffffu;                 \
            g_tl_rec[k_][0] = (kid);                                              \
            g_tl_rec[k_][1] = blockIdx.x;                                         \
            for (int i_ = 0; i_ < 20; i_++) g_tl_rec[k_][2 + i_] = tl_[i_];       \
        }                                                                         \
    } while (0)
#else
#define TL_DECL
#define TL(i) do { } while (0)
#define TL_FLUSH(kid) do { } while (0)
#endif
// Stamps inside the tile body (first two tiles of a unit), timeline build only.
#ifdef QKV_TIMELINE
#define TLT_ARG , unsigned long long *tl_, int tli
#define TLT_PASS(x) , tl_, (x)
#define TLT(k) do { if (threadIdx.x == 0 && tli >= 0) tl_[tli + (k)] = global_ns(); } while (0)
#else
#define TLT_ARG
#define TLT_PASS(x)
#define TLT(k) do { } while (0)
#endif
// Bounded wait: gives up after limit_ns (a copy that never lands) instead of spinning forever.
__device__ __noinline__ bool mbar_wait(uint64_t *bar, uint32_t phase, uint64_t limit_ns) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, phase)) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
}
// Limit of the waits that follow one that gave up (1 ms, or less): they only cover copies issued
// before it, which land within microseconds; stages whose next copy was never started time out.
__device__ __forceinline__ uint64_t after_abort(uint64_t limit_ns) { return limit_ns < 1000000ull ? limit_ns : 1000000ull; }
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// One arrival on bar once all of this thread's earlier cp.async copies have landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void *p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }
__device__ __forceinline__ void bulk_prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma_s8(uint32_t (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1, uint32_t c) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
    return *reinterpret_cast<uint32_t *>(&r);
}
// int8 x4 (two's complement) -> two f16x2 holding the exact values: bytes 0,1 -> lo, 2,3 -> hi.
__device__ __forceinline__ void s8x4_to_f16(uint32_t w, uint32_t &lo, uint32_t &hi) {
    const uint32_t u = w ^ 0x80808080u;                  // x + 128 as unsigned bytes
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);  // f16 1024 + u (exact)
    const uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    __half2 ha = __hsub2(*reinterpret_cast<const __half2 *>(&a), bias);
    __half2 hb = __hsub2(*reinterpret_cast<const __half2 *>(&b), bias);
    lo = *reinterpret_cast<uint32_t *>(&ha);
    hi = *reinterpret_cast<uint32_t *>(&hb);
}
// Row order of the 16 K rows of a QK mma: A row m holds token pi(m) of the warp's 16 tokens, so
// after movmatrix a thread's P pairs are the consecutive tokens 4*tig .. 4*tig+3 that the PV
// A fragment (one int8x4 word of V^T) covers.
__device__ __forceinline__ int pi16(int m) { return ((m & 6) << 1) | (m & 1) | ((m & 8) >> 2); }
// Byte position of element e (0..31) of a quantised query block in the fragment order
// [tig][b0 word, b1 word]: one LDS.64 fetches both B registers of an m16n8k32 B fragment.
__device__ __forceinline__ int qperm(int e) { return ((e & 15) >> 2) * 8 + ((e >> 4) << 2) + (e & 3); }


// Row stride (floats) of the epilogue's O buffer: rows 4 banks apart, so a warp's stores (4 rows x
// 8 consecutive dims) hit 32 distinct banks; 16-byte aligned rows for the float4 reads.
constexpr int OSTR = HD + 4;

// Stages of the tile ring: one 34816-byte stage per CTA keeps 4 CTAs (16 warps) per SM; two let
// a unit's second tile load while the first is processed (the host takes two when a launch has
// at most two units per SM).  The O buffer of the epilogue reuses the stages, so wide query
// groups (NQ > 34) always take two.
template <int NT>
struct Stages { static constexpr int N = NT * 8 * OSTR * 4 <= TILE_BYTES ? 1 : 2; };

// Shared memory of the four warps that work on one tile.
template <int NT>
struct alignas(16) LaneShared {
    __half   ps[NT * 8 * PSTR];          // P of the current tile, [row][token]
    float    red[4 * NT * 8];            // chunk maxima of warps that outgrew the reference
    float    lpart[4 * NT * 8];          // per-warp row sums (epilogue)
    int32_t  flag[4];                    // warp outgrew the softmax reference in this tile
};

template <int NT, int NSR>
struct Smem {
    static constexpr int NQ = NT * 8;
    static constexpr int NS = NSR > Stages<NT>::N ? NSR : Stages<NT>::N;
    uint8_t  tile[NS][TILE_BYTES];       // after the tile loop: the unit's O rows [NQ][HD] fp32
    uint8_t  qq[NQ * QSTR];
    float    qd[NBLK * NQ];
    LaneShared<NT> ln;
    float    ml[2 * NQ];                 // the unit's m (log2 domain) and l per row
    uint64_t full[NS];
    int32_t  stage_blk[NS];              // block id of the tile in each stage (-1 skip, < -1 error)
};

struct Unit {
    int s, h, p;          // plan position of the sequence, KV head, pair = s * n_head_kv + h
    int io;               // the sequence's index in the caller's arrays (Q, out, K/V new, selection)
    int t0, t1;           // tile range of the pair this unit runs
    int pu0, pu1;         // unit range of the pair
};

__device__ __forceinline__ Unit unit_of(const DecodeParams &P, int u) {
    int lo = 0, hi = P.n_seq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.seq_unit0[mid] <= u) lo = mid; else hi = mid - 1;
    }
    Unit x;
    x.s = lo;
    x.io = P.seq_idx[lo];
    const int per = P.seq_units[lo], tiles = P.seq_tiles[lo];
    const int off = u - P.seq_unit0[lo];
    x.h = off / per;
    const int r = off % per;
    x.p = lo * P.n_head_kv + x.h;
    // the first tiles % per units take one tile more, so the pair's last unit -- the one holding
    // the newest positions and any fused append -- has the fewest
    const int base = tiles / per, rem = tiles % per;
    x.t0 = r * base + min(r, rem);
    x.t1 = x.t0 + base + (r < rem ? 1 : 0);
    x.pu0 = P.seq_unit0[lo] + x.h * per;
    x.pu1 = x.pu0 + per;
    return x;
}

struct TileRef {
    int32_t  blk;   // block id (64-token tile of the sequence); -1 skip, -2 bad index, -3 bad page
    uint8_t *src;   // global tile address
};

__device__ __forceinline__ TileRef tile_ref(const DecodeParams &P, const Unit &U, int k) {
    TileRef r{-1, nullptr};
    const int blkid = P.sel ? P.sel[((int64_t)U.io * P.n_head_kv + U.h) * P.n_sel + k] : k;
    if (blkid < 0) return r;
    const int n_kv = P.seq_pos0[U.s] + P.T;
    if (blkid >= (n_kv + TILE_TOK - 1) / TILE_TOK) {
        r.blk = -2;
        return r;
    }
    const int32_t page = P.block_table[(int64_t)P.seq_slot[U.s] * P.max_pages + (blkid >> 2)];
    if (page < 0 || page >= P.n_pages) {
        r.blk = -3;
        return r;
    }
    r.blk = blkid;
    r.src = const_cast<uint8_t *>(P.pool) + (int64_t)page * P.page_bytes +
            (int64_t)(U.h * TILES_PER_PAGE + (blkid & 3)) * TILE_BYTES;
    return r;
}

// One thread: start the copy of the unit's i-th tile into stage i % NS.  `withhold` (failure tests
// only) arms the barrier for the tile's bytes but starts no copy, so the wait for it runs out.
// A stage that the CTA's warps have read before is fenced against the copy's (async-proxy)
// writes; a stage's first copy needs no fence.
template <typename SM>
__device__ __forceinline__ void issue_ref(const DecodeParams &P, SM &sm, const TileRef &r, int i, bool withhold) {
    constexpr int NS = SM::NS;
    uint64_t *bar = &sm.full[i % NS];
    sm.stage_blk[i % NS] = r.blk;    // published to the consumers by the barrier's completion
    if (r.blk >= 0) {
        if (i >= NS) fence_proxy_async();
        mbar_expect_tx(bar, TILE_BYTES);
        if (!withhold) bulk_load(sm.tile[i % NS], r.src, TILE_BYTES, bar);
    } else {
        if (r.blk < -1) atomicOr(P.status, r.blk == -2 ? ST_BAD_INDEX : ST_BAD_PAGE);
        mbar_arrive(bar);
    }
}
template <typename SM>
__device__ __forceinline__ void issue_tile(const DecodeParams &P, SM &sm, const Unit &U, int i) {
    issue_ref(P, sm, tile_ref(P, U, U.t0 + i), i, false);
}

// QSA mode: tile k of a sequence is its kept blocks 16k .. 16k+15 (4 cells each).  Thread tid
// serves block g = tid >> 3 of the tile: it resolves the block's source (its 4 cells in the slot's
// page tile), then copies an eighth of them -- 8 of the 64 16-byte K chunks (re-swizzled for the
// destination rows), one token's K scales (threads 0-3), 32 of the 256 4-byte V words (the 4 cells
// of one dim are one word of the transposed V) and one block's 4 V scales -- and arrives on the
// stage barrier (128 arrivals per phase) when they have landed.  Slots past the kept list copy the
// last kept block: their cells lie past the sequence's length and are masked.
struct GrpSrc {
    const uint8_t *src;   // the block's page tile (nullptr: bad index or page, reported)
    int ts;               // the block's first cell inside it
};
__device__ __forceinline__ GrpSrc grp_resolve(const DecodeParams &P, const Unit &U, int k, int tid) {
    GrpSrc r{nullptr, 0};
    const int ng = P.grp_n[U.io];
    if (ng < 1) return r;
    const int j = min(16 * k + (tid >> 3), ng - 1);
    const int32_t b = P.grp[(int64_t)U.io * P.grp_stride + j], c0 = b * 4;
    if (b < 0 || c0 > P.seq_vpos[U.s] || (c0 >> 8) >= P.max_pages) {
        if ((tid & 7) == 0) atomicOr(P.status, ST_BAD_INDEX);
        return r;
    }
    const int32_t page = P.block_table[(int64_t)P.seq_slot[U.s] * P.max_pages + (c0 >> 8)];
    if (page < 0 || page >= P.n_pages) {
        if ((tid & 7) == 0) atomicOr(P.status, ST_BAD_PAGE);
        return r;
    }
    r.src = P.pool + (int64_t)page * P.page_bytes + (int64_t)(U.h * TILES_PER_PAGE + ((c0 >> 6) & 3)) * TILE_BYTES;
    r.ts = c0 & 63;
    return r;
}
template <typename SM>
__device__ __forceinline__ void grp_issue(SM &sm, const GrpSrc &r, int i, int tid) {
    uint8_t *dst = sm.tile[i % SM::NS];
    if (r.src) {
        const int td = 4 * (tid >> 3), q0 = tid & 7;
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const int e = q0 + 8 * q, m = e >> 4, c = e & 15;
            cp_async16(dst + TILE_KQ + (td + m) * HD + ((c ^ kswz(td + m)) << 4),
                       r.src + TILE_KQ + (r.ts + m) * HD + ((c ^ kswz(r.ts + m)) << 4));
        }
        if (q0 < 4) cp_async16(dst + kd_off(td + q0, 0), r.src + kd_off(r.ts + q0, 0));
#pragma unroll 8
        for (int q = 0; q < HD / 8; q++) {
            const int dim = q0 + 8 * q;
            cp_async4(dst + v_off(dim, td), r.src + v_off(dim, r.ts));
        }
        cp_async8(dst + vd_off(q0, td), r.src + vd_off(q0, r.ts));
    }
    cp_async_arrive(&sm.full[i % SM::NS]);
}

// Quantise the new rows of this tile (positions pos0..pos0+T-1 inside it) for KV head h and store
// them in the cache tile in global memory.  One thread per (row, 32-element block, K or V): it
// loads its 32 values with eight vector loads and rounds them exactly as kernel A does.
__device__ __forceinline__ void fused_append(const DecodeParams &P, const Unit &U, uint8_t *gtile, int cell0) {
    const int pos0 = P.seq_pos0[U.s];
    const int r0 = max(pos0, cell0), r1 = min(pos0 + P.T, cell0 + TILE_TOK);
    const int work = (r1 - r0) * NBLK * 2;   // at most 4 * 8 * 2 = 64 <= blockDim
    const int wi = threadIdx.x;
    if (wi >= work) return;
    const int kv = wi & 1, b = (wi >> 1) % NBLK, row = r0 + (wi >> 1) / NBLK;
    const float4 *src = reinterpret_cast<const float4 *>(
        (kv ? P.Vnew : P.Knew) + (((int64_t)U.io * P.T + (row - pos0)) * P.n_head_kv + U.h) * HD + b * QK);
    float x[QK];
#pragma unroll
    for (int i = 0; i < QK / 4; i++) {
        const float4 v = src[i];
        x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
    }
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < QK; i++) amax = fmaxf(amax, fabsf(x[i]));
    const float d  = div127_rn(amax);
    const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
    uint32_t q[QK / 4];
#pragma unroll
    for (int i = 0; i < QK / 4; i++) {
        q[i] = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) q[i] |= (uint32_t)(uint8_t)(int8_t)round_half_away(__fmul_rn(x[4 * i + e], id)) << (8 * e);
    }
    const int t = row - cell0;
    if (!kv) {   // two swizzled 16-byte chunks of the token's K row
        *reinterpret_cast<uint4 *>(gtile + TILE_KQ + t * HD + (((2 * b) ^ kswz(t)) << 4)) = make_uint4(q[0], q[1], q[2], q[3]);
        *reinterpret_cast<uint4 *>(gtile + TILE_KQ + t * HD + (((2 * b + 1) ^ kswz(t)) << 4)) = make_uint4(q[4], q[5], q[6], q[7]);
    } else {     // V is stored transposed: one byte in each of the block's 32 dims
#pragma unroll
        for (int e = 0; e < QK; e++) gtile[v_off(b * QK + e, t)] = (uint8_t)(q[e >> 2] >> (8 * (e & 3)));
    }
    *reinterpret_cast<__half *>(gtile + (kv ? vd_off(b, t) : kd_off(t, b))) = __float2half_rn(d);
}

// Row state a thread carries through the tile loop: for its two query rows per 8-row group j
// (rows 8j + 2tig + e), the last visible position, the softmax reference (log2 domain, the same in
// every warp that works on the unit), its row sums over its own tokens, and its 64 dims of O.
template <int NT>
struct RowState {
    int   qlim[NT][2];
    float mref[NT][2];
    float lsum[NT][2];
    float O[4][NT][4];
};

template <int NT>
__device__ __forceinline__ void row_state_init(RowState<NT> &rs, int nq, int G, int pos0, int tig) {
#pragma unroll
    for (int j = 0; j < NT; j++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int n = 8 * j + 2 * tig + e;
            rs.qlim[j][e] = n < nq ? pos0 + n / G : -1;
            rs.mref[j][e] = -INFINITY;
            rs.lsum[j][e] = 0.0f;
        }
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int j = 0; j < NT; j++) rs.O[mt][j][0] = rs.O[mt][j][1] = rs.O[mt][j][2] = rs.O[mt][j][3] = 0.0f;
}

// Barrier of the four warps that share a tile (the whole CTA).
struct CtaSync {
    __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// One 64-token tile for the four warps w = 0..3 that share it: QK for the warp's 16 tokens, the
// causal mask, the lazily rescaled softmax (P through `ls.ps`), and PV for the warp's 64 dims.
// Ends after PV; the caller's next barrier frees the tile's stage and P.
template <int NT, class Sync>
__device__ __forceinline__ void tile_step(const uint8_t *tile, int blk, bool live, const uint8_t *qq, const float *qd,
                                          LaneShared<NT> &ls, RowState<NT> &rs, float c2, int w, int lane,
                                          const Sync &sync TLT_ARG) {
    constexpr int NQ = NT * 8;
    const int g = lane >> 2, tig = lane & 3;
    const int lm = lane & 7, lmat = lane >> 3;
    const int k_tok = 16 * w + pi16(lm + 8 * (lmat & 1));   // K row this lane addresses in ldmatrix
    const int k_key = kswz(k_tok), k_hi = lmat >> 1;
    const int tk_lo = 16 * w + pi16(g), tk_hi = 16 * w + pi16(g + 8);   // tokens of the S rows
    const int v_dim0 = 64 * w + 8 * lmat + lm;   // V^T row this lane addresses (+32: second block)
    const int cell0 = blk * TILE_TOK;
    // ---------------- QK for this warp's 16 tokens ----------------------------------------
    float S[NT][4];
#pragma unroll
    for (int j = 0; j < NT; j++) S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.0f;
    if (live) {
        const __half *dkl_h = reinterpret_cast<const __half *>(tile + TILE_KD + tk_lo * 16);
        const __half *dkh_h = reinterpret_cast<const __half *>(tile + TILE_KD + tk_hi * 16);
        const uint32_t kbase = smem_u32(tile) + k_tok * HD;
        // the A fragments are loaded one block ahead of their MMAs
        uint32_t af[2][4];
        ldsm_x4(kbase + ((k_hi ^ k_key) << 4), af[0][0], af[0][1], af[0][2], af[0][3]);
#pragma unroll
        for (int b = 0; b < NBLK; b++) {
            if (b + 1 < NBLK)
                ldsm_x4(kbase + (((2 * (b + 1) + k_hi) ^ k_key) << 4), af[(b + 1) & 1][0], af[(b + 1) & 1][1],
                        af[(b + 1) & 1][2], af[(b + 1) & 1][3]);
            const uint32_t a0 = af[b & 1][0], a1 = af[b & 1][1], a2 = af[b & 1][2], a3 = af[b & 1][3];
            const float dlo = __half2float(dkl_h[b]), dhi = __half2float(dkh_h[b]);
#pragma unroll
            for (int j = 0; j < NT; j++) {
                const uint2 bq = *reinterpret_cast<const uint2 *>(qq + (8 * j + g) * QSTR + b * 32 + tig * 8);
                uint32_t dd[4];
                mma_s8(dd, a0, a1, a2, a3, bq.x, bq.y, MAGIC_I);
                const float2 dq = *reinterpret_cast<const float2 *>(&qd[b * NQ + 8 * j + 2 * tig]);
                const float2 f01 = __fadd2_rn(make_float2(__uint_as_float(dd[0]), __uint_as_float(dd[1])),
                                              make_float2(-MAGIC_F, -MAGIC_F));
                const float2 f23 = __fadd2_rn(make_float2(__uint_as_float(dd[2]), __uint_as_float(dd[3])),
                                              make_float2(-MAGIC_F, -MAGIC_F));
                const float2 wlo = __fmul2_rn(dq, make_float2(dlo, dlo));
                const float2 whi = __fmul2_rn(dq, make_float2(dhi, dhi));
                const float2 s01 = __ffma2_rn(f01, wlo, make_float2(S[j][0], S[j][1]));
                const float2 s23 = __ffma2_rn(f23, whi, make_float2(S[j][2], S[j][3]));
                S[j][0] = s01.x; S[j][1] = s01.y; S[j][2] = s23.x; S[j][3] = s23.y;
            }
        }
    }
    TLT(0);
    // ---------------- mask; does this warp outgrow the reference? -----------------------
    const int clo = cell0 + tk_lo, chi = cell0 + tk_hi;
    bool over = false;
#pragma unroll
    for (int j = 0; j < NT; j++) {
        if (!live || clo > rs.qlim[j][0]) S[j][0] = -INFINITY;
        if (!live || clo > rs.qlim[j][1]) S[j][1] = -INFINITY;
        if (!live || chi > rs.qlim[j][0]) S[j][2] = -INFINITY;
        if (!live || chi > rs.qlim[j][1]) S[j][3] = -INFINITY;
#pragma unroll
        for (int e = 0; e < 4; e++) over = over || S[j][e] * c2 > rs.mref[j][e & 1] + 4.0f;
    }
    const bool warp_over = __any_sync(0xffffffffu, over);
    if (warp_over) {
#pragma unroll
        for (int j = 0; j < NT; j++) {
            float mx0 = fmaxf(S[j][0], S[j][2]), mx1 = fmaxf(S[j][1], S[j][3]);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            if (g == 0) {
                ls.red[w * NQ + 8 * j + 2 * tig]     = mx0 * c2;
                ls.red[w * NQ + 8 * j + 2 * tig + 1] = mx1 * c2;
            }
        }
    }
    if (lane == 0) ls.flag[w] = warp_over;
    // P relative to the current reference (rewritten below if the reference moves)
    float psum[NT][2];
#pragma unroll
    for (int j = 0; j < NT; j++) {
        float pr[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float mm = rs.mref[j][e & 1];
            pr[e] = mm == -INFINITY ? 0.0f : exp2f(fmaf(S[j][e], c2, -mm));
        }
        psum[j][0] = pr[0] + pr[2];
        psum[j][1] = pr[1] + pr[3];
        if (!warp_over) {
            const uint32_t lo = movm_t(pack_f16x2(pr[0], pr[1]));   // tokens 4tig, 4tig+1 of row 8j+g
            const uint32_t hi = movm_t(pack_f16x2(pr[2], pr[3]));   // tokens 4tig+2, 4tig+3
            *reinterpret_cast<uint2 *>(&ls.ps[(8 * j + g) * PSTR + 16 * w + 4 * tig]) = make_uint2(lo, hi);
        }
    }
    sync();   // barrier 1: P (or the posted maxima) of every warp are in shared memory
    TLT(1);
    if (ls.flag[0] | ls.flag[1] | ls.flag[2] | ls.flag[3]) {
        // ---- the reference moves: new reference, rescale O and sums, rewrite every P -------
#pragma unroll
        for (int j = 0; j < NT; j++) {
            float alpha[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int n = 8 * j + 2 * tig + e;
                float mn = rs.mref[j][e];
#pragma unroll
                for (int ww = 0; ww < 4; ww++)
                    if (ls.flag[ww]) mn = fmaxf(mn, ls.red[ww * NQ + n]);
                alpha[e] = rs.mref[j][e] == -INFINITY ? 0.0f : exp2f(rs.mref[j][e] - mn);
                rs.mref[j][e] = mn;
                rs.lsum[j][e] *= alpha[e];
            }
            const float2 al = make_float2(alpha[0], alpha[1]);
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                const float2 o01 = __fmul2_rn(make_float2(rs.O[mt][j][0], rs.O[mt][j][1]), al);
                const float2 o23 = __fmul2_rn(make_float2(rs.O[mt][j][2], rs.O[mt][j][3]), al);
                rs.O[mt][j][0] = o01.x; rs.O[mt][j][1] = o01.y; rs.O[mt][j][2] = o23.x; rs.O[mt][j][3] = o23.y;
            }
            float pr[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float mm = rs.mref[j][e & 1];
                pr[e] = mm == -INFINITY ? 0.0f : exp2f(fmaf(S[j][e], c2, -mm));
            }
            psum[j][0] = pr[0] + pr[2];
            psum[j][1] = pr[1] + pr[3];
            const uint32_t lo = movm_t(pack_f16x2(pr[0], pr[1]));
            const uint32_t hi = movm_t(pack_f16x2(pr[2], pr[3]));
            *reinterpret_cast<uint2 *>(&ls.ps[(8 * j + g) * PSTR + 16 * w + 4 * tig]) = make_uint2(lo, hi);
        }
        sync();   // rewritten P visible
    }
#pragma unroll
    for (int j = 0; j < NT; j++) {
        rs.lsum[j][0] += psum[j][0];
        rs.lsum[j][1] += psum[j][1];
    }
    TLT(2);
    // ---------------- PV for this warp's 64 dims ------------------------------------------
    if (live) {
        const uint32_t vbase = smem_u32(tile) + TILE_VQ;
        // V^T fragments one 16-token step ahead of their MMAs
        uint32_t vf[2][8];
        auto load_v = [&](int kk, uint32_t (&va)[8]) {
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const int dim = v_dim0 + 32 * half;
                ldsm_x4(vbase + dim * TILE_TOK + ((kk ^ ((dim >> 1) & 3)) << 4), va[4 * half], va[4 * half + 1],
                        va[4 * half + 2], va[4 * half + 3]);
            }
        };
        load_v(0, vf[0]);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            if (kk + 1 < 4) load_v(kk + 1, vf[(kk + 1) & 1]);
            const uint32_t (&va)[8] = vf[kk & 1];
#pragma unroll
            for (int bb = 0; bb < 2; bb++) {   // the warp's two q8_0 blocks (32 dims each)
                const int blkv = 2 * w + bb;
                const uint2 dv =
                    *reinterpret_cast<const uint2 *>(tile + TILE_VD + (blkv * TILE_TOK + 16 * kk + 4 * tig) * 2);
                uint32_t alo[2], ahi[2], blo[2], bhi[2];
                s8x4_to_f16(va[4 * bb + 0], alo[0], ahi[0]);
                s8x4_to_f16(va[4 * bb + 1], alo[1], ahi[1]);
                s8x4_to_f16(va[4 * bb + 2], blo[0], bhi[0]);
                s8x4_to_f16(va[4 * bb + 3], blo[1], bhi[1]);
#pragma unroll
                for (int j = 0; j < NT; j++) {
                    const uint2 pb = *reinterpret_cast<const uint2 *>(&ls.ps[(8 * j + g) * PSTR + 16 * kk + 4 * tig]);
                    const uint32_t b0 = hmul2(pb.x, dv.x), b1 = hmul2(pb.y, dv.y);
                    mma_f16(rs.O[2 * bb][j], alo[0], alo[1], ahi[0], ahi[1], b0, b1);
                    mma_f16(rs.O[2 * bb + 1][j], blo[0], blo[1], bhi[0], bhi[1], b0, b1);
                }
            }
        }
    }
#ifdef QKV_TIMELINE
    if (tli >= 0) {   // the accumulators are complete once this warp's MMAs have retired
        float z = 0.0f;
#pragma unroll
        for (int j = 0; j < NT; j++) z += rs.O[0][j][0] + rs.O[3][j][3];
        if (threadIdx.x == 0) tl_[tli + 3] = global_ns() + (z == 12345.0f ? 1 : 0);
    }
#endif
}


// Throughput mode (k_decode): CTA = 4 warps, up to 4 CTAs per SM, one unit per CTA.  Per 64-token
// tile, warp w computes QK for tokens 16w..16w+15 and PV for dims 64w..64w+63; P crosses between
// them through shared memory.  The softmax uses a per-row reference held in registers (identical
// in every warp); a warp whose scores outgrow it by more than 2^4 posts its maximum and the whole
// CTA moves the reference (rescaling O and the row sums) before PV -- rare after the first tile,
// so a tile normally costs two barriers: P ready, stage free.
template <int NT, int NSR, bool QSA>
__global__ void __launch_bounds__(128, NT <= 3 ? 4 : 2) k_decode(const DecodeParams P) {
    constexpr int NQ = NT * 8;
    using SM = Smem<NT, NSR>;
    constexpr int NS = SM::NS;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    SM &sm = *reinterpret_cast<SM *>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, tig = lane & 3;
    const int u = blockIdx.x;
    TL_DECL
    TL(0);
    // The next launch on the stream may start as soon as every CTA of this one got here; it then
    // waits (below) until this grid has completed and its writes are visible.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bool has_unit = u < P.n_units;
    Unit U{};
    int n_tiles = 0;
    TileRef first[NS];      // thread 0: the unit's first tiles
    if (has_unit) {
        U = unit_of(P, u);   // kernel parameters only
        n_tiles = U.t1 - U.t0;
        // While the previous kernel finishes, pull this unit's query rows and first tiles into L2.
        // No kernel of this library writes queries or the block table; a page the previous
        // launch appends to is updated in L2 by those stores, so a prefetch is never stale.
        // (Selected block ids come from the previous kernel: sparse units prefetch queries only.)
        const float *qsrc = P.Q + (int64_t)U.io * P.T * P.n_head * HD + U.h * P.G * HD;
        for (int e = tid; e < P.nq * (HD * 4 / 128); e += 128) {
            const int n = e / (HD * 4 / 128), t = n / P.G, jj = n % P.G;
            prefetch_l2(qsrc + ((int64_t)t * P.n_head + jj) * HD + (e % (HD * 4 / 128)) * 32);
        }
#ifdef QKV_TIMELINE
        if (!P.sel && !QSA && tid < min(n_tiles, PF_TILES) && !P.tl_nopf) {
#else
        if (!P.sel && !QSA && tid < min(n_tiles, PF_TILES)) {
#endif
            const TileRef r = tile_ref(P, U, U.t0 + tid);
            if (r.blk >= 0) bulk_prefetch_l2(r.src, TILE_BYTES);
        }
        // thread 0: the barriers, and the first tiles' pages (dense), resolved before the wait
        if (tid == 0) {
            for (int st = 0; st < NS; st++) {
                mbar_init(&sm.full[st], QSA ? 128 : 1);   // QSA mode: every thread's copies arrive
                first[st] = !P.sel && !QSA && st < n_tiles ? tile_ref(P, U, U.t0 + st) : TileRef{-1, nullptr};
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
    }
    // Everything global below (pages, block table, queries, new rows, scratch, output) may have
    // been written by the previous kernel on the stream: wait for it to complete.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    TL(1);
    float *obuf = reinterpret_cast<float *>(sm.tile[0]);   // [NQ][OSTR], valid after the tile loop
    bool aborted = false;

    if (has_unit) {
        const bool withhold = u == P.withhold_unit;
        const int pos0 = P.seq_pos0[U.s];
#ifdef QKV_TIMELINE
        if (tid == 0) tl_[9] = global_ns() + (pos0 == -12345 ? 1 : 0);   // pos0 resolved
#endif
        const float c2 = P.scale * 1.4426950408889634f;   // softmax in base 2
        // ---- query rows: 32 threads per row, 8 elements each (4 threads per 32-element block) ---
        const float *qsrc = P.Q + (int64_t)U.io * P.T * P.n_head * HD + U.h * P.G * HD;
        constexpr int QP = (NQ + 3) / 4;   // rows per warp
        // fused append (dense only): tiles nb_lo .. nb_hi hold the T new positions; the unit that
        // owns one writes the new rows into the page before it copies that tile in (below)
        const int nb_lo = pos0 / TILE_TOK, nb_hi = (pos0 + P.T - 1) / TILE_TOK;
        const bool appends = P.Knew != nullptr && U.t1 > nb_lo && U.t0 <= nb_hi;
        if (appends) {   // the new rows' 128-byte blocks, into L1 now for the append below
            const int r0 = max(pos0, max(U.t0, nb_lo) * TILE_TOK), nrow = min(pos0 + P.T, U.t1 * TILE_TOK) - r0;
            if (tid < nrow * NBLK * 2) {
                const int kv = tid & 1, b = (tid >> 1) % NBLK, row = r0 + (tid >> 1) / NBLK;
                const float *src = (kv ? P.Vnew : P.Knew) + (((int64_t)U.io * P.T + (row - pos0)) * P.n_head_kv + U.h) * HD + b * QK;
                asm volatile("prefetch.global.L1 [%0];" ::"l"(src));
            }
        }
        float qv[QP][8];
#pragma unroll
        for (int it = 0; it < QP; it++) {
            const int n = it * 4 + w;
            if (n < P.nq) {
                const int t = n / P.G, jj = n % P.G;
                const float4 *src = reinterpret_cast<const float4 *>(qsrc + ((int64_t)t * P.n_head + jj) * HD + lane * 8);
                const float4 u0 = src[0], u1 = src[1];
                qv[it][0] = u0.x; qv[it][1] = u0.y; qv[it][2] = u0.z; qv[it][3] = u0.w;
                qv[it][4] = u1.x; qv[it][5] = u1.y; qv[it][6] = u1.z; qv[it][7] = u1.w;
            } else {
#pragma unroll
                for (int q = 0; q < 8; q++) qv[it][q] = 0.0f;
            }
        }
        // thread 0 starts the first tiles' copies once its query loads are in flight (sparse
        // units resolve their block ids only now: the previous kernel wrote them)
        if (tid == 0 && !QSA) {
            if (P.sel)
                for (int st = 0; st < NS; st++) first[st] = st < n_tiles ? tile_ref(P, U, U.t0 + st) : TileRef{-1, nullptr};
            for (int st = 0; st < NS && st < n_tiles; st++)
                if (!(appends && U.t0 + st >= nb_lo && U.t0 + st <= nb_hi)) issue_ref(P, sm, first[st], st, withhold && st == 0);
        }
        if constexpr (QSA) {   // every thread's share of the first tiles, behind its query loads
            __syncthreads();   // thread 0 initialised the stage barriers (before the dependency wait)
            for (int st = 0; st < NS && st < n_tiles; st++) grp_issue(sm, grp_resolve(P, U, U.t0 + st, tid), st, tid);
        }
        TL(6);
#ifdef QKV_TIMELINE
        if (tid == 0) tl_[18] = global_ns() + (qv[0][0] == -12345.0f ? 1 : 0);   // thread 0's query values in
        {
            float z = 0.0f;
#pragma unroll
            for (int it = 0; it < QP; it++) z += qv[it][0] + qv[it][7];
            if (tid == 0) tl_[19] = global_ns() + (z == -12345.0f ? 1 : 0);        // all of them
        }
#endif
        // q8_0 quantisation exactly as ggml's CPU flash_attn_ext converts its query row.  Each step
        // runs over all of the warp's rows before the next (block maxima, then d = amax / 127 and
        // 1 / d, then the rounding), so the rows' dependent chains overlap instead of queueing.
        {
            const int b = lane >> 2, sub = lane & 3;
            float d[QP], id[QP];
#pragma unroll
            for (int it = 0; it < QP; it++) {
                float amax = 0.0f;
#pragma unroll
                for (int q = 0; q < 8; q++) amax = fmaxf(amax, fabsf(qv[it][q]));
                d[it] = amax;
            }
#pragma unroll
            for (int it = 0; it < QP; it++) d[it] = fmaxf(d[it], __shfl_xor_sync(0xffffffffu, d[it], 1));
#pragma unroll
            for (int it = 0; it < QP; it++) d[it] = fmaxf(d[it], __shfl_xor_sync(0xffffffffu, d[it], 2));
#pragma unroll
            for (int it = 0; it < QP; it++) d[it] = div127_rn(d[it]);
#pragma unroll
            for (int it = 0; it < QP; it++) id[it] = d[it] != 0.0f ? rcp_rn(d[it]) : 0.0f;
#pragma unroll
            for (int it = 0; it < QP; it++) {
                const int n = it * 4 + w;
                uint32_t w0 = 0, w1 = 0;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    w0 |= (uint32_t)(uint8_t)(int8_t)round_half_away(__fmul_rn(qv[it][q], id[it])) << (8 * q);
                    w1 |= (uint32_t)(uint8_t)(int8_t)round_half_away(__fmul_rn(qv[it][4 + q], id[it])) << (8 * q);
                }
                if (n < NQ) {
                    uint8_t *row = sm.qq + n * QSTR + b * 32;
                    *reinterpret_cast<uint32_t *>(row + qperm(sub * 8)) = w0;
                    *reinterpret_cast<uint32_t *>(row + qperm(sub * 8 + 4)) = w1;
                    if (sub == 0) sm.qd[b * NQ + n] = __half2float(__float2half_rn(d[it]));
                }
            }
        }
        TL(7);
        RowState<NT> rs;
        row_state_init(rs, P.nq, P.G, pos0, tig);
        if (appends) {
            for (int t = max(U.t0, nb_lo); t <= min(U.t1 - 1, nb_hi); t++) {
                const TileRef r = tile_ref(P, U, t);
                if (r.blk >= 0) fused_append(P, U, r.src, t * TILE_TOK);
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");   // the rows before the bulk copy reads them
        }
        __syncthreads();   // query rows ready, barriers initialised
        TL(2);
        if (appends && tid == 0)   // the first tiles held back for the append
            for (int st = 0; st < NS && st < n_tiles; st++)
                if (U.t0 + st >= nb_lo && U.t0 + st <= nb_hi) issue_ref(P, sm, first[st], st, withhold && st == 0);

        for (int i = 0; i < n_tiles; i++) {
            const int stage = i % NS;
            const bool landed = mbar_wait(&sm.full[stage], (uint32_t)((i / NS) & 1),
                                          aborted ? after_abort(P.wait_ns) : P.wait_ns);
            aborted = aborted || !__all_sync(0xffffffffu, landed);
            if (i == 0) TL(8);
            const int blk = QSA ? U.t0 + i : sm.stage_blk[stage];
            tile_step<NT>(sm.tile[stage], blk, blk >= 0 && !aborted, sm.qq, sm.qd, sm.ln, rs, c2, w, lane, CtaSync{} TLT_PASS(i == 0 ? 10 : i == 1 ? 14 : -1));
            __syncthreads();   // barrier 2: the stage and P are free
            // After a wait that gave up no new copy starts: every copy this CTA issued has then
            // been waited for (bounded) by the time it exits.
            if (i + NS < n_tiles && !aborted) {
                if constexpr (QSA) grp_issue(sm, grp_resolve(P, U, U.t0 + i + NS, tid), i + NS, tid);
                else if (tid == 0) issue_tile(P, sm, U, i + NS);
            }
            if (i == 0) TL(3);
        }
        if constexpr (QSA) asm volatile("cp.async.wait_all;" ::: "memory");   // nothing of this thread still in flight
        TL(4);
        // ---------------- unit epilogue: O, m, l into shared memory ------------------------------
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                float v = rs.lsum[j][e];
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (g == 0) sm.ln.lpart[w * NQ + 8 * j + 2 * tig + e] = v;
            }
#pragma unroll
        for (int j = 0; j < NT; j++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int n = 8 * j + 2 * tig + e;
#pragma unroll
                for (int mt = 0; mt < 4; mt++) {
                    const int d0 = 64 * w + 16 * mt + g;
                    obuf[n * OSTR + d0]     = rs.O[mt][j][e];
                    obuf[n * OSTR + d0 + 8] = rs.O[mt][j][2 + e];
                }
            }
        __syncthreads();
        if (w == 0 && g == 0) {
#pragma unroll
            for (int j = 0; j < NT; j++)
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    const int n = 8 * j + 2 * tig + e;
                    const float *lp = sm.ln.lpart;
                    sm.ml[n] = rs.mref[j][e];   // log2 domain
                    sm.ml[NQ + n] = lp[n] + lp[NQ + n] + lp[2 * NQ + n] + lp[3 * NQ + n];
                }
        }
        if (aborted && lane == 0) atomicOr(P.status, ST_TIMEOUT);
        __syncthreads();
        // ---------------- the unit's result: the output itself when the pair has one unit, else
        // its partial record for k_decode_merge.  Thread: float4 column tid & 63 of rows
        // (tid >> 6) + 2i, so each row's 1 KiB is written by 64 adjacent threads.
        const bool single = U.pu1 - U.pu0 == 1;
        float *rec = P.partial + (int64_t)u * partial_stride(P.nq);
        const int q4 = tid & 63;
        for (int n = tid >> 6; n < P.nq; n += 2) {
            const float4 o = reinterpret_cast<const float4 *>(obuf + n * OSTR)[q4];
            if (single) {
                const float L = sm.ml[NQ + n], inv = L == 0.0f ? 0.0f : 1.0f / L;
                const int t = n / P.G, jj = n % P.G;
                float *orow = P.out + (((int64_t)U.io * P.T + t) * P.n_head + U.h * P.G + jj) * HD;
                reinterpret_cast<float4 *>(orow)[q4] = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
            } else {
                reinterpret_cast<float4 *>(rec + n * HD)[q4] = o;
            }
        }
        if (!single && tid < P.nq) {
            rec[P.nq * HD + tid] = sm.ml[tid];
            rec[P.nq * HD + P.nq + tid] = sm.ml[NQ + tid];
        }
        TL(5);
        TL_FLUSH(2);
    }
}


// Merge of the partial records of the pairs with more than one unit (plan positions first, so
// pairs 0 .. n_merge-1): CTA = (pair, query row, 1/SPLIT of the dims), MG_THREADS threads.
// O = sum_u 2^(m_u - M) O_u / sum_u 2^(m_u - M) l_u in a fixed order: thread group gi (one float4
// column of the CTA's dims each) sums the units gi, gi + MG_GROUPS, ... and the groups are added in
// order.  The first MG_GROUPS * MG_UNROLL units' O columns are loaded together with (m, l), so a
// pair of up to that many units costs one round trip to L2.  SPLIT is chosen per launch so that
// the grid stays within two CTAs per SM: then it is resident (waiting) while k_decode runs, and
// the next launch on the stream can launch and become resident as the decode CTAs leave.
constexpr int MG_THREADS = 512, MG_MAX_UNITS = 1024;
static_assert(MG_MAX_UNITS <= 2 * MG_THREADS, "two (m, l) pairs per thread");
template <int SPLIT>
__global__ void __launch_bounds__(MG_THREADS) k_decode_merge(const DecodeParams P) {
    constexpr int MG_LANES = HD / 4 / SPLIT, MG_GROUPS = MG_THREADS / MG_LANES;
    constexpr int MG_UNROLL = SPLIT == 2 ? 9 : 8;   // units per thread loaded at once (registers <= 64)
    __shared__ float wgt[MG_MAX_UNITS];
    __shared__ float4 part[MG_GROUPS][MG_LANES];
    __shared__ float red[2][MG_THREADS / 32];
    // The next launch on the stream may become resident now; it waits for this grid.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    TL_DECL
    TL(0);
    const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
    const int dq = blockIdx.x % SPLIT, rowid = blockIdx.x / SPLIT;
    const int pair = rowid / P.nq, n = rowid % P.nq;
    const int s = pair / P.n_head_kv, h = pair % P.n_head_kv;
    const int nu = min(P.seq_units[s], MG_MAX_UNITS), u0 = P.seq_unit0[s] + h * P.seq_units[s];
    const int64_t stride = partial_stride(P.nq);
    const int gi = tid / MG_LANES, ql = tid % MG_LANES, q4 = dq * MG_LANES + ql;
    asm volatile("griddepcontrol.wait;" ::: "memory");   // the records of k_decode
    TL(1);
    const float *base = P.partial + (int64_t)u0 * stride;
    auto ocol = [&](int i) {   // this thread's float4 of unit i's row (i clamped into range)
        return __ldcg(reinterpret_cast<const float4 *>(base + (int64_t)min(i, nu - 1) * stride + n * HD) + q4);
    };
    // (m, l) of up to two units per thread, and the first batch of O columns, in flight together
    float m[2], l[2], M = -INFINITY;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int i = tid + k * MG_THREADS;
        m[k] = i < nu ? __ldcg(base + (int64_t)i * stride + P.nq * HD + n) : -INFINITY;
        l[k] = i < nu ? __ldcg(base + (int64_t)i * stride + P.nq * HD + P.nq + n) : 0.0f;
    }
    float4 v[MG_UNROLL];
#pragma unroll
    for (int k = 0; k < MG_UNROLL; k++) v[k] = ocol(gi + k * MG_GROUPS);
    M = fmaxf(m[0], m[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    if (lane == 0) red[0][wp] = M;
    __syncthreads();
    M = red[0][0];
#pragma unroll
    for (int k = 1; k < MG_THREADS / 32; k++) M = fmaxf(M, red[0][k]);
    float L = 0.0f;
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int i = tid + k * MG_THREADS;
        const float w = m[k] == -INFINITY ? 0.0f : exp2f(m[k] - M);
        if (i < nu) wgt[i] = w;
        L = fmaf(w, l[k], L);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) red[1][wp] = L;
    __syncthreads();   // weights and partial sums visible
    L = 0.0f;
#pragma unroll
    for (int k = 0; k < MG_THREADS / 32; k++) L += red[1][k];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i0 = gi;; i0 += MG_GROUPS * MG_UNROLL) {
#pragma unroll
        for (int k = 0; k < MG_UNROLL; k++) {
            const int i = i0 + k * MG_GROUPS;
            const float w = i < nu ? wgt[i] : 0.0f;
            acc.x = fmaf(v[k].x, w, acc.x);
            acc.y = fmaf(v[k].y, w, acc.y);
            acc.z = fmaf(v[k].z, w, acc.z);
            acc.w = fmaf(v[k].w, w, acc.w);
        }
        if (i0 + MG_GROUPS * MG_UNROLL >= nu) break;
#pragma unroll
        for (int k = 0; k < MG_UNROLL; k++) v[k] = ocol(i0 + MG_GROUPS * MG_UNROLL + k * MG_GROUPS);
    }
    part[gi][ql] = acc;
    __syncthreads();
    if (tid < MG_LANES) {
        float4 o = part[0][tid];
#pragma unroll
        for (int k = 1; k < MG_GROUPS; k++) {
            const float4 b = part[k][tid];
            o.x += b.x; o.y += b.y; o.z += b.z; o.w += b.w;
        }
        const float inv = L == 0.0f ? 0.0f : 1.0f / L;
        const int t = n / P.G, jj = n % P.G;
        float *orow = P.out + (((int64_t)P.seq_idx[s] * P.T + t) * P.n_head + h * P.G + jj) * HD;
        reinterpret_cast<float4 *>(orow)[dq * MG_LANES + tid] = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    }
    TL(2);
    TL_FLUSH(3);
}

// The same merge for pairs of at most MR_MAX_UNITS units (wide batches: many pairs, few units
// each): CTA = (pair, MR_ROWS query rows), 64 threads per row, one float4 column each; every
// thread loads the (m, l) and O columns of all the pair's units at once and sums them in unit
// order.
constexpr int MR_ROWS = 8, MR_MAX_UNITS = 16;
__global__ void __launch_bounds__(64 * MR_ROWS) k_decode_merge_rows(const DecodeParams P) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    TL_DECL
    TL(0);
    const int tid = threadIdx.x, q4 = tid & 63;
    const int nrb = (P.nq + MR_ROWS - 1) / MR_ROWS;
    const int pair = blockIdx.x / nrb, n = (blockIdx.x % nrb) * MR_ROWS + (tid >> 6);
    const int s = pair / P.n_head_kv, h = pair % P.n_head_kv;
    const int nu = min(P.seq_units[s], MR_MAX_UNITS), u0 = P.seq_unit0[s] + h * P.seq_units[s];
    const int64_t stride = partial_stride(P.nq);
    asm volatile("griddepcontrol.wait;" ::: "memory");   // the records of k_decode
    TL(1);
    if (n >= P.nq) {
        TL_FLUSH(4);
        return;
    }
    const float *base = P.partial + (int64_t)u0 * stride;
    float m[MR_MAX_UNITS], l[MR_MAX_UNITS];
    float4 v[MR_MAX_UNITS];
#pragma unroll
    for (int k = 0; k < MR_MAX_UNITS; k++) {
        if (k < nu) {
            const float *rec = base + (int64_t)k * stride;
            m[k] = __ldcg(rec + P.nq * HD + n);
            l[k] = __ldcg(rec + P.nq * HD + P.nq + n);
            v[k] = __ldcg(reinterpret_cast<const float4 *>(rec + n * HD) + q4);
        } else {
            m[k] = -INFINITY;
            l[k] = 0.0f;
            v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < MR_MAX_UNITS; k++) M = fmaxf(M, m[k]);
    float L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < MR_MAX_UNITS; k++) {
        const float w = m[k] == -INFINITY ? 0.0f : exp2f(m[k] - M);
        L = fmaf(w, l[k], L);
        acc.x = fmaf(v[k].x, w, acc.x);
        acc.y = fmaf(v[k].y, w, acc.y);
        acc.z = fmaf(v[k].z, w, acc.z);
        acc.w = fmaf(v[k].w, w, acc.w);
    }
    const float inv = L == 0.0f ? 0.0f : 1.0f / L;
    const int t = n / P.G, jj = n % P.G;
    float *orow = P.out + (((int64_t)P.seq_idx[s] * P.T + t) * P.n_head + h * P.G + jj) * HD;
    reinterpret_cast<float4 *>(orow)[q4] = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    TL(2);
    TL_FLUSH(4);
}

}  // namespace dec

// Launch with programmatic stream serialisation: the grid may become resident while the previous
// kernel on the stream finishes (if that kernel triggers, as k_decode and k_decode_merge do); it
// waits (griddepcontrol.wait) before reading anything that kernel may have written.
template <typename K>
static cudaError_t launch_pdl(K kernel, unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                              const DecodeParams &p) {
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
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int NT, int NSR, bool QSA>
static cudaError_t configure_nt() {
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64 && configured[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(dec::k_decode<NT, NSR, QSA>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(dec::Smem<NT, NSR>));
    if (e == cudaSuccess && dev >= 0 && dev < 64) configured[dev] = true;
    return e;
}

// Co-resident CTAs of the decode kernel (0 = unknown).
template <int NT, int NSR, bool QSA = false>
static int max_ctas_nt() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cached[dev]) return cached[dev];
    int per_sm = 0, sms = 0;
    if (configure_nt<NT, NSR, QSA>() != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dec::k_decode<NT, NSR, QSA>, 128, sizeof(dec::Smem<NT, NSR>)) !=
            cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cached[dev] = per_sm * sms;
    return cached[dev];
}

template <int NT, int NSR, bool QSA>
static cudaError_t launch_ns(const DecodeParams &p, cudaStream_t st) {
    cudaError_t e = configure_nt<NT, NSR, QSA>();
    if (e != cudaSuccess) return e;
    if ((e = launch_pdl(dec::k_decode<NT, NSR, QSA>, (unsigned)p.n_units, 128, sizeof(dec::Smem<NT, NSR>), st, p)) !=
        cudaSuccess)
        return e;
    count_launches(1);
    if (p.n_merge > 0) {
        // pairs are in plan order, most units first
        if (p.seq_units[0] <= dec::MR_MAX_UNITS)
            e = launch_pdl(dec::k_decode_merge_rows, (unsigned)(p.n_merge * ((p.nq + dec::MR_ROWS - 1) / dec::MR_ROWS)),
                           64 * dec::MR_ROWS, 0, st, p);
        else {
            // the largest split whose grid fits two CTAs per SM beside the decode grid
            int sms = 148, dev = 0;
            if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
                sms = 148;
            const int64_t rows = (int64_t)p.n_merge * p.nq;
            if (rows * 4 <= 2 * sms)
                e = launch_pdl(dec::k_decode_merge<4>, (unsigned)(rows * 4), dec::MG_THREADS, 0, st, p);
            else if (rows * 2 <= 2 * sms)
                e = launch_pdl(dec::k_decode_merge<2>, (unsigned)(rows * 2), dec::MG_THREADS, 0, st, p);
            else
                e = launch_pdl(dec::k_decode_merge<1>, (unsigned)rows, dec::MG_THREADS, 0, st, p);
        }
        if (e != cudaSuccess) return e;
        count_launches(1);
    }
    return cudaSuccess;
}

// Two tile stages when every unit fits co-resident with them, else one (more CTAs per SM).
// The QSA mode (kept 4-cell blocks read in place) is an instantiation of its own, so the dense and
// selected-block kernels carry none of its code (measured: 2.5% on the ragged batch).
template <int NT, bool QSA = false>
static cudaError_t launch_nt(const DecodeParams &p, cudaStream_t st) {
    if (dec::Stages<NT>::N == 2 || p.n_units <= max_ctas_nt<NT, 2, QSA>()) return launch_ns<NT, 2, QSA>(p, st);
    return launch_ns<NT, 1, QSA>(p, st);
}

int decode_max_nq() { return 64; }
int decode_merge_max_units() { return dec::MG_MAX_UNITS; }

int decode_max_ctas(int nq) {
    switch ((nq + 7) / 8) {
        case 1: return max_ctas_nt<1, 1>();
        case 2: return max_ctas_nt<2, 1>();
        case 3: return max_ctas_nt<3, 1>();
        case 4: return max_ctas_nt<4, 1>();
        case 5: return max_ctas_nt<5, 1>();
        case 6: return max_ctas_nt<6, 1>();
        case 7: return max_ctas_nt<7, 1>();
        case 8: return max_ctas_nt<8, 1>();
        default: return 0;
    }
}

void plan_decode(DecodeParams &P, const int32_t *slots, const int32_t *pos0, const int32_t *tiles, int ns,
                 int64_t target, int64_t umax, int64_t max_units) {
    const int H = P.n_head_kv;
#ifdef QKV_TIMELINE
    P.tl_nopf = getenv("QKV_TL_NOPF") != nullptr;   // analysis builds: no pre-wait tile prefetch
#endif
    std::vector<int32_t> units(ns);
    int64_t total = 0;
    for (int i = 0; i < ns; i++) total += (int64_t)H * tiles[i];
    // Units: proportional to tiles, about one wave of co-resident CTAs in total, at least two
    // tiles each.  A pair with one unit writes its output itself; the units of the others
    // leave partial records for the merge kernel, which takes the pairs at the front of the plan.
    target = std::min(target, max_units);
    double scale_u = (double)target / (double)total;
    int64_t n_units = 0;
    for (int attempt = 0; attempt < 8; attempt++) {
        n_units = 0;
        for (int i = 0; i < ns; i++) {
            int64_t u = (int64_t)((double)tiles[i] * scale_u);
            u = std::min<int64_t>(std::min<int64_t>(u, tiles[i] / 2), umax);
            u = std::max<int64_t>(1, u);
            units[i] = (int32_t)u;
            n_units += u * H;
        }
        if (n_units <= target) break;
        scale_u *= 0.9 * (double)target / (double)n_units;
    }
    // The launch lasts as long as its longest unit: where the budget allows, raise a pair's
    // units until the most tiles any unit gets drops by one.
    for (int i = 0; i < ns; i++) {
        const int64_t u = units[i];
        const int64_t k = (tiles[i] + u - 1) / u;
        if (k <= 1) continue;
        const int64_t u2 = std::min<int64_t>((tiles[i] + k - 2) / (k - 1), umax);
        if (u2 > u && n_units + (u2 - u) * H <= target) {
            n_units += (u2 - u) * H;
            units[i] = (int32_t)u2;
        }
    }
    // plan order: multi-unit pairs first (the merge kernel takes pairs 0 .. n_merge-1)
    std::vector<int32_t> order(ns);
    for (int i = 0; i < ns; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return units[a] > units[b]; });
    int64_t acc = 0;
    int n_multi = 0;
    for (int j = 0; j < ns; j++) {
        const int i = order[j];
        P.seq_idx[j] = i;
        P.seq_slot[j] = slots[i];
        P.seq_pos0[j] = pos0[i];
        P.seq_tiles[j] = tiles[i];
        P.seq_units[j] = units[i];
        P.seq_unit0[j] = (int32_t)acc;
        acc += (int64_t)units[i] * H;
        n_multi += units[i] > 1;
    }
    P.seq_unit0[ns] = (int32_t)acc;
    P.n_units = (int32_t)acc;
    P.n_merge = n_multi * H;
}

cudaError_t launch_decode(const DecodeParams &p, cudaStream_t st) {
    if (p.grp) {   // QSA mode: T = 1, so G query rows (up to 16)
        switch ((p.nq + 7) / 8) {
            case 1: return launch_nt<1, true>(p, st);
            case 2: return launch_nt<2, true>(p, st);
            default: return cudaErrorInvalidValue;
        }
    }
    switch ((p.nq + 7) / 8) {
        case 1: return launch_nt<1>(p, st);
        case 2: return launch_nt<2>(p, st);
        case 3: return launch_nt<3>(p, st);
        case 4: return launch_nt<4>(p, st);
        case 5: return launch_nt<5>(p, st);
        case 6: return launch_nt<6>(p, st);
        case 7: return launch_nt<7>(p, st);
        case 8: return launch_nt<8>(p, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace qkv

// ============================================================================================
// Allocation-free decode: qkv_attn_decode_static (include/qkv.h).
//
// For callers that must not allocate device memory -- e.g. a custom op running inside ggml's
// graph executor, whose memory is planned ahead by ggml-alloc and may not grow mid-graph, or code
// running under an allocator that owns all of the device's memory.  The kernels' split-K scratch
// lives in the file-scope arrays below (6,340,608 bytes = 6.05 MiB of partial records for up to
// 192 units of 32 query rows), allocated once by the CUDA module on every GPU that loads the library and held until exit.
// Every call shares them: calls that overlap on the GPU race.
// ============================================================================================
namespace qkv {
namespace stat {

constexpr int MAX_NQ    = 32;    // query rows per KV head (T * n_head / n_head_kv)
constexpr int MAX_UNITS = 192;   // units (CTAs) per launch
constexpr int64_t PARTIAL_FLOATS = (int64_t)MAX_UNITS * (MAX_NQ * HD + 2 * MAX_NQ);

static __device__ __align__(256) float   g_partial[PARTIAL_FLOATS];
static __device__ __align__(256) int32_t g_status[64];

struct Scratch {
    float   *partial  = nullptr;
    int32_t *status   = nullptr;
};

// Device addresses of the arrays for the current device, resolved once per device.  In host
// code the arrays' names are host-side stand-ins, never device addresses.
static cudaError_t scratch_for_current_device(Scratch &out) {
    static Scratch cached[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!cached[dev].partial) {
        Scratch s;
        if ((e = cudaGetSymbolAddress(reinterpret_cast<void **>(&s.partial), g_partial)) != cudaSuccess) return e;
        if ((e = cudaGetSymbolAddress(reinterpret_cast<void **>(&s.status), g_status)) != cudaSuccess) return e;
        cached[dev] = s;
    }
    out = cached[dev];
    return cudaSuccess;
}

}  // namespace stat
}  // namespace qkv

extern "C" qkv_status qkv_attn_decode_static(const qkv_cache_view *view, int32_t n_slots, const int32_t *slots,
                                             const int32_t *pos0, int32_t n_seq, int32_t n_head, const float *Q,
                                             int32_t T, float scale, float *out, void *stream) {
    using namespace qkv;
    if (!view || !view->pool || !view->block_table || !slots || !pos0 || !Q || !out || n_seq < 1 || n_slots < 1)
        return QKV_ERR_INVALID;
    const int H = view->n_head_kv;
    if (view->head_dim != HD || view->page_tokens != PAGE_TOK || view->tile_tokens != TILE_TOK ||
        view->tile_bytes != (size_t)TILE_BYTES || view->page_bytes != (size_t)H * TILES_PER_PAGE * TILE_BYTES ||
        H < 1 || H > 8 || n_head < 1 || n_head % H || T < 1 || T > 4 || view->n_pages < 1 || view->max_pages_per_seq < 1)
        return QKV_ERR_INVALID;
    const int G = n_head / H;
    if (T * G > stat::MAX_NQ) return QKV_ERR_UNSUPPORTED;   // beyond the static scratch: T*n_head/n_head_kv <= 32
    for (int i = 0; i < n_seq; i++)
        if (slots[i] < 0 || slots[i] >= n_slots || pos0[i] < 0 ||
            (int64_t)pos0[i] + T > (int64_t)view->max_pages_per_seq * PAGE_TOK)
            return QKV_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    stat::Scratch sc;
    if (stat::scratch_for_current_device(sc) != cudaSuccess) return QKV_ERR_CUDA;
    if (cudaMemsetAsync(sc.status, 0, sizeof(int32_t), st) != cudaSuccess) return QKV_ERR_CUDA;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return QKV_ERR_CUDA;
    int max_ctas = decode_max_ctas(T * G);
    if (max_ctas <= 0) max_ctas = sms * 2;
    const int64_t target = std::min<int64_t>(max_ctas, stat::MAX_UNITS);
    // sequences per launch: every pair needs at least one unit within the budget
    const int per_launch = (int)std::min<int64_t>(MAX_SEQ, std::max<int64_t>(1, target / H));
    for (int base = 0; base < n_seq; base += per_launch) {
        const int ns = n_seq - base < per_launch ? n_seq - base : per_launch;
        DecodeParams P;
        memset(&P, 0, sizeof P);
        P.pool = static_cast<const uint8_t *>(view->pool);
        P.block_table = view->block_table;
        P.Q = Q + (size_t)base * T * n_head * HD;
        P.out = out + (size_t)base * T * n_head * HD;
        P.partial = sc.partial;
        P.status = sc.status;
        P.page_bytes = (int64_t)view->page_bytes;
        P.n_pages = view->n_pages;
        P.max_pages = view->max_pages_per_seq;
        P.n_head = n_head;
        P.n_head_kv = H;
        P.G = G;
        P.T = T;
        P.nq = T * G;
        P.n_seq = ns;
        P.scale = scale;
        P.wait_ns = WAIT_NS_DEFAULT;
        P.withhold_unit = -1;
        int32_t tiles[MAX_SEQ];
        for (int i = 0; i < ns; i++) tiles[i] = (pos0[base + i] + T + TILE_TOK - 1) / TILE_TOK;
        plan_decode(P, slots + base, pos0 + base, tiles, ns, target, decode_merge_max_units(), stat::MAX_UNITS);
        if (P.n_units > stat::MAX_UNITS) return QKV_ERR_UNSUPPORTED;
        if (launch_decode(P, st) != cudaSuccess) return QKV_ERR_CUDA;
    }
    return QKV_OK;
}

extern "C" qkv_status qkv_static_status(void *stream, int32_t *code) {
    using namespace qkv;
    if (!code) return QKV_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    stat::Scratch sc;
    if (stat::scratch_for_current_device(sc) != cudaSuccess) return QKV_ERR_CUDA;
    int32_t h = 0;
    if (cudaMemcpyAsync(&h, sc.status, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess || cudaMemsetAsync(sc.status, 0, sizeof(int32_t), st) != cudaSuccess)
        return QKV_ERR_CUDA;
    *code = h;
    return h ? QKV_ERR_DEVICE : QKV_OK;
}

#ifdef QKV_TIMELINE
extern "C" int qkv_tl_read(unsigned long long *host, int max_records) {
    unsigned int n = 0;
    if (cudaMemcpyFromSymbol(&n, qkv::dec::g_tl_n, sizeof n) != cudaSuccess) return -1;
    const int m = (int)(n < (unsigned)max_records ? n : (unsigned)max_records);
    if (m > 0 && cudaMemcpyFromSymbol(host, qkv::dec::g_tl_rec, (size_t)m * 22 * 8) != cudaSuccess) return -1;
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(qkv::dec::g_tl_n, &zero, sizeof zero);
    return m;
}
#endif
