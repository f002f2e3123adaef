// qkv_kernels.cu -- kernel A (q8_0 append), the ggml-layout transforms (read / gather / write
// rows), kernel E (batched device copies) and kernel B (block summaries, block selection).
//
// All of these move or reshape bytes; none is compute bound.  They are written for the HBM:
// 16-byte vector accesses where the layout allows, grids sized from the SM count.
#include "qkv_internal.h"

#include <algorithm>
#include <cooperative_groups.h>
#include <cuda_fp16.h>

namespace qkv {
namespace cg = cooperative_groups;

// The block-table entry of position pos (-1 outside the table), and the tile of KV head h at pos
// in that page (nullptr for an entry outside the pool).
__device__ __forceinline__ int32_t page_of_pos(const PoolRef &pr, int32_t pos) {
    return pos < 0 || (pos >> 8) >= pr.max_pages ? -1 : pr.bt[pos >> 8];
}
__device__ __forceinline__ uint8_t *tile_in_page(const PoolRef &pr, int32_t page, int32_t pos, int h) {
    if (page < 0 || page >= pr.n_pages) return nullptr;
    return pr.pool + (int64_t)page * pr.page_bytes + (int64_t)(h * TILES_PER_PAGE + ((pos >> 6) & 3)) * TILE_BYTES;
}
__device__ __forceinline__ uint8_t *tile_ptr(const PoolRef &pr, int32_t pos, int h) {
    return tile_in_page(pr, page_of_pos(pr, pos), pos, h);
}

// ------------------------------------------------------------------------------------ kernel A
// q8_0 quantisation, restating ggml's quantize_row_q8_0 (and its CUDA set_rows/cpy twin):
// d = amax / 127 (IEEE division), id = d ? 1/d : 0 (IEEE reciprocal), q = roundf(x * id)
// (half away from zero), d stored as fp16 with round-to-nearest-even.  One warp per 32-element
// block: lane j owns element j.
__device__ __forceinline__ void quant_block_warp(float x, int lane, int8_t &q, __half &dh) {
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d  = div127_rn(amax);
    const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
    q  = (int8_t)round_half_away(__fmul_rn(x, id));
    dh = __float2half_rn(d);
    (void)lane;
}

// CTA = (16-token group g, KV head h), 256 threads.  A team of 4 threads quantises one 32-element
// block (8 elements each, amax by two shuffles); a warp's 8 teams cover one token's 256 dims of
// the head, so its loads read 1 KiB contiguously.  K and V quants are staged token-major in shared
// memory (8-byte stores, conflict-free), then each thread writes one 16-byte chunk: a K row's
// chunk, and for its dim the transposed V chunk of the group's 16 tokens, gathered byte by byte
// from the 16 token rows (same-word reads of neighbouring dims).  Only a group that the append
// covers partly (its first or last) writes the transposed V byte by byte.
constexpr int AP_TOK = 16;
// The group's F32 inputs of this thread: 2 teams x (K, V) x 8 elements (team p = token p / 8,
// block p % 8); positions outside [lo, hi) read as zeros.
struct ApIn {
    float x[2][2][8];
};
__device__ __forceinline__ void ap_load(ApIn &in, const float *__restrict__ K, const float *__restrict__ V, int32_t pos,
                                        int32_t g0, int32_t lo, int32_t hi, int n_head_kv, int h, int tid) {
    const int sub = tid & 3;
#pragma unroll
    for (int it = 0; it < 2; it++) {
        const int p = (tid >> 2) + 64 * it, t = p >> 3, b = p & 7;
        const int32_t row = g0 + t;
#pragma unroll
        for (int kv = 0; kv < 2; kv++) {
            if (row >= lo && row < hi) {
                const float4 *src = reinterpret_cast<const float4 *>((kv ? V : K) + (int64_t)(row - pos) * n_head_kv * HD +
                                                                     h * HD + b * QK + sub * 8);
                const float4 u0 = __ldcs(src), u1 = __ldcs(src + 1);   // streamed: read once
                in.x[it][kv][0] = u0.x; in.x[it][kv][1] = u0.y; in.x[it][kv][2] = u0.z; in.x[it][kv][3] = u0.w;
                in.x[it][kv][4] = u1.x; in.x[it][kv][5] = u1.y; in.x[it][kv][6] = u1.z; in.x[it][kv][7] = u1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) in.x[it][kv][e] = 0.0f;
            }
        }
    }
}

// CTA = (16-token group blockIdx.x, KV head blockIdx.y), 256 threads, one wave for 4096-row
// appends: every CTA issues all of its loads at once (a grid-stride loop with the next group's
// loads in flight measured slower: twice the registers, half the CTAs per SM).  A team of 4
// threads quantises one 32-element block (8 elements each, amax by two shuffles); a warp's 8 teams
// cover one token's 256 dims of the head, so its loads read 1 KiB contiguously.  K and V quants
// are staged token-major in shared memory (8-byte stores, conflict-free), then each thread writes
// one 16-byte chunk: a K row's chunk, and for its dim the transposed V chunk of the group's 16
// tokens, gathered byte by byte from the 16 token rows (same-word reads of neighbouring dims).
// Only a group that the append covers partly (its first or last) writes the transposed V byte by
// byte.
__global__ void __launch_bounds__(256) k_append(PoolRef pr, int32_t pos, const float *__restrict__ K,
                                                const float *__restrict__ V, int32_t n_rows) {
    __shared__ __align__(16) uint8_t ks[AP_TOK][HD];            // K quants of the group's tokens
    __shared__ __align__(16) uint8_t vs[AP_TOK][HD];            // V quants of the group's tokens
    __shared__ __align__(16) __half kd[AP_TOK][NBLK];           // K scales [token][block]
    __shared__ __align__(16) __half vd[NBLK][AP_TOK];           // V scales [block][token]
    const int h = blockIdx.y, tid = threadIdx.x, sub = tid & 3;
    const int32_t g0 = (pos / AP_TOK + (int32_t)blockIdx.x) * AP_TOK;          // first position of the group
    const int32_t lo = max(pos, g0), hi = min(pos + n_rows, g0 + AP_TOK);       // new positions [lo, hi)
    uint8_t *tile = tile_ptr(pr, g0, h);
    if (!tile) {
        if (tid == 0) atomicOr(pr.status, ST_BAD_PAGE);
        return;
    }
    ApIn in;
    ap_load(in, K, V, pos, g0, lo, hi, pr.n_head_kv, h, tid);
#pragma unroll
    for (int it = 0; it < 2; it++) {
        const int p = (tid >> 2) + 64 * it, t = p >> 3, b = p & 7;
#pragma unroll
        for (int kv = 0; kv < 2; kv++) {
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(in.x[it][kv][e]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float d  = div127_rn(amax);
            const float id = d != 0.0f ? rcp_rn(d) : 0.0f;
            uint8_t q[8];
#pragma unroll
            for (int e = 0; e < 8; e++) q[e] = (uint8_t)(int8_t)round_half_away(__fmul_rn(in.x[it][kv][e], id));
            const int dim0 = b * QK + sub * 8;
            *reinterpret_cast<uint2 *>(kv ? &vs[t][dim0] : &ks[t][dim0]) =
                make_uint2(q[0] | q[1] << 8 | q[2] << 16 | (uint32_t)q[3] << 24,
                           q[4] | q[5] << 8 | q[6] << 16 | (uint32_t)q[7] << 24);
            if (sub == 0) {
                if (kv) vd[b][t] = __float2half_rn(d);
                else kd[t][b] = __float2half_rn(d);
            }
        }
    }
    __syncthreads();
    const int tt0 = g0 & 63;   // the group's first token inside the tile
    {   // K: row tid >> 4, chunk tid & 15
        const int t = tid >> 4, c = tid & 15;
        if (g0 + t >= lo && g0 + t < hi)
            *reinterpret_cast<uint4 *>(tile + TILE_KQ + (tt0 + t) * HD + ((c ^ kswz(tt0 + t)) << 4)) =
                *reinterpret_cast<const uint4 *>(&ks[t][c * 16]);
    }
    {   // V: dim tid, the group's 16-token chunk of that dim
        const int dim = tid;
        uint8_t *dst = tile + v_off(dim, tt0);   // 16-byte aligned: tt0 is a multiple of 16
        if (lo == g0 && hi == g0 + AP_TOK) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                w[k] = vs[4 * k][dim] | vs[4 * k + 1][dim] << 8 | vs[4 * k + 2][dim] << 16 | (uint32_t)vs[4 * k + 3][dim] << 24;
            *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
            for (int32_t r = lo; r < hi; r++) dst[r - g0] = vs[r - g0][dim];
        }
    }
    if (tid < AP_TOK) {   // K scales of token tid (16 bytes), V scales of the group per block
        const int t = tid;
        if (g0 + t >= lo && g0 + t < hi)
            *reinterpret_cast<uint4 *>(tile + kd_off(tt0 + t, 0)) = *reinterpret_cast<const uint4 *>(&kd[t][0]);
    } else if (tid < AP_TOK + NBLK) {
        const int b = tid - AP_TOK;
        for (int32_t r = lo; r < hi; r++)
            *reinterpret_cast<__half *>(tile + vd_off(b, tt0 + (r - g0))) = vd[b][r - g0];
    }
}

cudaError_t launch_append(const PoolRef &pr, int32_t pos, const float *K, const float *V, int32_t n_rows,
                          cudaStream_t st) {
    if (n_rows < 1) return cudaSuccess;
    const int32_t groups = (pos + n_rows - 1) / AP_TOK - pos / AP_TOK + 1;
    k_append<<<dim3((unsigned)groups, (unsigned)pr.n_head_kv), 256, 0, st>>>(pr, pos, K, V, n_rows);
    count_launches(1);
    return cudaGetLastError();
}

// ------------------------------------------------------------------- fused projection + append
// The decode-time projections of an attention layer (graph_builder::qsa_dec_qkv,
// src/qwfn_graph.cpp:582-608) ahead of kernel A: for each new token t,
//   Q_h = rope(rms_norm(Wq_h x_t) * q_norm),  K_h = rope(rms_norm(Wk_h x_t) * k_norm),  V_h = Wv_h x_t
// (the reference's rms() and rope(), src/qwfn_graph.cpp:125-132), then K and V quantised to q8_0
// into the page (kernel A's rounding).  One kernel:
//
// k_project_dot: a warp per four rows; lane l reads each row's 16-byte chunks l, l+32, ... (coalesced:
// a warp load covers 512 contiguous bytes; the rows are prefetched into L2 first), and sums
//   lane_l = fmaf(w, x, ...) over its chunks in order, dims in order within a chunk
// (bf16 weights are exact in fp32); y = xor butterfly 16, 8, 4, 2, 1 of the lane sums.  Rows in
// the order: query heads (the query rows of attn_q.weight's per-head query/gate interleave), K
// heads, V heads; a head's 256 rows are the 8 CTAs of one cluster, each keeping its rows' y in
// shared memory.
// Epilogue, run by the first CTA of each head's cluster once it has gathered the head's y through
// distributed shared memory: rms-norm (per warp the xor butterfly of y^2, warp sums added in
// warp order, scale = 1/sqrt(sum/256 + eps), y * scale * w), rope on pairs (i, i + half) of the
// first rope_dim dims with cos/sin from the host (glibc cosf/sinf of angles built by repeated fp32
// multiplication); the query to Q_out, K and V quantised into the page.
// Phase timestamps of k_project_dot, compiled only with -DQKV_TIMELINE (analysis builds; the
// product build never defines it): thread 0 of every CTA notes %globaltimer at its phases.
#ifdef QKV_TIMELINE
__device__ unsigned long long g_ktl_rec[1 << 14][8];
__device__ unsigned int g_ktl_n;
#define KTL_DECL unsigned long long ktl_[6] = {};
#define KTL(i, dep)                                                                              \
    do {                                                                                         \
        if (threadIdx.x == 0) {                                                                  \
            unsigned long long t_;                                                               \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                               \
            ktl_[i] = t_ + ((dep) ? 1 : 0);                                                      \
        }                                                                                        \
    } while (0)
#define KTL_FLUSH()                                                                              \
    do {                                                                                         \
        if (threadIdx.x == 0) {                                                                  \
            const unsigned k_ = atomicAdd(&g_ktl_n, 1u) & 0x3fffu;                               \
            g_ktl_rec[k_][0] = 5;                                                                \
            g_ktl_rec[k_][1] = blockIdx.x;                                                       \
            for (int i_ = 0; i_ < 6; i_++) g_ktl_rec[k_][2 + i_] = ktl_[i_];                     \
        }                                                                                        \
    } while (0)
#else
#define KTL_DECL
#define KTL(i, dep) do { } while (0)
#define KTL_FLUSH() do { } while (0)
#endif

constexpr int PJ_RW = 4;       // rows per warp: each x value read from shared memory serves four rows
constexpr int PJ_DOT_THREADS = 256, PJ_ROWS_CTA = PJ_DOT_THREADS / 32 * PJ_RW;
// Weight chunks stream through a ring of PJ_NS stages in shared memory by per-thread asynchronous
// copies: in stage s, lane l of a warp copies 8-dim chunk 32 s + l of each of its PJ_RW rows (16
// bytes each) into its own slots and later reads exactly those, so no barrier is involved; a
// lane keeps PJ_NS - 1 stages (4 x 16 B each) in flight without holding registers.
constexpr int PJ_NS = 3, PJ_STAGE = PJ_DOT_THREADS * PJ_RW * 16;   // 16 KiB per stage

__device__ __forceinline__ void pj_cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void pj_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void pj_wait_groups() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float warp_sum_bfly(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Head u's kind (0 query, 1 key, 2 value) and index within its kind.
__device__ __forceinline__ int pj_kind(const ProjectParams &p, int u, int &h) {
    const int nq = p.Wq ? p.n_head : 0;
    if (u < nq) { h = u; return 0; }
    if (u < nq + p.n_head_kv) { h = u - nq; return 1; }
    h = u - nq - p.n_head_kv;
    return 2;
}

static_assert(PJ_DOT_THREADS == HD && HD / PJ_ROWS_CTA == 8, "a head is one cluster of 8 CTAs of HD threads");
__global__ void __cluster_dims__(8, 1, 1) __launch_bounds__(PJ_DOT_THREADS, 2) k_project_dot(const ProjectParams p) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, T = p.T;
    const int nq = p.Wq ? p.n_head : 0;
    const int g0 = (blockIdx.x * (PJ_DOT_THREADS / 32) + wid) * PJ_RW;   // this warp's first row (all in one head)
    const uint16_t *W;
    if (g0 < nq * HD) W = p.Wq + ((int64_t)(g0 / HD) * 2 * HD + g0 % HD) * p.n_embd;
    else if (g0 < (nq + p.n_head_kv) * HD) W = p.Wk + (int64_t)(g0 - nq * HD) * p.n_embd;
    else W = p.Wv + (int64_t)(g0 - (nq + p.n_head_kv) * HD) * p.n_embd;
    // dynamic shared memory: x as [2][T][n_embd / 8] float4 (dims 0-3, then dims 4-7 of every
    // 8-dim chunk), then the ring [PJ_NS][warp][row][lane] of 16-byte weight chunks
    extern __shared__ __align__(128) uint8_t pj_dyn[];
    float4 *xs4 = reinterpret_cast<float4 *>(pj_dyn);
    uint4 *ring = reinterpret_cast<uint4 *>(pj_dyn + (size_t)T * p.n_embd * sizeof(float)) + (wid * PJ_RW) * 32 + lane;
    const int nc = p.n_embd / 8, nst = nc / 32;
    const uint4 *w4 = reinterpret_cast<const uint4 *>(W) + lane;   // row r, stage s at w4 + r nc + 32 s
    auto issue = [&](int s) {
        if (s < nst)
#pragma unroll
            for (int r = 0; r < PJ_RW; r++) pj_cp16(ring + (s % PJ_NS) * (PJ_STAGE / 16) + r * 32, w4 + (int64_t)r * nc + 32 * s);
        pj_commit();   // an empty group past the end keeps the group count uniform
    };
    KTL_DECL
    KTL(0, false);
    // the weight copies of the first stages go out first; then the epilogue's inputs (norm
    // weight, block-table entry: nothing waits for them before the epilogue); then x (a
    // thread's loads all in flight before its stores; conflict-free reads: lane stride 16 B), the
    // rest of the warp's rows requested into L2 behind them (one bulk prefetch per row)
#pragma unroll
    for (int s = 0; s < PJ_NS - 1; s++) issue(s);
    // the epilogue's inputs: this CTA's 32 dims of head u are 32 k .. 32 k + 31 (k: its rank in
    // the cluster), a lane's dim is 32 k + lane
    const int u = blockIdx.x * PJ_ROWS_CTA / HD, k8 = blockIdx.x & 7, d = 32 * k8 + lane;
    int h;
    const int kind = pj_kind(p, u, h);
    const float nwt = kind != 2 ? (kind == 0 ? p.q_norm : p.k_norm)[d] : 0.f;
    const int32_t page = kind != 0 && wid < T ? page_of_pos(p.pr, p.pos + wid) : -1;   // warp t: token t
    const float4 *x4 = reinterpret_cast<const float4 *>(p.x);
    {
        constexpr int XU = 8;
        const int nx = T * p.n_embd / 4;
        for (int i0 = tid, first = 1;; i0 += XU * PJ_DOT_THREADS, first = 0) {
            float4 v[XU];
#pragma unroll
            for (int k = 0; k < XU; k++) {
                const int i = i0 + k * PJ_DOT_THREADS;
                if (i < nx) v[k] = x4[i];
            }
            if (first && lane < PJ_RW && nst > PJ_NS - 1)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(W + (int64_t)lane * p.n_embd + (PJ_NS - 1) * 256),
                             "r"((nst - PJ_NS + 1) * 512)
                             : "memory");
#pragma unroll
            for (int k = 0; k < XU; k++) {
                const int i = i0 + k * PJ_DOT_THREADS;
                if (i < nx) xs4[(i & 1) * T * nc + i / 2] = v[k];
            }
            if (i0 + XU * PJ_DOT_THREADS >= nx) break;
        }
    }
    __syncthreads();
    KTL(1, false);
    // lane l takes chunk 32 s + l of its rows in stage s: chunks l, l + 32, ... in order
    float acc[PJ_RW][PJ_MAX_T] = {};
    for (int s = 0; s < nst; s++) {
        issue(s + PJ_NS - 1);          // into the slot this lane finished reading last iteration
        pj_wait_groups<PJ_NS - 1>();   // stage s landed (this lane's own copies)
        const int c = 32 * s + lane;
        uint4 wb[PJ_RW];
#pragma unroll
        for (int r = 0; r < PJ_RW; r++) wb[r] = ring[(s % PJ_NS) * (PJ_STAGE / 16) + r * 32];
#pragma unroll
        for (int t = 0; t < PJ_MAX_T; t++) {
            if (t >= T) break;
            const float4 xa = xs4[t * nc + c], xb = xs4[(T + t) * nc + c];   // one read for the warp's rows
#pragma unroll
            for (int r = 0; r < PJ_RW; r++) {
                const uint32_t wv[4] = {wb[r].x, wb[r].y, wb[r].z, wb[r].w};
                float a = acc[r][t];
                a = __fmaf_rn(__uint_as_float(wv[0] << 16), xa.x, a);
                a = __fmaf_rn(__uint_as_float(wv[0] & 0xffff0000u), xa.y, a);
                a = __fmaf_rn(__uint_as_float(wv[1] << 16), xa.z, a);
                a = __fmaf_rn(__uint_as_float(wv[1] & 0xffff0000u), xa.w, a);
                a = __fmaf_rn(__uint_as_float(wv[2] << 16), xb.x, a);
                a = __fmaf_rn(__uint_as_float(wv[2] & 0xffff0000u), xb.y, a);
                a = __fmaf_rn(__uint_as_float(wv[3] << 16), xb.z, a);
                a = __fmaf_rn(__uint_as_float(wv[3] & 0xffff0000u), xb.w, a);
                acc[r][t] = a;
            }
        }
    }
    pj_wait_groups<0>();   // nothing in flight at exit (the trailing groups are empty)
    KTL(2, acc[0][0] == 12345.0f);
    // A head's 256 rows are the 8 CTAs of one cluster, CTA k holding dims 32 k .. 32 k + 31: one
    // warp butterfly of the rms norm and one q8_0 block.  Warp t runs token t's epilogue for this
    // CTA's dims; the eight sums of squares and rope's partner dims cross the cluster through
    // distributed shared memory.  Each step is the single-head arithmetic of the reference's
    // rms() / rope() and kernel A's rounding, in the same order (the sum of squares: warp
    // butterflies of 32 dims, added in dim order).
    __shared__ float ys[PJ_MAX_T][PJ_ROWS_CTA];   // raw projections of this CTA's dims
    __shared__ float ssq[PJ_MAX_T];               // per token: their sum of squares
    __shared__ float yn[PJ_MAX_T][PJ_ROWS_CTA];   // normalised and weighted
#pragma unroll
    for (int r = 0; r < PJ_RW; r++)
#pragma unroll
        for (int t = 0; t < PJ_MAX_T; t++) {
            if (t >= T) break;
            const float y = warp_sum_bfly(acc[r][t]);
            if (lane == t) ys[t][wid * PJ_RW + r] = y;
        }
    __syncthreads();
    const int t = wid;   // this warp's token (t < T)
    float o = t < T ? ys[t][lane] : 0.f;
    if (t < T && kind != 2) {
        const float s2 = warp_sum_bfly(__fmul_rn(o, o));
        if (lane == 0) ssq[t] = s2;
    }
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();   // every CTA's sums of squares posted
    if (t < T && kind != 2) {
        float sq[HD / 32];
#pragma unroll
        for (int k = 0; k < HD / 32; k++) sq[k] = *cluster.map_shared_rank(&ssq[t], k);
        float sum = sq[0];
#pragma unroll
        for (int k = 1; k < HD / 32; k++) sum = __fadd_rn(sum, sq[k]);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(sum, 1.0f / HD), p.eps)));
        yn[t][lane] = __fmul_rn(__fmul_rn(o, scale), nwt);
    }
    cluster.sync();   // every CTA's normalised dims posted
    KTL(3, false);
    if (t < T) {
        if (kind != 2) {
            const int hh = p.rope_half;
            const float v = yn[t][lane];
            o = v;
            if (d < hh) {
                const float2 c = p.cs[t][d];
                const float w2 = *cluster.map_shared_rank(&yn[t][(d + hh) % 32], (d + hh) / 32);
                o = __fsub_rn(__fmul_rn(v, c.x), __fmul_rn(w2, c.y));
            } else if (d < 2 * hh) {
                const float2 c = p.cs[t][d - hh];
                const float w1 = *cluster.map_shared_rank(&yn[t][(d - hh) % 32], (d - hh) / 32);
                o = __fadd_rn(__fmul_rn(w1, c.y), __fmul_rn(v, c.x));
            }
        }
        if (kind == 0) {
            p.Q_out[((int64_t)t * p.n_head + h) * HD + d] = o;
        } else {
            uint8_t *tile = tile_in_page(p.pr, page, p.pos + t, h);
            int8_t qv;
            __half dh;
            quant_block_warp(o, lane, qv, dh);   // this CTA's dims are q8_0 block k8 of the row
            const int tt = (p.pos + t) & 63;
            if (!tile) {
                if (lane == 0) atomicOr(p.pr.status, ST_BAD_PAGE);
            } else if (kind == 1) {
                tile[k_off(tt, d)] = (uint8_t)qv;
                if (lane == 0) *reinterpret_cast<__half *>(tile + kd_off(tt, k8)) = dh;
            } else {
                tile[v_off(d, tt)] = (uint8_t)qv;
                if (lane == 0) *reinterpret_cast<__half *>(tile + vd_off(k8, tt)) = dh;
            }
        }
    }
    KTL(4, false);
    cluster.sync();   // the partners' reads of this CTA's dims are done before it exits
    KTL_FLUSH();
}

cudaError_t launch_project(const ProjectParams &p, cudaStream_t st) {
    const int units = (p.Wq ? p.n_head : 0) + 2 * p.n_head_kv, n_rows = units * HD;
    const size_t xbytes = (size_t)p.T * p.n_embd * sizeof(float);
    if (xbytes > 48 * 1024 || p.n_embd % 256) return cudaErrorInvalidValue;
    constexpr int SMEM_MAX = 48 * 1024 + PJ_NS * PJ_STAGE;
    const size_t smem = xbytes + PJ_NS * PJ_STAGE;   // staged x, then the ring of weight stages
    // beyond the default 48 KiB window: opt in once per device (up to 96 KiB: two CTAs per SM)
    static uint64_t opted = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(opted >> dev & 1)) {
        if ((e = cudaFuncSetAttribute(k_project_dot, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX)) != cudaSuccess)
            return e;
        opted |= 1ull << dev;
    }
    k_project_dot<<<n_rows / PJ_ROWS_CTA, PJ_DOT_THREADS, smem, st>>>(p);
    count_launches(1);
    return cudaGetLastError();
}

// --------------------------------------------------------------------- ggml-layout transforms
// One warp per (row, head, block): 32 quants + the fp16 scale, moved between the page layout
// and ggml's block_q8_0 rows {fp16 d, int8 qs[32]} (34 bytes, head h at h*272 in a row).
__global__ void __launch_bounds__(256) k_read_rows(PoolRef pr, const int32_t *__restrict__ cells, int32_t pos,
                                                   int32_t n, uint8_t *__restrict__ K_out,
                                                   uint8_t *__restrict__ V_out) {
    const int warp = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int per_row = pr.n_head_kv * NBLK;
    if (warp >= n * per_row) return;
    const int r = warp / per_row, hb = warp % per_row, h = hb / NBLK, b = hb % NBLK;
    const int32_t p = cells ? cells[r] : pos + r;
    const int64_t row_bytes = (int64_t)pr.n_head_kv * ROW_Q8;
    uint8_t *ko = K_out + r * row_bytes + h * ROW_Q8 + b * 34;
    uint8_t *vo = V_out + r * row_bytes + h * ROW_Q8 + b * 34;
    const uint8_t *tile = p >= 0 ? tile_ptr(pr, p, h) : nullptr;
    if (!tile) {
        if (lane == 0) atomicOr(pr.status, p >= 0 ? ST_BAD_PAGE : ST_BAD_INDEX);
        return;
    }
    const int t = p & 63, dim = b * QK + lane;
    ko[2 + lane] = tile[k_off(t, dim)];
    vo[2 + lane] = tile[v_off(dim, t)];
    if (lane < 2) {
        ko[lane] = tile[kd_off(t, b) + lane];
        vo[lane] = tile[vd_off(b, t) + lane];
    }
}

__global__ void __launch_bounds__(256) k_write_rows(PoolRef pr, int32_t pos, int32_t n, const uint8_t *__restrict__ K_in,
                                                    const uint8_t *__restrict__ V_in) {
    const int warp = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int per_row = pr.n_head_kv * NBLK;
    if (warp >= n * per_row) return;
    const int r = warp / per_row, hb = warp % per_row, h = hb / NBLK, b = hb % NBLK;
    const int32_t p = pos + r;
    const int64_t row_bytes = (int64_t)pr.n_head_kv * ROW_Q8;
    const uint8_t *ki = K_in + r * row_bytes + h * ROW_Q8 + b * 34;
    const uint8_t *vi = V_in + r * row_bytes + h * ROW_Q8 + b * 34;
    uint8_t *tile = tile_ptr(pr, p, h);
    if (!tile) {
        if (lane == 0) atomicOr(pr.status, ST_BAD_PAGE);
        return;
    }
    const int t = p & 63, dim = b * QK + lane;
    tile[k_off(t, dim)] = ki[2 + lane];
    tile[v_off(dim, t)] = vi[2 + lane];
    if (lane < 2) {
        tile[kd_off(t, b) + lane] = ki[lane];
        tile[vd_off(b, t) + lane] = vi[lane];
    }
}

cudaError_t launch_read_rows(const PoolRef &pr, const int32_t *cells, int32_t pos, int32_t n, uint8_t *K_out,
                             uint8_t *V_out, cudaStream_t st) {
    const int64_t warps = (int64_t)n * pr.n_head_kv * NBLK;
    k_read_rows<<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>(pr, cells, pos, n, K_out, V_out);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_write_rows(const PoolRef &pr, int32_t pos, int32_t n, const uint8_t *K_in, const uint8_t *V_in,
                              cudaStream_t st) {
    const int64_t warps = (int64_t)n * pr.n_head_kv * NBLK;
    k_write_rows<<<(int)((warps * 32 + 255) / 256), 256, 0, st>>>(pr, pos, n, K_in, V_in);
    count_launches(1);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------ kernel E
// Batched copies (snapshot restore, copy-on-write of shared pages, rollback).  The descriptors
// travel by value; every copy is cut into 64 KiB chunks that a grid sized to the SM count
// walks with 16-byte loads and stores.  (One launch instead of one cudaMemcpyAsync per slot.)
struct CopyBatch {
    int32_t  n;
    int64_t  chunk0[COPY_MAX + 1];
    CopyDesc d[COPY_MAX];
};
constexpr int64_t COPY_CHUNK = 65536;

__global__ void __launch_bounds__(512) k_copy_batch(const CopyBatch cb) {
    const int64_t total = cb.chunk0[cb.n];
    for (int64_t c = blockIdx.x; c < total; c += gridDim.x) {
        int i = 0;
        while (cb.chunk0[i + 1] <= c) i++;
        const int64_t off   = (c - cb.chunk0[i]) * COPY_CHUNK;
        const int64_t bytes = min(COPY_CHUNK, cb.d[i].bytes - off);
        const uint4 *s = reinterpret_cast<const uint4 *>(cb.d[i].src + off);
        uint4 *d       = reinterpret_cast<uint4 *>(cb.d[i].dst + off);
        const int64_t n16 = bytes >> 4;
        for (int64_t k = threadIdx.x; k < n16; k += blockDim.x) d[k] = __ldcs(s + k);
    }
}

cudaError_t launch_copy_batch(const CopyDesc *descs, int n, int num_sms, cudaStream_t st) {
    for (int base = 0; base < n; base += COPY_MAX) {
        CopyBatch cb;
        cb.n = n - base < COPY_MAX ? n - base : COPY_MAX;
        cb.chunk0[0] = 0;
        for (int i = 0; i < cb.n; i++) {
            cb.d[i] = descs[base + i];
            cb.chunk0[i + 1] = cb.chunk0[i] + (cb.d[i].bytes + COPY_CHUNK - 1) / COPY_CHUNK;
        }
        if (cb.chunk0[cb.n] == 0) continue;
        int64_t grid = cb.chunk0[cb.n];
        const int64_t cap = (int64_t)num_sms * 4;
        if (grid > cap) grid = cap;
        k_copy_batch<<<(int)grid, 512, 0, st>>>(cb);
        count_launches(1);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// ------------------------------------------------------------------------------------ kernel B0
// Block summary: summary[h][b][i] = fp16((sum_{t<64} d_t * q_t,i) * (1/64)), the sum in fp32 in
// token order (each d*q is exact in fp32).  One CTA of 256 threads per (block, head), thread i
// owns element i.
__global__ void __launch_bounds__(256) k_block_summary(PoolRef pr, int32_t b0, uint16_t *__restrict__ summary,
                                                       int32_t max_blocks) {
    const int b = b0 + blockIdx.x, h = blockIdx.y, i = threadIdx.x;
    const uint8_t *tile = tile_ptr(pr, b * TILE_TOK, h);
    if (!tile) {
        if (i == 0) atomicOr(pr.status, ST_BAD_PAGE);
        return;
    }
    float acc = 0.0f;
    for (int t = 0; t < TILE_TOK; t++) {
        const float d = __half2float(*reinterpret_cast<const __half *>(tile + kd_off(t, i >> 5)));
        const float q = (float)(int8_t)tile[k_off(t, i)];
        acc = __fadd_rn(acc, __fmul_rn(d, q));
    }
    const __half s = __float2half_rn(__fmul_rn(acc, 1.0f / (float)TILE_TOK));
    summary[((int64_t)h * max_blocks + b) * HD + i] = __half_as_ushort(s);
}

cudaError_t launch_block_summary(const PoolRef &pr, int32_t b0, int32_t b1, uint16_t *summary, int32_t max_blocks,
                                 cudaStream_t st) {
    if (b1 <= b0) return cudaSuccess;
    dim3 grid(b1 - b0, pr.n_head_kv);
    k_block_summary<<<grid, 256, 0, st>>>(pr, b0, summary, max_blocks);
    count_launches(1);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------ kernel B1
// Block scores and top-k, two kernels.
// k_select_score: CTA (sequence x KV head, chunk of p.chunk candidate blocks), 256 threads.
// Groups of 8 lanes compute one dot product in the oracle's fixed order: lane l takes dims
// 32l..32l+31 with sequential fmaf, then a fixed tree over the 8 lanes.  The group's lane 0 sums
// relu(dot) over the G*T query rows in order (t-major), so every score is bit-exact with the CPU
// restatement; four rows' dot products run side by side.  The query rows sit in shared memory as
// 8 segments of 32 dims padded to 36 floats, so the 8 lanes of a group read their segments with
// conflict-free 16-byte loads; the next round's summary bytes are loaded during the current round.
// k_select_rank: CTA (sequence x KV head, 1/p.rk of the candidates): all scores into shared
// memory, then each candidate's rank (score descending, block index ascending) is the number of
// candidates ahead of it, counted by a whole warp.
// Both are latency chains over few blocks: launch_select splits the candidates as finely as keeps
// the grids within about two CTAs per SM (a finer split repeats each CTA's staging: the query rows,
// all scores), so a single sequence's selection runs on most SMs and a wide batch as before.
constexpr int SEL_SEG = 36, SEL_CHUNK_MIN = 16, SEL_CHUNK_MAX = 64, SEL_RK_MIN = 8, SEL_RK_MAX = 144;
__global__ void __launch_bounds__(256) k_select_score(const SelectParams p) {
    extern __shared__ float qs[];                    // [nq][8][SEL_SEG]
    const int sh = blockIdx.x, s = sh / p.n_head_kv, h = sh % p.n_head_kv;
    const int nq = p.T * p.G;
    const int slot = p.seq_slot[s], nb = p.seq_nblk[s];
    const int c0 = blockIdx.y * p.chunk, c1 = min(nb, c0 + p.chunk);
    if (c0 >= nb) return;
    // the group's query rows, float4 loads all issued before the stores (nq * HD / 4 <= 16 per thread)
    {
        constexpr int QV = 16;
        float4 v[QV];
#pragma unroll
        for (int k = 0; k < QV; k++) {
            const int e = threadIdx.x + k * 256;   // float4 index
            if (e < nq * HD / 4) {
                const int n = e / (HD / 4), i = 4 * (e % (HD / 4)), t = n / p.G, j = n % p.G;
                v[k] = *reinterpret_cast<const float4 *>(p.Q + (((int64_t)s * p.T + t) * p.n_head + h * p.G + j) * HD + i);
            }
        }
#pragma unroll
        for (int k = 0; k < QV; k++) {
            const int e = threadIdx.x + k * 256;
            if (e < nq * HD / 4) {
                const int n = e / (HD / 4), i = 4 * (e % (HD / 4));
                *reinterpret_cast<float4 *>(&qs[(n * 8 + (i >> 5)) * SEL_SEG + (i & 31)]) = v[k];
            }
        }
    }
    __syncthreads();
    // Warp-uniform loop: each warp takes 4 blocks per round (one per 8-lane group); every lane
    // runs the shuffles, groups past the end or on a forced block discard their result.
    const int lane8 = threadIdx.x & 7, grp = (threadIdx.x & 31) >> 3;
    const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    const uint16_t *sum_base = p.summary + ((int64_t)slot * p.n_head_kv + h) * p.max_blocks * HD;
    auto load_sum = [&](int bw_, uint4 (&w)[4]) {   // the lane's 64 summary bytes of the group's block
        const int b_ = bw_ + grp;
        const bool live_ = b_ < c1 && !(b_ == 0 || b_ >= nb - 2);
        const uint4 *srow = reinterpret_cast<const uint4 *>(sum_base + (int64_t)(live_ ? b_ : 0) * HD + lane8 * 32);
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = live_ ? srow[k] : make_uint4(0, 0, 0, 0);
    };
    float *scores = p.scores + ((int64_t)s * p.n_head_kv + h) * p.max_blocks;
    uint4 wnext[4];
    if (c0 + warp * 4 < c1) load_sum(c0 + warp * 4, wnext);
    for (int bw = c0 + warp * 4; bw < c1; bw += nwarp * 4) {
        const int b = bw + grp;
        const bool forced = b == 0 || b >= nb - 2;
        uint4 w[4];
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = wnext[k];
        if (bw + nwarp * 4 < c1) load_sum(bw + nwarp * 4, wnext);
        float sv[32];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const __half2 *hh = reinterpret_cast<const __half2 *>(&w[k]);
#pragma unroll
            for (int m = 0; m < 4; m++) {
                const float2 f = __half22float2(hh[m]);
                sv[k * 8 + m * 2]     = f.x;
                sv[k * 8 + m * 2 + 1] = f.y;
            }
        }
        float score = 0.0f;
        for (int n0 = 0; n0 < nq; n0 += 4) {
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int k = 0; k < 8; k++) {
#pragma unroll
                for (int rr = 0; rr < 4; rr++) {
                    const int n = min(n0 + rr, nq - 1);
                    const float4 qk = reinterpret_cast<const float4 *>(qs + (n * 8 + lane8) * SEL_SEG)[k];
                    acc[rr] = __fmaf_rn(qk.x, sv[4 * k], acc[rr]);
                    acc[rr] = __fmaf_rn(qk.y, sv[4 * k + 1], acc[rr]);
                    acc[rr] = __fmaf_rn(qk.z, sv[4 * k + 2], acc[rr]);
                    acc[rr] = __fmaf_rn(qk.w, sv[4 * k + 3], acc[rr]);
                }
            }
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                // fixed tree: ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7))
                float a = acc[rr];
                a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 1));
                a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 2));
                a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
                if (n0 + rr < nq) score = __fadd_rn(score, a > 0.0f ? a : 0.0f);
            }
        }
        if (forced) score = __int_as_float(0x7f800000);
        if (lane8 == 0 && b < c1) scores[b] = score;
    }
}

__global__ void __launch_bounds__(256) k_select_rank(const SelectParams p) {
    extern __shared__ float sc[];                    // [nb] every candidate's score
    const int sh = blockIdx.x, s = sh / p.n_head_kv, h = sh % p.n_head_kv, r = blockIdx.y;
    const int nb = p.seq_nblk[s];
    const int c0 = (int)((int64_t)nb * r / p.rk), c1 = (int)((int64_t)nb * (r + 1) / p.rk);
    int32_t *out = p.idx_out + ((int64_t)s * p.n_head_kv + h) * p.top_k;
    if (nb <= p.top_k) {
        for (int k = c0 + threadIdx.x; k < c1; k += blockDim.x) out[k] = k;
        if (r == p.rk - 1)
            for (int k = nb + threadIdx.x; k < p.top_k; k += blockDim.x) out[k] = -1;
        return;
    }
    const float *scores = p.scores + ((int64_t)s * p.n_head_kv + h) * p.max_blocks;
    for (int i = threadIdx.x; i < nb; i += blockDim.x) sc[i] = scores[i];
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    for (int i = c0 + warp; i < c1; i += nwarp) {
        const float si = sc[i];
        int cnt = 0;
#pragma unroll 8
        for (int j = lane; j < nb; j += 32) {
            const float sj = sc[j];
            cnt += (sj > si) || (sj == si && j < i);
        }
        const int rank = __reduce_add_sync(0xffffffffu, cnt);
        if (lane == 0 && rank < p.top_k) out[rank] = i;
    }
}

cudaError_t launch_select(const SelectParams &p_in, cudaStream_t st) {
    SelectParams p = p_in;
    int max_nb = 1;
    for (int i = 0; i < p.n_seq; i++) max_nb = std::max(max_nb, p.seq_nblk[i]);
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        sms = 148;
    const int64_t heads = (int64_t)p.n_seq * p.n_head_kv, budget = 2 * (int64_t)sms;
    p.chunk = SEL_CHUNK_MIN;
    while (p.chunk < SEL_CHUNK_MAX && heads * ((max_nb + p.chunk - 1) / p.chunk) > budget) p.chunk *= 2;
    p.rk = (int)std::max<int64_t>(SEL_RK_MIN, std::min<int64_t>(SEL_RK_MAX, budget / std::max<int64_t>(heads, 1)));
    const size_t qsm = (size_t)p.T * p.G * 8 * SEL_SEG * sizeof(float), rsm = (size_t)max_nb * sizeof(float);
    cudaError_t e;
    if (qsm > 48 * 1024 && (e = cudaFuncSetAttribute(k_select_score, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qsm)) != cudaSuccess)
        return e;
    if (rsm > 48 * 1024 && (e = cudaFuncSetAttribute(k_select_rank, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm)) != cudaSuccess)
        return e;
    k_select_score<<<dim3((unsigned)(p.n_seq * p.n_head_kv), (unsigned)((max_nb + p.chunk - 1) / p.chunk)), 256, qsm, st>>>(p);
    k_select_rank<<<dim3((unsigned)(p.n_seq * p.n_head_kv), (unsigned)p.rk), 256, rsm, st>>>(p);
    count_launches(2);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------- numerics check
// Every non-negative float against the device's IEEE division and reciprocal (test entry).
__global__ void __launch_bounds__(256) k_check_q8_scale(unsigned long long *bad) {
    unsigned long long nd = 0, nr = 0;
    for (uint64_t u = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; u <= 0x7F800000ull;
         u += (uint64_t)gridDim.x * blockDim.x) {
        const float x = __uint_as_float((uint32_t)u);
        nd += __float_as_uint(div127_rn(x)) != __float_as_uint(__fdiv_rn(x, 127.0f));
        nr += __float_as_uint(rcp_rn(x)) != __float_as_uint(__frcp_rn(x));
    }
    if (nd) atomicAdd(&bad[0], nd);
    if (nr) atomicAdd(&bad[1], nr);
}

}  // namespace qkv

extern "C" qkv_status qkv_debug_check_q8_scale(uint64_t *mismatch_div, uint64_t *mismatch_rcp) {
    if (!mismatch_div || !mismatch_rcp) return QKV_ERR_INVALID;
    unsigned long long *bad = nullptr, host[2] = {0, 0};
    int sms = 0, dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaMalloc(&bad, sizeof host) != cudaSuccess)
        return QKV_ERR_CUDA;
    cudaError_t e = cudaMemset(bad, 0, sizeof host);
    if (e == cudaSuccess) {
        qkv::k_check_q8_scale<<<sms * 8, 256>>>(bad);
        qkv::count_launches(1);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(host, bad, sizeof host, cudaMemcpyDeviceToHost);
    cudaFree(bad);
    if (e != cudaSuccess) return QKV_ERR_CUDA;
    *mismatch_div = host[0];
    *mismatch_rcp = host[1];
    return QKV_OK;
}

#ifdef QKV_TIMELINE
// Analysis builds only: copy out (and reset) the projection kernel's phase records.
extern "C" int qkv_tl_read_k(unsigned long long *host, int max_records) {
    unsigned int n = 0;
    if (cudaMemcpyFromSymbol(&n, qkv::g_ktl_n, sizeof n) != cudaSuccess) return -1;
    const int m = (int)(n < (unsigned)max_records ? n : (unsigned)max_records);
    if (m > 0 && cudaMemcpyFromSymbol(host, qkv::g_ktl_rec, (size_t)m * 8 * 8) != cudaSuccess) return -1;
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(qkv::g_ktl_n, &zero, sizeof zero) != cudaSuccess) return -1;
    return m;
}
#endif
