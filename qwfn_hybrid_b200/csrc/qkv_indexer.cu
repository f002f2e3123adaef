// qkv_indexer.cu -- the QSA lightning indexer: raw indexer keys and pooled block keys
// (k_idx_append), block scores (k_idx_score), exact top-k per token (k_idx_topk) and the kept-block
// bitsets of the sparse prefill (k_idx_bits).  The decode kernel reads each token's kept blocks in
// place (its QSA mode), so no copy of them is made.
//
// Every floating-point step is written with explicit round-to-nearest operations in a fixed
// order (lane l of a warp owns dims 4l .. 4l+3; cross-lane sums are xor butterflies 16, 8, 4, 2,
// 1), so the CPU oracle (oracle/qkv_oracle.c, orc_idx_*) reproduces the pooled keys, the scores
// and therefore the kept blocks bit for bit.  All of this is HBM / latency bound byte work.
#include "qkv_internal.h"

#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace qkv {

__device__ __forceinline__ float warp_sum_bfly(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ const uint8_t *idx_page(const uint8_t *pool, const int32_t *bt, int32_t max_pages,
                                                   int32_t n_pages, int32_t pos) {
    if (pos < 0 || (pos >> 8) >= max_pages) return nullptr;
    const int32_t page = bt[pos >> 8];
    if (page < 0 || page >= n_pages) return nullptr;
    return pool + (int64_t)page * IDX_PAGE_BYTES;
}

// ------------------------------------------------------------------------------ keys and pooling
// Warps [0, n_rows): store row r's raw key as fp16 (round to nearest even, the F32 -> F16 copy
// of src/qwfn_graph.cpp:330-336).  Warps [n_rows, n_rows + n_blk): pool block b_lo + k, whose
// last cell is in this batch (qsa_pool_blocks, src/qwfn_graph.cpp:280-299):
//   x   = (((k0 + k1) + k2) + k3) * 0.25            k_m = fp16 raw key of cell 4b + m
//   s   = butterfly sum over lanes of ((x0*x0 + x1*x1) + x2*x2) + x3*x3
//   y   = (x * (1 / sqrt(s * (1/128) + eps))) * w
//   rot = y_i*c_i - y_{i+h}*s_i,  y_i*s_i + y_{i+h}*c_i  for i < h = rope_dim/2; other dims y
// and store fp16.  Members before `pos` come from the cache, the others from this batch.
__global__ void __launch_bounds__(256) k_idx_append(const IdxAppendParams p, int32_t b_lo, int32_t n_blk) {
    __shared__ float ybuf[8][IDX_KEY];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int warp = (int)(blockIdx.x * 8 + wid);
    if (warp < p.n_rows) {
        const int32_t c = p.pos + warp;
        uint8_t *pg = const_cast<uint8_t *>(idx_page(p.pool, p.bt, p.max_pages, p.n_pages, c));
        if (!pg) {
            if (lane == 0) atomicOr(p.status, ST_BAD_PAGE);
            return;
        }
        const float4 v = *reinterpret_cast<const float4 *>(p.k_raw + (int64_t)warp * IDX_KEY + 4 * lane);
        __half2 lo = __floats2half2_rn(v.x, v.y), hi = __floats2half2_rn(v.z, v.w);
        uint2 w;
        w.x = *reinterpret_cast<uint32_t *>(&lo);
        w.y = *reinterpret_cast<uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(pg + (int64_t)(c & (PAGE_TOK - 1)) * IDX_KEY * 2 + 8 * lane) = w;
        return;
    }
    const int k = warp - p.n_rows;
    if (k >= n_blk) return;
    const int32_t b = b_lo + k, c0 = b * IDX_R;
    uint8_t *pg = const_cast<uint8_t *>(idx_page(p.pool, p.bt, p.max_pages, p.n_pages, c0));
    if (!pg) {
        if (lane == 0) atomicOr(p.status, ST_BAD_PAGE);
        return;
    }
    float x[4];
#pragma unroll
    for (int m = 0; m < IDX_R; m++) {
        const int32_t c = c0 + m;
        float km[4];
        if (c >= p.pos) {   // this batch: the same fp16 rounding the store applies
            const float4 v = *reinterpret_cast<const float4 *>(p.k_raw + (int64_t)(c - p.pos) * IDX_KEY + 4 * lane);
            km[0] = __half2float(__float2half_rn(v.x));
            km[1] = __half2float(__float2half_rn(v.y));
            km[2] = __half2float(__float2half_rn(v.z));
            km[3] = __half2float(__float2half_rn(v.w));
        } else {
            const uint2 w = *reinterpret_cast<const uint2 *>(pg + (int64_t)(c & (PAGE_TOK - 1)) * IDX_KEY * 2 + 8 * lane);
            const __half2 lo = *reinterpret_cast<const __half2 *>(&w.x), hi = *reinterpret_cast<const __half2 *>(&w.y);
            km[0] = __low2float(lo);
            km[1] = __high2float(lo);
            km[2] = __low2float(hi);
            km[3] = __high2float(hi);
        }
#pragma unroll
        for (int j = 0; j < 4; j++) x[j] = m == 0 ? km[j] : __fadd_rn(x[j], km[j]);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        x[j] = __fmul_rn(x[j], 1.0f / IDX_R);
        s = j == 0 ? __fmul_rn(x[0], x[0]) : __fadd_rn(s, __fmul_rn(x[j], x[j]));
    }
    s = warp_sum_bfly(s);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, 1.0f / IDX_KEY), p.eps)));
#pragma unroll
    for (int j = 0; j < 4; j++) ybuf[wid][4 * lane + j] = __fmul_rn(__fmul_rn(x[j], scale), p.norm_w[4 * lane + j]);
    __syncwarp();
    const int h = p.rope_half;
    const float2 *cs = p.rope + (int64_t)b * h;
    float o[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int d = 4 * lane + j;
        const float y = ybuf[wid][d];
        if (d < h) {
            const float2 t = cs[d];
            o[j] = __fsub_rn(__fmul_rn(y, t.x), __fmul_rn(ybuf[wid][d + h], t.y));
        } else if (d < 2 * h) {
            const float2 t = cs[d - h];
            o[j] = __fadd_rn(__fmul_rn(ybuf[wid][d - h], t.y), __fmul_rn(y, t.x));
        } else {
            o[j] = y;
        }
    }
    __half2 lo = __floats2half2_rn(o[0], o[1]), hi = __floats2half2_rn(o[2], o[3]);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t *>(&lo);
    w.y = *reinterpret_cast<uint32_t *>(&hi);
    *reinterpret_cast<uint2 *>(pg + IDX_RAW_BYTES + (int64_t)(b & (IDX_BPP - 1)) * IDX_KEY * 2 + 8 * lane) = w;
}

cudaError_t launch_idx_append(const IdxAppendParams &p, cudaStream_t st) {
    // blocks whose last cell 4b+3 lies in [pos, pos + n_rows)
    const int32_t b_lo = (p.pos + IDX_R) / IDX_R - 1, b_hi = (p.pos + p.n_rows) / IDX_R;
    const int32_t n_blk = b_hi > b_lo ? b_hi - b_lo : 0;
    const int64_t warps = (int64_t)p.n_rows + n_blk;
    k_idx_append<<<(int)((warps + 7) / 8), 256, 0, st>>>(p, b_lo, n_blk);
    count_launches(1);
    return cudaGetLastError();
}

// Pool blocks b_lo .. b_lo+n_blk-1 from the raw keys already in the pages (a snapshot import).
cudaError_t launch_idx_pool(const IdxAppendParams &p, int32_t b_lo, int32_t n_blk, cudaStream_t st) {
    if (n_blk <= 0) return cudaSuccess;
    IdxAppendParams q = p;
    q.n_rows = 0;
    q.pos = 0x7fffffff;   // every member from the cache
    k_idx_append<<<(n_blk + 7) / 8, 256, 0, st>>>(q, b_lo, n_blk);
    count_launches(1);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------- scores
// score[v][b] = (float)(((0.0 + r_0) + r_1) + ...)  in double over the heads, r_h = max(0, dot_h),
// dot_h = (s_0 + s_1) + (s_2 + s_3), s_j the fp32 sum in dim order over dims 32j .. 32j+31 of
// q_d * k_d, with q = fp16(q_idx) (ggml's F16 mul_mat converts its F32 operand to F16) and k the
// pooled fp16 key: the products of two fp16 values are exact in fp32, so fused multiply-adds round
// as the sums do.  Whole blocks b < (pos+1)/4 only.  Four lanes per block (lane quarter j owns
// s_j; all of its 64 key bytes are loaded up front), 64 blocks per CTA; CTA (x, g) serves the T
// entries g*T .. g*T+T-1 (the tokens of one sequence), which share every pooled-key load.
constexpr int SC_THREADS = 256, SC_BLOCKS = SC_THREADS / 4, SC_PER = 2;   // blocks per thread
constexpr int QROW = IDX_KEY + 16;   // each 32-dim quarter 4 words further on: conflict-free quarter reads
__device__ __forceinline__ int qcol(int d) { return d + 4 * (d >> 5); }

// TT, HH > 0: the token and head counts fixed at compile time (the loops over them have no
// runtime bounds); 0: taken from the parameters.
template <int TT, int HH>
__global__ void __launch_bounds__(SC_THREADS) k_idx_score(const IdxSelectParams p) {
    __shared__ __align__(16) float qs[4][IDX_MAX_HEAD][QROW];
    const int T = TT > 0 ? TT : p.T, H = HH > 0 ? HH : p.n_head, g = blockIdx.y, v0 = g * T;
    // the key loads first: their latency overlaps the query staging.  Thread: quarter j of the
    // dims of SC_PER blocks (SC_BLOCKS apart), so each query read from shared memory serves SC_PER
    // keys; every block's sums run in the same order as for a block alone.
    const int j = threadIdx.x & 3;                                 // quarter of the dims
    const int32_t whole_max = (p.v_pos[v0 + T - 1] + 1) / IDX_R;   // positions ascend with t
    int32_t b[SC_PER];
    const uint8_t *pg[SC_PER];
    uint4 w[SC_PER][4];
#pragma unroll
    for (int k = 0; k < SC_PER; k++) {
        b[k] = blockIdx.x * (SC_PER * SC_BLOCKS) + k * SC_BLOCKS + (threadIdx.x >> 2);
        pg[k] = nullptr;
        if (b[k] < whole_max) {
            pg[k] = idx_page(p.pool, p.bt + (int64_t)p.v_slot[v0] * p.max_pages, p.max_pages, p.n_pages, b[k] * IDX_R);
            if (!pg[k] && j == 0) atomicOr(p.status, ST_BAD_PAGE);
        }
#pragma unroll
        for (int c = 0; c < 4; c++) w[k][c] = make_uint4(0, 0, 0, 0);
        if (pg[k]) {
            const uint4 *key = reinterpret_cast<const uint4 *>(pg[k] + IDX_RAW_BYTES + (int64_t)(b[k] & (IDX_BPP - 1)) * IDX_KEY * 2 + 64 * j);
#pragma unroll
            for (int c = 0; c < 4; c++) w[k][c] = key[c];
        }
    }
    {   // the queries (fp16-rounded): a thread's loads all in flight before its stores
        constexpr int QU = 4 * IDX_MAX_HEAD * IDX_KEY / SC_THREADS;   // the most any thread stages
        const int nq = T * H * IDX_KEY;
        float qv[QU];
#pragma unroll
        for (int k = 0; k < QU; k++) {
            const int i = threadIdx.x + k * SC_THREADS;
            qv[k] = i < nq ? p.q[(int64_t)v0 * H * IDX_KEY + i] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < QU; k++) {
            const int i = threadIdx.x + k * SC_THREADS;
            if (i < nq) {
                const int th = i / IDX_KEY, d = i % IDX_KEY;
                qs[th / H][th % H][qcol(d)] = __half2float(__float2half_rn(qv[k]));
            }
        }
    }
    __syncthreads();
    float acc[SC_PER][4][IDX_MAX_HEAD];
#pragma unroll
    for (int k = 0; k < SC_PER; k++)
#pragma unroll
        for (int t = 0; t < 4; t++)
#pragma unroll
            for (int h = 0; h < IDX_MAX_HEAD; h++) acc[k][t][h] = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        float kv[SC_PER][8];
#pragma unroll
        for (int k = 0; k < SC_PER; k++) {
            const __half2 *hw = reinterpret_cast<const __half2 *>(&w[k][c]);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                kv[k][2 * e] = __low2float(hw[e]);
                kv[k][2 * e + 1] = __high2float(hw[e]);
            }
        }
        const int d0 = 32 * j + 8 * c;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            if (t >= T) break;
#pragma unroll
            for (int h = 0; h < IDX_MAX_HEAD; h++) {
                if (h >= H) break;
                const float4 qa = *reinterpret_cast<const float4 *>(&qs[t][h][qcol(d0)]);
                const float4 qb = *reinterpret_cast<const float4 *>(&qs[t][h][qcol(d0) + 4]);
#pragma unroll
                for (int k = 0; k < SC_PER; k++) {
                    float a = acc[k][t][h];
                    a = __fmaf_rn(qa.x, kv[k][0], a);
                    a = __fmaf_rn(qa.y, kv[k][1], a);
                    a = __fmaf_rn(qa.z, kv[k][2], a);
                    a = __fmaf_rn(qa.w, kv[k][3], a);
                    a = __fmaf_rn(qb.x, kv[k][4], a);
                    a = __fmaf_rn(qb.y, kv[k][5], a);
                    a = __fmaf_rn(qb.z, kv[k][6], a);
                    a = __fmaf_rn(qb.w, kv[k][7], a);
                    acc[k][t][h] = a;
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < SC_PER; k++)
#pragma unroll
        for (int t = 0; t < 4; t++) {
            if (t >= T) break;
            double tot = 0.0;
#pragma unroll
            for (int h = 0; h < IDX_MAX_HEAD; h++) {
                if (h >= H) break;
                float d = __fadd_rn(acc[k][t][h], __shfl_xor_sync(0xffffffffu, acc[k][t][h], 1));   // s0+s1, s2+s3
                d = __fadd_rn(d, __shfl_xor_sync(0xffffffffu, d, 2));                                 // (s0+s1)+(s2+s3)
                tot = __dadd_rn(tot, (double)(d > 0.0f ? d : 0.0f));
            }
            if (pg[k] && j == 0 && b[k] < (p.v_pos[v0 + t] + 1) / IDX_R)
                p.scores[(int64_t)(v0 + t) * p.score_stride + b[k]] = __double2float_rn(tot);
        }
}

// -------------------------------------------------------------------------------------- top-k
// Per entry v (a cluster of TK_CL CTAs): the k_blocks kept blocks in ascending order.  With more
// than k_blocks candidate blocks, the incomplete tail block (if any) is kept and the other
// need = k_blocks - tail come from the whole blocks by score, descending, ties by lower index:
// an exact radix select of the need-th largest key (four 8-bit digits, most significant first)
// gives the threshold; every key above it is kept and, of the keys equal to it, the lowest
// indices.  Keys are the scores' bits mapped so that unsigned order is float order.  CTA r of the
// cluster holds the keys of blocks [r*chunk, (r+1)*chunk) in shared memory; per digit every CTA
// counts its keys, rank 0 sums the TK_CL histograms through distributed shared memory and picks
// the digit; the CTAs' outputs are contiguous runs of the ascending result.
constexpr int TK_CL = 8, TK_THREADS = 256;
constexpr int TK_MAX_CHUNK = 48 * 1024;   // keys per CTA (192 KiB): n_ctx up to 1.5M positions

__device__ __forceinline__ uint32_t score_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// exclusive block-wide prefix sum of one value per thread; returns the thread's prefix, total in *tot
__device__ int block_excl_scan(int x, int *warp_tot, int *tot) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int inc = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) warp_tot[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        const int n = blockDim.x >> 5;
        int t = lane < n ? warp_tot[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        if (lane < n) warp_tot[lane] = t;   // inclusive
    }
    __syncthreads();
    const int base = wid ? warp_tot[wid - 1] : 0;
    const int total = warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();   // warp_tot reusable
    *tot = total;
    return base + inc - x;
}

__global__ void __cluster_dims__(TK_CL, 1, 1) __launch_bounds__(TK_THREADS) k_idx_topk(const IdxSelectParams p) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ uint32_t skeys[];
    __shared__ int hist[2][256];                   // this CTA's counts, two passes alternating
    __shared__ int ctot[256];                      // the cluster's counts
    __shared__ int warp_tot[32];
    __shared__ uint32_t s_prefix;                  // the same in every CTA of the cluster
    __shared__ int s_remaining, s_eq;
    __shared__ int s_cnt[2];                       // this CTA's equal / taken counts
    const int v = blockIdx.y, r = (int)cluster.block_rank(), tid = threadIdx.x, lane = tid & 31;
    const int32_t pos = p.v_pos[v], n_whole = (pos + 1) / IDX_R, b_last = pos / IDX_R;
    const int tail = b_last >= n_whole ? 1 : 0;
    int32_t *out = p.blocks + (int64_t)v * p.k_blocks;
    if (b_last + 1 <= p.k_blocks) {   // every block is kept (uniform over the cluster: no cluster barrier)
        if (r == 0) {
            for (int i = tid; i < p.k_blocks; i += blockDim.x) out[i] = i <= b_last ? i : -1;
            if (tid == 0) p.n_out[v] = b_last + 1;
        }
        return;
    }
    const int need = p.k_blocks - tail;
    const float *sc = p.scores + (int64_t)v * p.score_stride;
    const int chunk = (n_whole + TK_CL - 1) / TK_CL;
    const int k0 = min(n_whole, r * chunk), k1 = min(n_whole, k0 + chunk), nk = k1 - k0;
    for (int i = tid; i < nk; i += blockDim.x) skeys[i] = score_key(sc[k0 + i]);
    uint32_t prefix = 0, mask = 0;
    int remaining = need;
    for (int shift = 24, pass = 0; shift >= 0; shift -= 8, pass++) {
        // histograms alternate between two buffers: the one written now was last read two passes
        // ago, before every CTA reached the previous pass's barrier
        int *h = hist[pass & 1];
        if (tid < 256) h[tid] = 0;
        __syncthreads();
        for (int i = tid; i < nk; i += blockDim.x) {
            const uint32_t key = skeys[i];
            if ((key & mask) == prefix) atomicAdd(&h[(key >> shift) & 0xffu], 1);
        }
        cluster.sync();                            // every CTA's histogram is complete
        if (tid < 256) {                           // every CTA sums all of them and picks the same digit
            int c = 0;
#pragma unroll
            for (int q = 0; q < TK_CL; q++) c += cluster.map_shared_rank(h, q)[tid];
            ctot[tid] = c;
        }
        __syncthreads();
        if (tid < 32) {   // digit of the need-th largest: lane l holds bins 255-8l .. 248-8l
            int bins[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                bins[j] = ctot[255 - 8 * lane - j];
                sum += bins[j];
            }
            int incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const unsigned hit = __ballot_sync(0xffffffffu, incl >= remaining);
            if (lane == __ffs(hit) - 1) {
                int above = incl - sum, j = 0;
#pragma unroll
                for (int jj = 0; jj < 7; jj++) {
                    if (j == jj && above + bins[jj] < remaining) {
                        above += bins[jj];
                        j = jj + 1;
                    }
                }
                int bj = bins[0];
#pragma unroll
                for (int jj = 1; jj < 8; jj++) bj = j == jj ? bins[jj] : bj;
                s_remaining = remaining - above;
                s_prefix = prefix | ((uint32_t)(255 - 8 * lane - j) << shift);
                s_eq = bj;
            }
        }
        __syncthreads();
        prefix = s_prefix;
        remaining = s_remaining;
        mask |= 0xffu << shift;
    }
    const int eq_total = s_eq;
    const bool all_eq = eq_total == remaining;     // no tie at the threshold to break
    // per CTA: keys above the threshold, and (ties) the first `remaining` equal keys by index
    const int per = (nk + blockDim.x - 1) / blockDim.x;
    const int i0 = min(nk, tid * per), i1 = min(nk, i0 + per);
    int tot = 0, eq_base = 0, eq_rank = 0;
    if (!all_eq) {
        int n_eq = 0;
        for (int i = i0; i < i1; i++) n_eq += skeys[i] == prefix;
        eq_rank = block_excl_scan(n_eq, warp_tot, &tot);
        if (tid == 0) s_cnt[0] = tot;
        cluster.sync();                            // equal counts of every CTA published (all_eq is
        for (int q = 0; q < r; q++) eq_base += cluster.map_shared_rank(s_cnt, q)[0];   // cluster-uniform)
    }
    int n_take = 0;
    for (int i = i0, e = eq_base + eq_rank; i < i1; i++) {
        const uint32_t key = skeys[i];
        if (key > prefix) n_take++;
        else if (key == prefix) n_take += all_eq || e++ < remaining;
    }
    int at = block_excl_scan(n_take, warp_tot, &tot);
    if (tid == 0) s_cnt[1] = tot;
    cluster.sync();                                // taken counts of every CTA published
    int base = 0, all = 0;
    for (int q = 0; q < TK_CL; q++) {
        const int c = cluster.map_shared_rank(s_cnt, q)[1];
        if (q < r) base += c;
        all += c;
    }
    at += base;
    for (int i = i0, e = eq_base + eq_rank; i < i1; i++) {
        const uint32_t key = skeys[i];
        bool take = key > prefix;
        if (key == prefix) take = all_eq || e++ < remaining;
        if (take && at < need) out[at++] = k0 + i;
    }
    if (r == 0 && tid == 0) {
        if (all != need) atomicOr(p.status, ST_BAD_INDEX);
        if (tail) out[need] = b_last;
        p.n_out[v] = p.k_blocks;
    }
    cluster.sync();                                // no CTA leaves while its shared memory is read
}

cudaError_t launch_idx_select(const IdxSelectParams &p, int32_t max_whole, cudaStream_t st) {
    static uint64_t attr_set = 0;   // devices whose k_idx_topk allows TK_MAX_CHUNK keys
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!(attr_set >> dev & 1)) {
        e = cudaFuncSetAttribute(k_idx_topk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 TK_MAX_CHUNK * (int)sizeof(uint32_t));
        if (e != cudaSuccess) return e;
        attr_set |= 1ull << dev;
    }
    if (max_whole > 0) {
        const dim3 grid((max_whole + SC_PER * SC_BLOCKS - 1) / (SC_PER * SC_BLOCKS), p.n_v / p.T);
        if (p.n_head == 4 && p.T == 1) k_idx_score<1, 4><<<grid, SC_THREADS, 0, st>>>(p);
        else if (p.n_head == 4 && p.T == 2) k_idx_score<2, 4><<<grid, SC_THREADS, 0, st>>>(p);
        else if (p.n_head == 4 && p.T == 3) k_idx_score<3, 4><<<grid, SC_THREADS, 0, st>>>(p);
        else if (p.n_head == 4 && p.T == 4) k_idx_score<4, 4><<<grid, SC_THREADS, 0, st>>>(p);
        else k_idx_score<0, 0><<<grid, SC_THREADS, 0, st>>>(p);
        count_launches(1);
    }
    const int chunk = (max_whole + TK_CL - 1) / TK_CL;
    if (chunk > TK_MAX_CHUNK) return cudaErrorInvalidValue;
    k_idx_topk<<<dim3(TK_CL, p.n_v), TK_THREADS, (size_t)std::max(chunk, 1) * sizeof(uint32_t), st>>>(p);
    count_launches(1);
    return cudaGetLastError();
}

// ------------------------------------------------------------------------------------ bitsets
// Sparse prefill: the kept blocks of each row v (blocks[v][0 .. n_out[v])) as a bitset of `words`
// words, bit b & 31 of word b >> 5 (kernel D reads word w for KV tile w).
__global__ void __launch_bounds__(256) k_idx_bits(const int32_t *blocks, const int32_t *n_out, int32_t k_blocks,
                                                  uint32_t *bits, int32_t words) {
    extern __shared__ uint32_t row[];
    const int v = blockIdx.x;
    for (int w = threadIdx.x; w < words; w += blockDim.x) row[w] = 0u;
    __syncthreads();
    const int n = min(n_out[v], k_blocks);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int b = blocks[(int64_t)v * k_blocks + i];
        if (b >= 0 && (b >> 5) < words) atomicOr(&row[b >> 5], 1u << (b & 31));
    }
    __syncthreads();
    for (int w = threadIdx.x; w < words; w += blockDim.x) bits[(int64_t)v * words + w] = row[w];
}

cudaError_t launch_idx_bits(const int32_t *blocks, const int32_t *n_out, int32_t k_blocks, int32_t n_v, uint32_t *bits,
                            int32_t words, cudaStream_t st) {
    if (n_v < 1 || words < 1 || (size_t)words * 4 > 48 * 1024) return cudaErrorInvalidValue;
    k_idx_bits<<<n_v, 256, (size_t)words * 4, st>>>(blocks, n_out, k_blocks, bits, words);
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace qkv
