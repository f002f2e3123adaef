// qkv_indexer.cu -- the QSA lightning indexer, decode path: raw indexer keys and pooled block
// keys (k_idx_append), block scores (k_idx_score), exact top-k per token (k_idx_topk), and the
// gather of each token's kept cells into scratch pages that the decode kernel reads as a dense
// sequence (k_idx_gather).
//
// Every floating-point step is written with explicit round-to-nearest operations in a fixed
// order (lane l of a warp owns dims 4l .. 4l+3; cross-lane sums are xor butterflies 16, 8, 4, 2,
// 1), so the CPU oracle (oracle/qkv_oracle.c, orc_idx_*) reproduces the pooled keys, the scores
// and therefore the kept blocks bit for bit.  All of this is HBM / latency bound byte work.
#include "qkv_internal.h"

#include <cuda_fp16.h>

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
// score[v][b] = (float)(((0.0 + r_0) + r_1) + ... )  in double, r_h = max(0, dot_h), dot_h the
// butterfly sum over lanes of ((q0*k0 + q1*k1) + q2*k2) + q3*k3 with q = fp16(q_idx) (ggml's
// F16 mul_mat converts its F32 operand to F16) and k the pooled fp16 key; the products of two
// fp16 values are exact in fp32.  Whole blocks b < (pos+1)/4 only.
__global__ void __launch_bounds__(256) k_idx_score(const IdxSelectParams p) {
    __shared__ float qs[IDX_MAX_HEAD][IDX_KEY];
    const int v = blockIdx.y;
    const int32_t pos = p.v_pos[v], n_whole = (pos + 1) / IDX_R;
    for (int i = threadIdx.x; i < p.n_head * IDX_KEY; i += blockDim.x)
        qs[i / IDX_KEY][i % IDX_KEY] = __half2float(__float2half_rn(p.q[(int64_t)v * p.n_head * IDX_KEY + i]));
    __syncthreads();
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *bt = p.bt + (int64_t)p.v_slot[v] * p.max_pages;
    for (int k = 0; k < 4; k++) {
        const int32_t b = (blockIdx.x * 8 + wid) * 4 + k;
        if (b >= n_whole) return;
        const uint8_t *pg = idx_page(p.pool, bt, p.max_pages, p.n_pages, b * IDX_R);
        if (!pg) {
            if (lane == 0) atomicOr(p.status, ST_BAD_PAGE);
            return;
        }
        const uint2 w = *reinterpret_cast<const uint2 *>(pg + IDX_RAW_BYTES + (int64_t)(b & (IDX_BPP - 1)) * IDX_KEY * 2 +
                                                         8 * lane);
        const __half2 lo = *reinterpret_cast<const __half2 *>(&w.x), hi = *reinterpret_cast<const __half2 *>(&w.y);
        const float kk[4] = {__low2float(lo), __high2float(lo), __low2float(hi), __high2float(hi)};
        double tot = 0.0;
        for (int h = 0; h < p.n_head; h++) {
            const float *q = &qs[h][4 * lane];
            float a = __fmul_rn(q[0], kk[0]);
            a = __fadd_rn(a, __fmul_rn(q[1], kk[1]));
            a = __fadd_rn(a, __fmul_rn(q[2], kk[2]));
            a = __fadd_rn(a, __fmul_rn(q[3], kk[3]));
            a = warp_sum_bfly(a);
            tot = __dadd_rn(tot, (double)(a > 0.0f ? a : 0.0f));
        }
        if (lane == 0) p.scores[(int64_t)v * p.score_stride + b] = __double2float_rn(tot);
    }
}

// -------------------------------------------------------------------------------------- top-k
// Per entry v (one CTA of 1024 threads): the k_blocks kept blocks in ascending order.  With more
// than k_blocks candidate blocks, the incomplete tail block (if any) is kept and the other
// need = k_blocks - tail come from the whole blocks by score, descending, ties by lower index:
// an exact radix select of the need-th largest key (four 8-bit digits, most significant first)
// gives the threshold; every key above it is kept and, of the keys equal to it, the lowest
// indices.  Keys are the scores' bits mapped so that unsigned order is float order.
constexpr int TK_THREADS = 1024;

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

__global__ void __launch_bounds__(TK_THREADS) k_idx_topk(const IdxSelectParams p) {
    __shared__ int hist[256];
    __shared__ int warp_tot[32];
    __shared__ uint32_t s_prefix;
    __shared__ int s_remaining;
    const int v = blockIdx.x, tid = threadIdx.x;
    const int32_t pos = p.v_pos[v], n_whole = (pos + 1) / IDX_R, b_last = pos / IDX_R;
    const int tail = b_last >= n_whole ? 1 : 0;
    int32_t *out = p.blocks + (int64_t)v * p.k_blocks;
    if (b_last + 1 <= p.k_blocks) {   // every block is kept
        for (int i = tid; i < p.k_blocks; i += blockDim.x) out[i] = i <= b_last ? i : -1;
        if (tid == 0) p.n_out[v] = b_last + 1;
        return;
    }
    const int need = p.k_blocks - tail;
    const float *sc = p.scores + (int64_t)v * p.score_stride;
    uint32_t prefix = 0, mask = 0;
    int remaining = need;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < n_whole; i += blockDim.x) {
            const uint32_t key = score_key(sc[i]);
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xff], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int above = 0, d = 255;
            for (; d > 0; d--) {
                if (above + hist[d] >= remaining) break;
                above += hist[d];
            }
            s_remaining = remaining - above;
            s_prefix = prefix | ((uint32_t)d << shift);
        }
        __syncthreads();
        remaining = s_remaining;
        prefix = s_prefix;
        mask |= 0xffu << shift;
        __syncthreads();
    }
    // prefix: the threshold key; keep every key above it and the first `remaining` equal to it
    const int chunk = (n_whole + blockDim.x - 1) / blockDim.x;
    const int i0 = min(n_whole, tid * chunk), i1 = min(n_whole, i0 + chunk);
    int n_eq = 0;
    for (int i = i0; i < i1; i++) n_eq += score_key(sc[i]) == prefix;
    int tot;
    int eq_rank = block_excl_scan(n_eq, warp_tot, &tot);
    int n_take = 0;
    for (int i = i0, r = eq_rank; i < i1; i++) {
        const uint32_t key = score_key(sc[i]);
        if (key > prefix) n_take++;
        else if (key == prefix) n_take += r++ < remaining;
    }
    int at = block_excl_scan(n_take, warp_tot, &tot);
    for (int i = i0, r = eq_rank; i < i1; i++) {
        const uint32_t key = score_key(sc[i]);
        bool take = key > prefix;
        if (key == prefix) take = r++ < remaining;
        if (take && at < need) out[at++] = i;
    }
    if (tid == 0) {
        if (tot != need) atomicOr(p.status, ST_BAD_INDEX);
        if (tail) out[need] = b_last;
        p.n_out[v] = p.k_blocks;
    }
}

cudaError_t launch_idx_select(const IdxSelectParams &p, int32_t max_whole, cudaStream_t st) {
    if (max_whole > 0) {
        k_idx_score<<<dim3((max_whole + 31) / 32, p.n_v), 256, 0, st>>>(p);
        count_launches(1);
    }
    k_idx_topk<<<p.n_v, TK_THREADS, 0, st>>>(p);
    count_launches(1);
    return cudaGetLastError();
}

// --------------------------------------------------------------------------------------- gather
// CTA (i, v), warp h: kept block i of entry v, KV head h.  Its 4 cells c0 .. c0+3 (c0 = 4 b) go to
// cells 4i .. 4i+3 of the entry's scratch sequence; cells past v_pos are written as zeros.  Per
// 4-cell group and head: 4 K rows (64 chunks of 16 B, re-swizzled), one 4-byte word per dim of
// the transposed V, 64 B of K scales and 8 x 8 B of V scales.
__global__ void __launch_bounds__(256) k_idx_gather(const IdxGatherParams p) {
    const int v = blockIdx.y, i = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (h >= p.n_head_kv || i >= p.n_out[v]) return;
    const int32_t b = p.blocks[(int64_t)v * p.k_blocks + i], pos = p.v_pos[v], c0 = b * IDX_R;
    if (b < 0 || c0 > pos) {
        if (lane == 0) atomicOr(p.status, ST_BAD_INDEX);
        return;
    }
    const int32_t *bt = p.bt + (int64_t)p.v_slot[v] * p.max_pages;
    const int32_t sp = (c0 >> 8) < p.max_pages ? bt[c0 >> 8] : -1;
    const int32_t j0 = i * IDX_R;
    const int32_t dp = (j0 >> 8) < p.dst_pages ? p.dst_bt[(int64_t)v * p.dst_pages + (j0 >> 8)] : -1;
    if (sp < 0 || sp >= p.n_pages || dp < 0) {
        if (lane == 0) atomicOr(p.status, ST_BAD_PAGE);
        return;
    }
    const uint8_t *src = p.pool + (int64_t)sp * p.page_bytes + (int64_t)(h * TILES_PER_PAGE + ((c0 >> 6) & 3)) * TILE_BYTES;
    uint8_t *dst = p.dst + (int64_t)dp * p.page_bytes + (int64_t)(h * TILES_PER_PAGE + ((j0 >> 6) & 3)) * TILE_BYTES;
    const int ts = c0 & 63, td = j0 & 63;
    const int nv = min(IDX_R, pos - c0 + 1);   // valid cells of the group
#pragma unroll
    for (int k = 0; k < 2; k++) {              // K quants
        const int q = lane + 32 * k, m = q >> 4, c = q & 15;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (m < nv) val = *reinterpret_cast<const uint4 *>(src + TILE_KQ + (ts + m) * HD + ((c ^ kswz(ts + m)) << 4));
        *reinterpret_cast<uint4 *>(dst + TILE_KQ + (td + m) * HD + ((c ^ kswz(td + m)) << 4)) = val;
    }
    const uint32_t vmask = nv >= 4 ? 0xffffffffu : ((1u << (8 * nv)) - 1u);
#pragma unroll
    for (int k = 0; k < HD / 32; k++) {        // V quants: 4 tokens of one dim are one word
        const int dim = lane + 32 * k;
        const uint32_t w = *reinterpret_cast<const uint32_t *>(src + v_off(dim, ts));
        *reinterpret_cast<uint32_t *>(dst + v_off(dim, td)) = w & vmask;
    }
    if (lane < 16) {                            // K scales: [tok][8] fp16, 16 B per token
        const int m = lane >> 2;
        const uint32_t w = m < nv ? *reinterpret_cast<const uint32_t *>(src + kd_off(ts, 0) + 4 * lane) : 0u;
        *reinterpret_cast<uint32_t *>(dst + kd_off(td, 0) + 4 * lane) = w;
    } else if (lane < 16 + NBLK) {              // V scales: [8][tok] fp16, 4 tokens = 8 B per block
        const int blk = lane - 16;
        uint2 w = *reinterpret_cast<const uint2 *>(src + vd_off(blk, ts));
        if (nv < 4) {
            const uint32_t lo = nv >= 2 ? 0xffffffffu : (nv >= 1 ? 0x0000ffffu : 0u);
            const uint32_t hi = nv >= 4 ? 0xffffffffu : (nv >= 3 ? 0x0000ffffu : 0u);
            w.x &= lo;
            w.y &= hi;
        }
        *reinterpret_cast<uint2 *>(dst + vd_off(blk, td)) = w;
    }
}

cudaError_t launch_idx_gather(const IdxGatherParams &p, cudaStream_t st) {
    k_idx_gather<<<dim3(p.k_blocks, p.n_v), 32 * p.n_head_kv, 0, st>>>(p);
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace qkv
