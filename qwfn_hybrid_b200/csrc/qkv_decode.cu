// qkv_decode.cu -- kernel C: split-K decode / MTP-verify attention over the paged q8_0 cache.
//
// Work plan (host-built, passed by value): pair = (sequence, KV head); each pair owns a run of
// 64-token tiles (dense: tiles 0..ceil(n_kv/64)-1; sparse: the selected block ids).  The runs of
// all pairs are laid end to end and cut into n_ctas equal ranges, one per CTA, so ragged
// batches balance by tiles rather than by sequences.  A CTA whose range holds a pair whole
// writes that pair's output; a pair cut by range boundaries leaves one partial (m, l, acc) per
// CTA and a combine kernel merges them in CTA order (deterministic, no atomics, no waits).
//
// Per pair, the G*T query rows of the KV head's group are quantised to q8_0 exactly as ggml's
// CPU flash_attn_ext quantises its query row, so every QK value is sum_b isum_b * (d_k * d_q)
// with an exact integer block dot.
#include "qkv_internal.h"

#include <cuda_fp16.h>

namespace qkv {

__device__ __forceinline__ int find_pair(const DecodeParams &P, int64_t x) {
    int lo = 0, hi = P.n_pairs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (P.pair_tile0[mid] <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}
__host__ __device__ __forceinline__ int64_t cta_begin(int64_t c, int64_t total, int64_t n_ctas) {
    return c * total / n_ctas;
}
__host__ __device__ __forceinline__ int cta_of(int64_t x, int64_t total, int64_t n_ctas) {
    return (int)(((x + 1) * n_ctas - 1) / total);
}

__device__ __forceinline__ void quant_block(float x, int8_t &q, __half &dh) {
    float amax = fabsf(x);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d  = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
    q  = (int8_t)(int)roundf(__fmul_rn(x, id));
    dh = __float2half_rn(d);
}

// Quantise the pair's query rows into shared memory: qq[n][256] int8, qd[n][8] fp32 (the fp16
// scale widened).  Rows n >= nq are zero.  Called by all threads of the CTA (warp per block).
template <int NQ>
__device__ __forceinline__ void load_query(const DecodeParams &P, int s, int h, int8_t *qq, float *qd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    for (int blk = warp; blk < NQ * NBLK; blk += nwarp) {
        const int n = blk / NBLK, b = blk % NBLK;
        float xv = 0.0f;
        if (n < P.nq) {
            const int t = n / P.G, j = n % P.G;
            xv = P.Q[(((int64_t)s * P.T + t) * P.n_head + h * P.G + j) * HD + b * QK + lane];
        }
        int8_t q;
        __half dh;
        quant_block(xv, q, dh);
        qq[n * HD + b * QK + lane] = q;
        if (lane == 0) qd[n * NBLK + b] = __half2float(dh);
    }
}

// ------------------------------------------------------------------------------ CUDA-core path
template <int NQ>
__global__ void __launch_bounds__(128) k_decode_simple(const DecodeParams P) {
    extern __shared__ __align__(16) uint8_t sm[];
    uint8_t *tile = sm;
    int8_t *qq    = reinterpret_cast<int8_t *>(sm + TILE_BYTES);
    float *qd     = reinterpret_cast<float *>(qq + NQ * HD);
    float *S      = qd + NQ * NBLK;     // [NQ][64]
    float *alpha  = S + NQ * TILE_TOK;  // [NQ]
    float *mrow   = alpha + NQ;
    float *lrow   = mrow + NQ;
    const int tid = threadIdx.x;
    const int c   = blockIdx.x;
    const int64_t a   = cta_begin(c, P.total_tiles, P.n_ctas);
    const int64_t bnd = cta_begin(c + 1, P.total_tiles, P.n_ctas);
    if (a >= bnd) return;
    int p = find_pair(P, a);
    const int p_first = p;
    const int d0 = tid * 2, vb = d0 / QK;
    for (int64_t x = a; x < bnd; p++) {
        const int64_t ps = P.pair_tile0[p], pe = P.pair_tile0[p + 1];
        if (pe <= x) continue;
        const int64_t xe = pe < bnd ? pe : bnd;
        const int s = p / P.n_head_kv, h = p % P.n_head_kv;
        const int slot = P.seq_slot[s], pos0 = P.seq_pos0[s];
        const int n_kv = pos0 + P.T;
        const int32_t *bt = P.block_table + (int64_t)slot * P.max_pages;
        load_query<NQ>(P, s, h, qq, qd);
        if (tid < NQ) {
            mrow[tid] = -INFINITY;
            lrow[tid] = 0.0f;
        }
        float acc[NQ][2];
#pragma unroll
        for (int n = 0; n < NQ; n++) acc[n][0] = acc[n][1] = 0.0f;
        __syncthreads();
        for (int64_t k = x - ps; k < xe - ps; k++) {
            const int blkid = P.sel ? P.sel[((int64_t)s * P.n_head_kv + h) * P.n_sel + k] : (int)k;
            if (blkid < 0) continue;
            const bool in_seq = blkid < (n_kv + TILE_TOK - 1) / TILE_TOK;
            const int32_t page = in_seq ? bt[blkid >> 2] : -1;
            if (page < 0 || page >= P.n_pages) {
                if (tid == 0) atomicOr(P.status, in_seq ? ST_BAD_PAGE : ST_BAD_INDEX);
                continue;
            }
            const uint4 *g = reinterpret_cast<const uint4 *>(
                P.pool + (int64_t)page * P.page_bytes + (int64_t)(h * TILES_PER_PAGE + (blkid & 3)) * TILE_BYTES);
            for (int i = tid; i < TILE_BYTES / 16; i += blockDim.x) reinterpret_cast<uint4 *>(tile)[i] = g[i];
            __syncthreads();
            for (int e = tid; e < NQ * TILE_TOK; e += blockDim.x) {
                const int n = e / TILE_TOK, tok = e % TILE_TOK;
                const int cell = blkid * TILE_TOK + tok;
                float sc = -INFINITY;
                if (n < P.nq && cell <= pos0 + n / P.G) {
                    float sumf = 0.0f;
#pragma unroll
                    for (int b = 0; b < NBLK; b++) {
                        const int4 k0 = *reinterpret_cast<const int4 *>(tile + tok * HD + (((2 * b) ^ kswz(tok)) << 4));
                        const int4 k1 = *reinterpret_cast<const int4 *>(tile + tok * HD + (((2 * b + 1) ^ kswz(tok)) << 4));
                        const int4 q0 = *reinterpret_cast<const int4 *>(qq + n * HD + b * QK);
                        const int4 q1 = *reinterpret_cast<const int4 *>(qq + n * HD + b * QK + 16);
                        int isum = 0;
                        isum = __dp4a(k0.x, q0.x, isum);
                        isum = __dp4a(k0.y, q0.y, isum);
                        isum = __dp4a(k0.z, q0.z, isum);
                        isum = __dp4a(k0.w, q0.w, isum);
                        isum = __dp4a(k1.x, q1.x, isum);
                        isum = __dp4a(k1.y, q1.y, isum);
                        isum = __dp4a(k1.z, q1.z, isum);
                        isum = __dp4a(k1.w, q1.w, isum);
                        const float dk = __half2float(*reinterpret_cast<const __half *>(tile + kd_off(tok, b)));
                        sumf = __fadd_rn(sumf, __fmul_rn((float)isum, __fmul_rn(dk, qd[n * NBLK + b])));
                    }
                    sc = __fmul_rn(sumf, P.scale);
                }
                S[e] = sc;
            }
            __syncthreads();
            if (tid < NQ) {
                float *row = S + tid * TILE_TOK;
                float mt = -INFINITY;
                for (int tok = 0; tok < TILE_TOK; tok++) mt = fmaxf(mt, row[tok]);
                const float mold = mrow[tid], mnew = fmaxf(mold, mt);
                float al = 1.0f, ls = 0.0f;
                if (mnew == -INFINITY) {
                    for (int tok = 0; tok < TILE_TOK; tok++) row[tok] = 0.0f;
                } else {
                    al = expf(mold - mnew);
                    for (int tok = 0; tok < TILE_TOK; tok++) {
                        const float pv = expf(row[tok] - mnew);
                        row[tok] = pv;
                        ls += pv;
                    }
                }
                alpha[tid] = al;
                mrow[tid]  = mnew;
                lrow[tid]  = lrow[tid] * al + ls;
            }
            __syncthreads();
#pragma unroll
            for (int n = 0; n < NQ; n++) {
                acc[n][0] *= alpha[n];
                acc[n][1] *= alpha[n];
            }
            for (int tok = 0; tok < TILE_TOK; tok++) {
                const float dv = __half2float(*reinterpret_cast<const __half *>(tile + vd_off(vb, tok)));
                const float v0 = dv * (float)(int8_t)tile[v_off(d0, tok)];
                const float v1 = dv * (float)(int8_t)tile[v_off(d0 + 1, tok)];
#pragma unroll
                for (int n = 0; n < NQ; n++) {
                    const float pv = S[n * TILE_TOK + tok];
                    acc[n][0] = fmaf(pv, v0, acc[n][0]);
                    acc[n][1] = fmaf(pv, v1, acc[n][1]);
                }
            }
            __syncthreads();
        }
        if (x == ps && xe == pe) {
#pragma unroll
            for (int n = 0; n < NQ; n++) {
                if (n >= P.nq) break;
                const float l = lrow[n], inv = l == 0.0f ? 0.0f : 1.0f / l;
                const int t = n / P.G, j = n % P.G;
                float *o = P.out + (((int64_t)s * P.T + t) * P.n_head + h * P.G + j) * HD + d0;
                *reinterpret_cast<float2 *>(o) = make_float2(acc[n][0] * inv, acc[n][1] * inv);
            }
        } else {
            const int pslot = 2 * c + (p == p_first ? 0 : 1);
            float *rec = P.partial + pslot * partial_stride(P.nq);
#pragma unroll
            for (int n = 0; n < NQ; n++) {
                if (n >= P.nq) break;
                *reinterpret_cast<float2 *>(rec + n * HD + d0) = make_float2(acc[n][0], acc[n][1]);
            }
            if (tid < P.nq) {
                rec[P.nq * HD + tid]        = mrow[tid];
                rec[P.nq * HD + P.nq + tid] = lrow[tid];
            }
        }
        __syncthreads();
        x = xe;
    }
}

// ------------------------------------------------------------------------------------ combine
// One CTA per (pair, query row), one thread per element; partials merged in CTA order.
__global__ void __launch_bounds__(256) k_combine(const DecodeParams P) {
    const int p = blockIdx.x, n = blockIdx.y, d = threadIdx.x;
    const int64_t ps = P.pair_tile0[p], pe = P.pair_tile0[p + 1];
    if (pe <= ps) return;
    const int c_lo = cta_of(ps, P.total_tiles, P.n_ctas), c_hi = cta_of(pe - 1, P.total_tiles, P.n_ctas);
    if (c_lo == c_hi) return;
    const int64_t stride = partial_stride(P.nq);
    float M = -INFINITY;
    for (int c = c_lo; c <= c_hi; c++) {
        const int pslot = 2 * c + (find_pair(P, cta_begin(c, P.total_tiles, P.n_ctas)) == p ? 0 : 1);
        M = fmaxf(M, __ldcg(P.partial + pslot * stride + P.nq * HD + n));
    }
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
        for (int c = c_lo; c <= c_hi; c++) {
            const int pslot = 2 * c + (find_pair(P, cta_begin(c, P.total_tiles, P.n_ctas)) == p ? 0 : 1);
            const float *rec = P.partial + pslot * stride;
            const float m = __ldcg(rec + P.nq * HD + n);
            if (m == -INFINITY) continue;
            const float w = expf(m - M);
            L = fmaf(__ldcg(rec + P.nq * HD + P.nq + n), w, L);
            O = fmaf(__ldcg(rec + n * HD + d), w, O);
        }
    }
    const int s = p / P.n_head_kv, h = p % P.n_head_kv, t = n / P.G, j = n % P.G;
    P.out[(((int64_t)s * P.T + t) * P.n_head + h * P.G + j) * HD + d] = L == 0.0f ? 0.0f : O * (1.0f / L);
}

template <int NQ>
static cudaError_t launch_simple(const DecodeParams &p, cudaStream_t st) {
    const size_t smem = TILE_BYTES + NQ * HD + NQ * NBLK * 4 + NQ * TILE_TOK * 4 + 3 * NQ * 4;
    cudaError_t e = cudaFuncSetAttribute(k_decode_simple<NQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_decode_simple<NQ><<<p.n_ctas, 128, smem, st>>>(p);
    count_launches(1);
    return cudaGetLastError();
}

int decode_max_nq() { return 32; }

cudaError_t launch_decode(const DecodeParams &p, cudaStream_t st) {
    cudaError_t e;
    if (p.nq <= 8) e = launch_simple<8>(p, st);
    else if (p.nq <= 16) e = launch_simple<16>(p, st);
    else if (p.nq <= 24) e = launch_simple<24>(p, st);
    else if (p.nq <= 32) e = launch_simple<32>(p, st);
    else return cudaErrorInvalidValue;
    if (e != cudaSuccess) return e;
    bool split = false;
    for (int q = 0; q < p.n_pairs && !split; q++) {
        const int64_t ps = p.pair_tile0[q], pe = p.pair_tile0[q + 1];
        if (pe > ps) split = cta_of(ps, p.total_tiles, p.n_ctas) != cta_of(pe - 1, p.total_tiles, p.n_ctas);
    }
    if (!split) return cudaSuccess;
    dim3 grid(p.n_pairs, p.nq);
    k_combine<<<grid, 256, 0, st>>>(p);
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace qkv
