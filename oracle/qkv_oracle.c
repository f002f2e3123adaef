/*
 * qkv_oracle.c -- CPU restatement of the reference's q8_0 KV / attention path.
 * TEST INFRASTRUCTURE ONLY (see qkv_oracle.h): the checker, never the product.
 *
 * Built with -ffp-contract=off so that every product/sum below rounds exactly as written;
 * the places that must be bit-exact (quantiser, block summaries, selection scores) spell out
 * their fused multiply-adds with fmaf().
 */
#include "qkv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------- fp16 ---- */

uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp  = (x >> 23) & 0xffu;
    uint32_t man        = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
    const int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {                         /* fp16 subnormal (or zero) */
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift    = 14 - e;
        uint32_t half      = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t h         = sign | ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;   /* a carry may reach inf: RNE */
    return (uint16_t)h;
}

float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp  = (h >> 10) & 0x1fu;
    const uint32_t man  = h & 0x3ffu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else {
            const float f = ldexpf((float)man, -24);
            return sign ? -f : f;
        }
    } else if (exp == 31) {
        x = sign | 0x7f800000u | (man << 13);
    } else {
        x = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ---------------------------------------------------------------- q8_0 ---- */

/* ggml quantize_row_q8_0_ref restated; the CUDA copy/set_rows quantiser of the same library
 * computes the same d, id and roundf.  gguf-py quants.py:381-393 pins it. */
void orc_quantize_row_q8_0(const float *x, uint8_t *y, int64_t k) {
    const int64_t nb = k / ORC_QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        const float *xb = x + i * ORC_QK8_0;
        uint8_t *yb     = y + i * ORC_Q8_0_BYTES;
        float amax = 0.0f;
        for (int j = 0; j < ORC_QK8_0; j++) {
            const float v = fabsf(xb[j]);
            amax = v > amax ? v : amax;
        }
        const float d  = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t dh = orc_fp32_to_fp16(d);
        yb[0] = (uint8_t)(dh & 0xffu);
        yb[1] = (uint8_t)(dh >> 8);
        for (int j = 0; j < ORC_QK8_0; j++) {
            const float x0 = xb[j] * id;
            yb[2 + j] = (uint8_t)(int8_t)roundf(x0);
        }
    }
}

void orc_dequantize_row_q8_0(const uint8_t *y, float *x, int64_t k) {
    const int64_t nb = k / ORC_QK8_0;
    for (int64_t i = 0; i < nb; i++) {
        const uint8_t *yb = y + i * ORC_Q8_0_BYTES;
        const float d = orc_fp16_to_fp32((uint16_t)(yb[0] | (yb[1] << 8)));
        for (int j = 0; j < ORC_QK8_0; j++) x[i * ORC_QK8_0 + j] = (float)(int8_t)yb[2 + j] * d;
    }
}

void orc_quantize_rows_q8_0(const float *x, uint8_t *y, int64_t n_rows, int64_t k, int n_threads) {
    const int64_t rb = k / ORC_QK8_0 * ORC_Q8_0_BYTES;
#pragma omp parallel for schedule(static) num_threads(n_threads > 0 ? n_threads : 1)
    for (int64_t r = 0; r < n_rows; r++) orc_quantize_row_q8_0(x + r * k, y + r * rb, k);
}

/* ----------------------------------------------------------- attention ---- */

/* ggml_vec_dot_q8_0_q8_0 restated: per block an exact integer dot, then
 * sumf += (float)isum * (d_x * d_y) in block order. */
static float dot_q8_0(const uint8_t *kx, const uint8_t *qy, int n) {
    const int nb = n / ORC_QK8_0;
    float sumf = 0.0f;
    for (int ib = 0; ib < nb; ib++) {
        const uint8_t *a = kx + ib * ORC_Q8_0_BYTES;
        const uint8_t *b = qy + ib * ORC_Q8_0_BYTES;
        int32_t isum = 0;
        for (int j = 0; j < ORC_QK8_0; j++) isum += (int32_t)(int8_t)a[2 + j] * (int32_t)(int8_t)b[2 + j];
        const float da = orc_fp16_to_fp32((uint16_t)(a[0] | (a[1] << 8)));
        const float db = orc_fp16_to_fp32((uint16_t)(b[0] | (b[1] << 8)));
        sumf += (float)isum * (da * db);
    }
    return sumf;
}

/* One query row (token t, head h) against a list of cells: the online-softmax loop of ggml's
 * CPU flash_attn_ext (F32 accumulation, non-F16 V branch). */
static void attn_row(const float *q, int head_dim, const uint8_t *K, const uint8_t *V, int64_t row_bytes,
                     int64_t head_off, const int32_t *cells, int64_t n_cells, int32_t qpos, float scale,
                     float *o, uint8_t *qq, float *v32) {
    orc_quantize_row_q8_0(q, qq, head_dim);
    float S = 0.0f, M = -INFINITY;
    for (int i = 0; i < head_dim; i++) o[i] = 0.0f;
    for (int64_t ic = 0; ic < n_cells; ic++) {
        const int64_t c = cells ? cells[ic] : ic;
        if (c > qpos) continue;                     /* mask == -inf: the cell is skipped */
        float s = dot_q8_0(K + c * row_bytes + head_off, qq, head_dim);
        s = s * scale;
        const float Mold = M;
        float ms = 1.0f, vs = 1.0f;
        if (s > M) {
            M  = s;
            ms = expf(Mold - M);
            for (int i = 0; i < head_dim; i++) o[i] *= ms;
        } else {
            vs = expf(s - M);
        }
        orc_dequantize_row_q8_0(V + c * row_bytes + head_off, v32, head_dim);
        for (int i = 0; i < head_dim; i++) o[i] += v32[i] * vs;
        S = S * ms + vs;
    }
    const float S_inv = S == 0.0f ? 0.0f : 1.0f / S;
    for (int i = 0; i < head_dim; i++) o[i] *= S_inv;
}

void orc_attn_q8_0(const float *Q, int64_t T, int n_head, int n_head_kv, int head_dim,
                   const uint8_t *K, const uint8_t *V, const int32_t *cells, int64_t n_cells,
                   const int32_t *q_pos, float scale, float *out, int n_threads) {
    const int64_t hrow      = (int64_t)head_dim / ORC_QK8_0 * ORC_Q8_0_BYTES;
    const int64_t row_bytes = hrow * n_head_kv;
    const int group         = n_head / n_head_kv;
#pragma omp parallel num_threads(n_threads > 0 ? n_threads : 1)
    {
        uint8_t *qq = (uint8_t *)malloc((size_t)hrow);
        float *v32  = (float *)malloc(sizeof(float) * (size_t)head_dim);
#pragma omp for schedule(dynamic, 1)
        for (int64_t th = 0; th < T * n_head; th++) {
            const int64_t t = th / n_head;
            const int h     = (int)(th % n_head);
            attn_row(Q + th * head_dim, head_dim, K, V, row_bytes, (h / group) * hrow, cells, n_cells,
                     q_pos[t], scale, out + th * head_dim, qq, v32);
        }
        free(qq);
        free(v32);
    }
}

void orc_attn_q8_0_sparse(const float *Q, int64_t T, int n_head, int n_head_kv, int head_dim,
                          const uint8_t *K, const uint8_t *V, const int32_t *const *cells,
                          const int64_t *n_cells, const int32_t *q_pos, float scale, float *out,
                          int n_threads) {
    const int64_t hrow      = (int64_t)head_dim / ORC_QK8_0 * ORC_Q8_0_BYTES;
    const int64_t row_bytes = hrow * n_head_kv;
    const int group         = n_head / n_head_kv;
#pragma omp parallel num_threads(n_threads > 0 ? n_threads : 1)
    {
        uint8_t *qq = (uint8_t *)malloc((size_t)hrow);
        float *v32  = (float *)malloc(sizeof(float) * (size_t)head_dim);
#pragma omp for schedule(dynamic, 1)
        for (int64_t th = 0; th < T * n_head; th++) {
            const int64_t t = th / n_head;
            const int h     = (int)(th % n_head);
            const int kvh   = h / group;
            attn_row(Q + th * head_dim, head_dim, K, V, row_bytes, kvh * hrow, cells[kvh], n_cells[kvh],
                     q_pos[t], scale, out + th * head_dim, qq, v32);
        }
        free(qq);
        free(v32);
    }
}

/* ----------------------------------------------------------- selection ---- */

void orc_block_summary(const uint8_t *K, int n_head_kv, int head_dim, int block_tokens,
                       int64_t n_blocks, uint16_t *summary, int n_threads) {
    const int64_t hrow      = (int64_t)head_dim / ORC_QK8_0 * ORC_Q8_0_BYTES;
    const int64_t row_bytes = hrow * n_head_kv;
    const float inv         = 1.0f / (float)block_tokens;
#pragma omp parallel for schedule(static) num_threads(n_threads > 0 ? n_threads : 1)
    for (int64_t hb = 0; hb < n_head_kv * n_blocks; hb++) {
        const int h     = (int)(hb / n_blocks);
        const int64_t b = hb % n_blocks;
        for (int i = 0; i < head_dim; i++) {
            const int blk = i / ORC_QK8_0, j = i % ORC_QK8_0;
            float acc = 0.0f;
            for (int t = 0; t < block_tokens; t++) {
                const uint8_t *blkp = K + (b * block_tokens + t) * row_bytes + h * hrow + blk * ORC_Q8_0_BYTES;
                const float d = orc_fp16_to_fp32((uint16_t)(blkp[0] | (blkp[1] << 8)));
                acc = acc + d * (float)(int8_t)blkp[2 + j];   /* d*q is exact in fp32 */
            }
            summary[(h * n_blocks + b) * head_dim + i] = orc_fp32_to_fp16(acc * inv);
        }
    }
}

static float fixed_dot(const float *q, const uint16_t *s, int head_dim) {
    /* eight lanes of 32 dims each, then a fixed pairwise tree */
    float p[8];
    const int lanes = head_dim / 32;
    for (int l = 0; l < 8; l++) {
        float acc = 0.0f;
        if (l < lanes)
            for (int i = 0; i < 32; i++) acc = fmaf(q[l * 32 + i], orc_fp16_to_fp32(s[l * 32 + i]), acc);
        p[l] = acc;
    }
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}

typedef struct { float s; int32_t b; } scored_t;

static int cmp_scored(const void *a, const void *b) {
    const scored_t *x = (const scored_t *)a, *y = (const scored_t *)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    return x->b < y->b ? -1 : (x->b > y->b);
}

void orc_select_blocks(const float *Q, int64_t T, int n_head, int n_head_kv, int head_dim,
                       const uint16_t *summary, int64_t n_blocks, int top_k, int32_t *idx_out,
                       float *scores_out) {
    const int group = n_head / n_head_kv;
    scored_t *sc    = (scored_t *)malloc(sizeof(scored_t) * (size_t)(n_blocks > 0 ? n_blocks : 1));
    for (int h = 0; h < n_head_kv; h++) {
        for (int64_t b = 0; b < n_blocks; b++) {
            float score;
            if (b == 0 || b >= n_blocks - 2) {
                score = INFINITY;
            } else {
                const uint16_t *s = summary + (h * n_blocks + b) * head_dim;
                score = 0.0f;
                for (int64_t t = 0; t < T; t++)
                    for (int j = 0; j < group; j++) {
                        const float d = fixed_dot(Q + (t * n_head + h * group + j) * head_dim, s, head_dim);
                        score = score + (d > 0.0f ? d : 0.0f);
                    }
            }
            sc[b].s = score;
            sc[b].b = (int32_t)b;
            if (scores_out) scores_out[h * n_blocks + b] = score;
        }
        if (n_blocks <= top_k) {
            for (int k = 0; k < top_k; k++) idx_out[h * top_k + k] = k < n_blocks ? k : -1;
            continue;
        }
        qsort(sc, (size_t)n_blocks, sizeof(scored_t), cmp_scored);
        for (int k = 0; k < top_k; k++) idx_out[h * top_k + k] = sc[k].b;
    }
    free(sc);
}

int64_t orc_blocks_to_cells(const int32_t *blocks, int top_k, int block_tokens, int64_t n_kv,
                            int32_t *cells_out) {
    int64_t n = 0;
    for (int k = 0; k < top_k; k++) {
        if (blocks[k] < 0) continue;
        for (int t = 0; t < block_tokens; t++) {
            const int64_t c = (int64_t)blocks[k] * block_tokens + t;
            if (c < n_kv) cells_out[n++] = (int32_t)c;
        }
    }
    return n;
}

/* ------------------------------------------------------ QSA lightning indexer ---- */

/* lane-0 value of an xor butterfly sum 16, 8, 4, 2, 1 over 32 lanes */
static float bfly32(const float *v_in) {
    float v[32], t[32];
    memcpy(v, v_in, sizeof v);
    for (int o = 16; o; o >>= 1) {
        for (int l = 0; l < 32; l++) t[l] = v[l] + v[l ^ o];
        memcpy(v, t, sizeof v);
    }
    return v[0];
}

void orc_idx_rope_table(int64_t n_blocks, int rope_dim, float freq_base, float *cs) {
    const int half = rope_dim / 2;
    const float theta_scale = powf(freq_base, -2.0f / (float)(rope_dim > 0 ? rope_dim : 1));
    for (int64_t b = 0; b < n_blocks; b++) {
        float th = (float)(b * ORC_IDX_R);
        for (int i = 0; i < half; i++) {
            cs[(b * half + i) * 2 + 0] = cosf(th);
            cs[(b * half + i) * 2 + 1] = sinf(th);
            th *= theta_scale;
        }
    }
}

void orc_idx_pool(const uint16_t *keys, int64_t n_blocks, const float *norm_w, float eps, int rope_dim,
                  const float *cs, uint16_t *pooled) {
    const int half = rope_dim / 2;
    for (int64_t b = 0; b < n_blocks; b++) {
        float x[ORC_IDX_KEY], y[ORC_IDX_KEY], part[32];
        for (int d = 0; d < ORC_IDX_KEY; d++) {
            float a = orc_fp16_to_fp32(keys[(b * ORC_IDX_R) * ORC_IDX_KEY + d]);
            for (int m = 1; m < ORC_IDX_R; m++) a = a + orc_fp16_to_fp32(keys[(b * ORC_IDX_R + m) * ORC_IDX_KEY + d]);
            x[d] = a * (1.0f / ORC_IDX_R);
        }
        for (int l = 0; l < 32; l++) {
            float s = x[4 * l] * x[4 * l];
            for (int j = 1; j < 4; j++) s = s + x[4 * l + j] * x[4 * l + j];
            part[l] = s;
        }
        const float s = bfly32(part);
        const float scale = 1.0f / sqrtf(s * (1.0f / ORC_IDX_KEY) + eps);
        for (int d = 0; d < ORC_IDX_KEY; d++) y[d] = (x[d] * scale) * norm_w[d];
        for (int d = 0; d < ORC_IDX_KEY; d++) {
            float o = y[d];
            if (d < half) {
                const float c = cs[(b * half + d) * 2], sn = cs[(b * half + d) * 2 + 1];
                o = y[d] * c - y[d + half] * sn;
            } else if (d < 2 * half) {
                const int i = d - half;
                const float c = cs[(b * half + i) * 2], sn = cs[(b * half + i) * 2 + 1];
                o = y[i] * sn + y[d] * c;
            }
            pooled[b * ORC_IDX_KEY + d] = orc_fp32_to_fp16(o);
        }
    }
}

/* the score with q already rounded to fp16 values (qh) */
static float idx_score_rounded(const float *qh, int n_head, const uint16_t *pooled_b) {
    float k[ORC_IDX_KEY];
    for (int d = 0; d < ORC_IDX_KEY; d++) k[d] = orc_fp16_to_fp32(pooled_b[d]);
    double tot = 0.0;
    for (int h = 0; h < n_head; h++) {
        float q4[4];   /* four quarter sums in dim order; products of fp16 values are exact */
        for (int j = 0; j < 4; j++) {
            float a = 0.0f;
            for (int d = 32 * j; d < 32 * j + 32; d++) a = a + qh[h * ORC_IDX_KEY + d] * k[d];
            q4[j] = a;
        }
        const float dot = (q4[0] + q4[1]) + (q4[2] + q4[3]);
        tot = tot + (double)(dot > 0.0f ? dot : 0.0f);
    }
    return (float)tot;
}

float orc_idx_score(const float *q, int n_head, const uint16_t *pooled_b) {
    float qh[8 * ORC_IDX_KEY];
    for (int i = 0; i < n_head * ORC_IDX_KEY && i < 8 * ORC_IDX_KEY; i++) qh[i] = orc_fp16_to_fp32(orc_fp32_to_fp16(q[i]));
    return idx_score_rounded(qh, n_head < 8 ? n_head : 8, pooled_b);
}

typedef struct { float s; int32_t b; } idx_scored_t;

static int cmp_idx_scored(const void *a, const void *b) {
    const idx_scored_t *x = (const idx_scored_t *)a, *y = (const idx_scored_t *)b;
    if (x->s != y->s) return x->s > y->s ? -1 : 1;
    return (x->b > y->b) - (x->b < y->b);
}

static int cmp_i32(const void *a, const void *b) {
    const int32_t x = *(const int32_t *)a, y = *(const int32_t *)b;
    return (x > y) - (x < y);
}

int64_t orc_idx_select(const float *q, int n_head, const uint16_t *pooled, int64_t pos, int k_blocks,
                       float *scores, int32_t *blocks_out) {
    const int64_t whole = (pos + 1) / ORC_IDX_R, b_last = pos / ORC_IDX_R;
    const int tail = b_last >= whole;
    for (int k = 0; k < k_blocks; k++) blocks_out[k] = -1;
    idx_scored_t *sc = (idx_scored_t *)malloc(sizeof(idx_scored_t) * (size_t)(whole > 0 ? whole : 1));
    float qh[8 * ORC_IDX_KEY];
    const int nh = n_head < 8 ? n_head : 8;
    for (int i = 0; i < nh * ORC_IDX_KEY; i++) qh[i] = orc_fp16_to_fp32(orc_fp32_to_fp16(q[i]));
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < whole; b++) {
        sc[b].s = idx_score_rounded(qh, nh, pooled + b * ORC_IDX_KEY);
        sc[b].b = (int32_t)b;
        if (scores) scores[b] = sc[b].s;
    }
    int64_t n;
    if (b_last + 1 <= k_blocks) {
        for (int64_t b = 0; b <= b_last; b++) blocks_out[b] = (int32_t)b;
        n = b_last + 1;
    } else {
        const int need = k_blocks - tail;
        qsort(sc, (size_t)whole, sizeof(idx_scored_t), cmp_idx_scored);
        for (int k = 0; k < need; k++) blocks_out[k] = sc[k].b;
        qsort(blocks_out, (size_t)need, sizeof(int32_t), cmp_i32);
        if (tail) blocks_out[need] = (int32_t)b_last;
        n = k_blocks;
    }
    free(sc);
    return n;
}

/* ------------------------------------------------------------ projections ---- */

static float bf16f(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* one head of 256 rows for T tokens: raw projection, then (kind < 2) norm + rope */
static void project_head(const float *x, int T, int n_embd, const uint16_t *W, int64_t row0, int kind,
                         const float *nw, float eps, int rope_dim, const float *cs, float *out, int64_t out_stride) {
    const int HDIM = 256;
    float y[4][256];
    for (int t = 0; t < T; t++)
        for (int r = 0; r < HDIM; r++) {
            const uint16_t *w = W + (row0 + r) * (int64_t)n_embd;
            float lanes[32];   /* lane l: chunks l, l+32, ... of 8 dims, in order */
            for (int l = 0; l < 32; l++) {
                float a = 0.0f;
                for (int c = l; c < n_embd / 8; c += 32)
                    for (int e = 0; e < 8; e++) a = fmaf(bf16f(w[8 * c + e]), x[(int64_t)t * n_embd + 8 * c + e], a);
                lanes[l] = a;
            }
            y[t][r] = bfly32(lanes);
        }
    const int half = rope_dim / 2;
    for (int t = 0; t < T; t++) {
        float o[256];
        if (kind == 2) {
            memcpy(o, y[t], sizeof o);
        } else {
            float ws[8];
            for (int w = 0; w < 8; w++) {
                float sq[32];
                for (int l = 0; l < 32; l++) sq[l] = y[t][32 * w + l] * y[t][32 * w + l];
                ws[w] = bfly32(sq);
            }
            float s = ws[0];
            for (int w = 1; w < 8; w++) s = s + ws[w];
            const float scale = 1.0f / sqrtf(s * (1.0f / 256) + eps);
            float yb[256];
            for (int r = 0; r < HDIM; r++) yb[r] = (y[t][r] * scale) * nw[r];
            for (int r = 0; r < HDIM; r++) {
                o[r] = yb[r];
                if (r < half) {
                    const float c = cs[(t * half + r) * 2], sn = cs[(t * half + r) * 2 + 1];
                    o[r] = yb[r] * c - yb[r + half] * sn;
                } else if (r < 2 * half) {
                    const int i = r - half;
                    const float c = cs[(t * half + i) * 2], sn = cs[(t * half + i) * 2 + 1];
                    o[r] = yb[i] * sn + yb[r] * c;
                }
            }
        }
        memcpy(out + t * out_stride, o, sizeof o);
    }
}

void orc_project(const float *x, int T, int n_embd, const uint16_t *Wq, const uint16_t *Wk, const uint16_t *Wv,
                 int n_head, int n_head_kv, const float *q_norm, const float *k_norm, float eps, int rope_dim,
                 float freq_base, int pos, float *Q_out, float *K_out, float *V_out) {
    const int half = rope_dim / 2;
    float *cs = (float *)malloc(sizeof(float) * 2 * (size_t)(T * (half > 0 ? half : 1)));
    const float theta_scale = powf(freq_base, -2.0f / (float)(rope_dim > 0 ? rope_dim : 1));
    for (int t = 0; t < T; t++) {
        float th = (float)(pos + t);
        for (int i = 0; i < half; i++) {
            cs[(t * half + i) * 2] = cosf(th);
            cs[(t * half + i) * 2 + 1] = sinf(th);
            th *= theta_scale;
        }
    }
    const int kvd = n_head_kv * 256;
#pragma omp parallel for schedule(dynamic)
    for (int u = 0; u < (Wq ? n_head : 0) + 2 * n_head_kv; u++) {
        const int nq = Wq ? n_head : 0;
        if (u < nq)
            project_head(x, T, n_embd, Wq, (int64_t)u * 512, 0, q_norm, eps, rope_dim, cs, Q_out + u * 256,
                         (int64_t)n_head * 256);
        else if (u < nq + n_head_kv)
            project_head(x, T, n_embd, Wk, (int64_t)(u - nq) * 256, 1, k_norm, eps, rope_dim, cs,
                         K_out + (u - nq) * 256, kvd);
        else
            project_head(x, T, n_embd, Wv, (int64_t)(u - nq - n_head_kv) * 256, 2, NULL, eps, rope_dim, cs,
                         V_out + (u - nq - n_head_kv) * 256, kvd);
    }
    free(cs);
}

