/*
 * qkv_oracle.h -- CPU restatement of the reference's q8_0 KV-cache / attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the qwfn_hybrid_b200 package, its
 * libqkv.so, include/qkv.h) may call, link or load this code.  It is the checker that the
 * parity tests, __graft_entry__.smoke() and bench.py's CPU-baseline arm compare against.
 *
 * What it restates (reference = thomaskleiven/QwFN-hybrid, whose arithmetic is ggml/llama.cpp
 * at unslothai/llama.cpp@ca1426903, cloned by scripts/build.sh:8-15 and NOT vendored):
 *
 *   - q8_0 quantisation of F32 rows, as emitted by graph_builder::kv_append
 *     (src/qwfn_graph.cpp:370-384, ggml_cpy F32 -> Q8_0) and qsa_dec_kv_write
 *     (src/qwfn_graph.cpp:612-628, ggml_set_rows).  The published ggml algorithm
 *     (quantize_row_q8_0_ref): d = amax/127 in fp32, id = d ? 1/d : 0, q = roundf(x*id),
 *     d stored as IEEE fp16 (round to nearest even).  Pinned against gguf-py 0.19.0
 *     gguf/quants.py:378-401 (class Q8_0, "bit-exact same results as ... ggml-quants.c").
 *
 *   - flash attention over a q8_0 cache: ggml_flash_attn_ext(q, k, v, mask, scale, 0, 0) with
 *     GGML_PREC_F32 (src/qwfn_graph.cpp:461-471 prefill, 697-699 decode).  Semantics of ggml's
 *     CPU kernel: the query row is converted to K's vec-dot type (q8_0), each KQ value is
 *     sum_b (float)isum_b * (d_k,b * d_q,b), scaled, a -inf mask entry skips the cell, online
 *     softmax in fp32 with expf, V rows dequantised to fp32 and accumulated, result / S
 *     (0 when S == 0).  The cache views follow src/qwfn_graph.cpp:458-464: token-major rows of
 *     n_head_kv*head_dim elements, head h at byte offset h*row_size(head_dim).
 *
 *   - the QSA-style block selection restated for the synthetic sparse config (score blocks
 *     by query . block-summary, ReLU per query head then sum, as the lightning indexer does in
 *     src/qwfn_graph.cpp:340-349 and 560-574; forced blocks as the 1e9 bias of
 *     src/qwfn_engine.cpp:1092-1096; top-k as ggml_top_k, src/qwfn_graph.cpp:575-578).
 *
 * Parity status: the q8_0 quantiser is pinned (golden vectors from gguf-py, tests/golden/).
 * The attention restatement is NOT pinned by any reference output: the reference ships no
 * golden vector for this path and ggml is absent from this machine ("parity unpinned").
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_QK8_0 32            /* elements per q8_0 block */
#define ORC_Q8_0_BYTES 34       /* {fp16 d, int8 qs[32]} */

/* IEEE binary16 <-> binary32, round to nearest even (subnormals kept). */
uint16_t orc_fp32_to_fp16(float f);
float    orc_fp16_to_fp32(uint16_t h);

/* k must be a multiple of 32.  y receives k/32 blocks of 34 bytes (ggml block_q8_0 layout). */
void orc_quantize_row_q8_0(const float *x, uint8_t *y, int64_t k);
void orc_dequantize_row_q8_0(const uint8_t *y, float *x, int64_t k);
/* n_rows independent rows of k elements (OpenMP over rows). */
void orc_quantize_rows_q8_0(const float *x, uint8_t *y, int64_t n_rows, int64_t k, int n_threads);

/*
 * Attention of T query tokens over a q8_0 K/V cache in ggml's token-major layout.
 *   Q        : float [T][n_head][head_dim]
 *   K, V     : n_kv rows of row_bytes = n_head_kv*head_dim/32*34 bytes
 *   cells    : the cache rows to visit, in order (NULL = rows 0..n_cells-1)
 *   q_pos    : [T] position of each query token; cell c is visible to token t iff c <= q_pos[t]
 *              (the causal -inf mask of src/qwfn_engine.cpp:1258-1270 / graph.cpp:671-675)
 *   out      : float [T][n_head][head_dim]
 * GQA: query head h reads KV head h / (n_head / n_head_kv).
 */
void orc_attn_q8_0(const float *Q, int64_t T, int n_head, int n_head_kv, int head_dim,
                   const uint8_t *K, const uint8_t *V,
                   const int32_t *cells, int64_t n_cells,
                   const int32_t *q_pos, float scale, float *out, int n_threads);

/*
 * Per-block key summary of the synthetic sparse config: for KV head h and block b of
 * `block_tokens` consecutive rows, summary[h][b][i] = fp16( (sum_t d*q) * (1/block_tokens) ),
 * the sum taken in fp32 in row order t = 0..block_tokens-1 (each d*q is exact in fp32).
 * Only whole blocks (b < n_blocks) are written.
 */
void orc_block_summary(const uint8_t *K, int n_head_kv, int head_dim, int block_tokens,
                       int64_t n_blocks, uint16_t *summary, int n_threads);

/*
 * Block selection for one decode step of T query tokens:
 *   score[h][b] = +inf                                  for forced blocks (0, nb-2, nb-1)
 *               = sum_{t<T} sum_{j<G} relu(dot(Q[t][h*G+j], summary[h][b]))   otherwise
 * where G = n_head/n_head_kv and dot() is the fixed-order product: eight partial sums over
 * 32 consecutive dims each (fmaf, ascending dim), combined ((p0+p1)+(p2+p3))+((p4+p5)+(p6+p7)).
 * The ReLU'd dots are summed in fp32, t-major then j.  The top_k blocks per KV head are
 * written to idx_out[h][0..top_k) ordered by score descending, ties by block index ascending.
 * When n_blocks <= top_k every block is selected (ascending).  scores_out (nullable) gets
 * [n_head_kv][n_blocks].
 */
void orc_select_blocks(const float *Q, int64_t T, int n_head, int n_head_kv, int head_dim,
                       const uint16_t *summary, int64_t n_blocks, int top_k,
                       int32_t *idx_out, float *scores_out);

/* Expand selected blocks (per KV head) to cell ids: block b -> rows b*bt .. b*bt+bt-1, clipped
 * to n_kv.  Returns the number of cells written to cells_out (capacity top_k*bt). */
int64_t orc_blocks_to_cells(const int32_t *blocks, int top_k, int block_tokens, int64_t n_kv,
                            int32_t *cells_out);

/* Sparse attention for one KV head group: like orc_attn_q8_0 but each KV head h visits its own
 * cell list cells[h][0..n_cells[h]). */
void orc_attn_q8_0_sparse(const float *Q, int64_t T, int n_head, int n_head_kv, int head_dim,
                          const uint8_t *K, const uint8_t *V,
                          const int32_t *const *cells, const int64_t *n_cells,
                          const int32_t *q_pos, float scale, float *out, int n_threads);

/*
 * QSA lightning indexer, decode path (the reference's own selector: src/qwfn_graph.cpp:280-311
 * qsa_pool_blocks / idx_query, 529-579 qsa_dec_index / qsa_dec_cells; bias and bucket
 * src/qwfn_engine.cpp:1072-1105).  Key length 128, 4 cells per block.  Every fp32 step has a
 * fixed order, the one the device kernels use (pooling: lane l of a warp owns dims 4l..4l+3,
 * cross-lane sums are xor butterflies 16,8,4,2,1, emulated here; scores: four quarter sums
 * in dim order), so pooled keys, scores and kept blocks
 * must match the device bit for bit.  ggml's own summation orders differ between its CPU and
 * CUDA backends, so these bits are this build's definition; the semantics are the reference's.
 */
#define ORC_IDX_KEY 128
#define ORC_IDX_R   4

/* cs[b][i] = {cosf(th_i), sinf(th_i)}, th_0 = (float)(4b), th_{i+1} = th_i * powf(base, -2/rope_dim)
 * (ggml's CPU rope cache: one fp32 multiplication per pair), i < rope_dim/2. */
void orc_idx_rope_table(int64_t n_blocks, int rope_dim, float freq_base, float *cs);

/* Pooled key of blocks 0..n_blocks-1 from the raw fp16 keys [4*n_blocks][128]:
 *   x = (((k0 + k1) + k2) + k3) * 0.25;  s = butterfly of ((x0^2 + x1^2) + x2^2) + x3^2 per lane;
 *   y = (x * (1 / sqrtf(s * (1/128) + eps))) * w;
 *   rotate pairs (i, i + rope_dim/2): y_i c - y_j s, y_i s + y_j c;  store fp16 (RNE). */
void orc_idx_pool(const uint16_t *keys, int64_t n_blocks, const float *norm_w, float eps, int rope_dim,
                  const float *cs, uint16_t *pooled);

/* Score of one pooled key: (float) of the double sum over heads of max(0, dot), dot =
 * (s0 + s1) + (s2 + s3), s_j the fp32 sum in dim order over dims 32j..32j+31 of the exact
 * fp16 x fp16 products, q rounded to fp16 first. */
float orc_idx_score(const float *q, int n_head, const uint16_t *pooled_b);

/* Kept blocks for the token at position pos (ascending; returns how many, the rest of
 * blocks_out is -1): every block 0..pos/4 when there are no more than k_blocks, else the
 * incomplete tail block (if pos+1 is not a multiple of 4) and the best remaining whole blocks
 * b < (pos+1)/4 by score (descending, ties by lower index).  scores (nullable) gets the whole
 * blocks' scores. */
int64_t orc_idx_select(const float *q, int n_head, const uint16_t *pooled, int64_t pos, int k_blocks,
                       float *scores, int32_t *blocks_out);

/*
 * Projections of new tokens (graph_builder::qsa_dec_qkv, src/qwfn_graph.cpp:582-608, with the
 * rms() and rope() helpers of src/qwfn_graph.cpp:125-132), in the order the device kernel uses:
 * per output row, 32 lane sums -- lane l takes the 8-dim chunks l, l+32, ... in order, fmaf
 * from 0 -- combined by an xor butterfly 16,8,4,2,1 (lane 0's value); per head rms-norm with the squares summed as 8 warp butterflies
 * added in warp order; y * (1/sqrtf(sum/256 + eps)) * w; NEOX-paired rope of the first rope_dim
 * dims with angles theta_0 = p, theta_{i+1} = theta_i * powf(base, -2/rope_dim).  Weights are
 * bf16 bits; Wq (nullable) holds query and gate rows interleaved per head (attn_q.weight).
 * Outputs F32: Q [T][n_head][256], K and V [T][n_head_kv*256] (K normed and roped).
 */
void orc_project(const float *x, int T, int n_embd, const uint16_t *Wq, const uint16_t *Wk, const uint16_t *Wv,
                 int n_head, int n_head_kv, const float *q_norm, const float *k_norm, float eps, int rope_dim,
                 float freq_base, int pos, float *Q_out, float *K_out, float *V_out);

int orc_max_threads(void);

#ifdef __cplusplus
}
#endif
