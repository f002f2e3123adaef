/*
 * qkv.h -- C ABI of the B200-native q8_0 KV-cache and attention engine.
 *
 * This is the drop-in boundary for the full-attention path of QwFN-hybrid
 * (thomaskleiven/QwFN-hybrid).  The reference reaches that path through C++ objects typed with
 * ggml (qwfn::state, engine::snapshot_*, and the ggml_flash_attn_ext / ggml_cpy / ggml_set_rows
 * nodes its graph builder emits).  ggml is not linked here, so every entry point below takes
 * plain pointers and sizes instead; each one names the reference interface it replaces.
 *
 * Conventions (the reference's, carried over -- src/qwfn_check.h:21-27, src/qwfn_engine.cpp:
 * 1023-1041):
 *   - every call returns a qkv_status and never aborts; qkv_last_error() explains the failure;
 *   - a recoverable failure leaves the engine as it was (no partial page allocation, an empty
 *     snapshot handle);
 *   - device work is stream-ordered on the cudaStream_t passed as `stream` (NULL = legacy
 *     default stream); pointers called "device" must be device memory of the engine's GPU;
 *   - one engine per GPU, driven by one host thread at a time (the reference serialises its
 *     single engine behind a mutex, tools/qwfn_server.cpp:1-12).
 *
 * Cache layout.  Positions are grouped in 256-token pages drawn from a pool shared by all
 * sequence slots; a per-slot block table maps page index -> page id, and page ids are shared by
 * all attention layers (each layer has its own pool).  Within a page, each KV head holds four
 * 64-token tiles of q8_0 data: int8 quantised K rows, int8 quantised V stored transposed, and
 * the fp16 block scales.  The quantised values are exactly ggml's q8_0 blocks; qkv_read_rows()
 * and qkv_gather_rows() return them in ggml's token-major block_q8_0 layout.
 */
#ifndef QKV_H
#define QKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum qkv_status {
    QKV_OK              = 0,
    QKV_ERR_INVALID     = 1,  /* bad argument: null pointer, layer/slot/size out of range      */
    QKV_ERR_NO_MEMORY   = 2,  /* device memory or page pool exhausted                           */
    QKV_ERR_CUDA        = 3,  /* a CUDA runtime call failed                                     */
    QKV_ERR_STATE       = 4,  /* not valid now: slot inactive, context exhausted, no snapshot   */
    QKV_ERR_MISMATCH    = 5,  /* snapshot / blob does not fit this engine                       */
    QKV_ERR_DEVICE      = 6,  /* a kernel reported a bounds violation or a wait that gave up    */
    QKV_ERR_UNSUPPORTED = 7   /* shape or mode this build does not provide (host-only engine)   */
} qkv_status;

typedef struct qkv_engine qkv_engine;
typedef struct qkv_snapshot qkv_snapshot;

/* Shapes.  Replaces qwfn::state_config + the attention fields of qwfn::hparams
 * (src/qwfn_state.h:28-37, src/qwfn_hparams.h:20-31, 44-48). */
typedef struct qkv_config {
    int32_t n_layer;        /* attention layers held by the engine (12)                          */
    int32_t n_head;         /* query heads (16 in the configs, 24 in the model)                  */
    int32_t n_head_kv;      /* KV heads (2)                                                      */
    int32_t head_dim;       /* 256 (the only value this build provides)                          */
    int32_t n_ctx;          /* positions per sequence                                            */
    int32_t n_slots;        /* sequence slots                                                    */
    int32_t n_pages;        /* 256-token pages in the pool; 0 = n_slots * ceil(n_ctx / 256)      */
    int32_t rec_n_layer;    /* recurrent (DeltaNet) layers whose state rides in snapshots (36)   */
    int32_t rec_head_dim;   /* DeltaNet state is [rec_head_dim, rec_head_dim, rec_n_head] F32    */
    int32_t rec_n_head;     /* value heads (48 in the model, 32 in the synthetic config)         */
    int32_t conv_channels;  /* conv state is [conv_hist, conv_channels] F32                      */
    int32_t conv_hist;      /* d_conv - 1 (3)                                                    */
    int32_t n_rollback;     /* rollback snapshots of the recurrent state kept per slot (0..4)    */
    int32_t select_block;   /* tokens per selection block (64), 0 = no block summaries           */
    int32_t attn_interval;  /* host-blob layer order: absolute layer il is attention iff           *
                             * (il+1) % attn_interval == 0 (hparams::is_attn_layer, 4 in the model; *
                             * needs n_layer * attn_interval == n_layer + rec_n_layer); 0 = all    *
                             * attention layers first, then the recurrent ones                     */
} qkv_config;

/* ------------------------------------------------------------------ engine / state ------ */

/* Replaces qwfn::state::init (src/qwfn_state.h:46-47, src/qwfn_state.cpp:21-46).  device < 0
 * creates a host-only engine: page tables, refcounts and snapshots work, kernels return
 * QKV_ERR_UNSUPPORTED (used to test the host logic on machines without a GPU). */
qkv_status qkv_create(const qkv_config *cfg, int device, qkv_engine **out);
/* Replaces qwfn::state::~state (src/qwfn_state.cpp:12-19). */
void qkv_destroy(qkv_engine *eng);
const char *qkv_last_error(const qkv_engine *eng);
const char *qkv_status_string(qkv_status st);

/* Replaces state::bytes() / state::summary() (src/qwfn_state.h:66-67, src/qwfn_state.cpp:154-173).
 * Writes a NUL-terminated line into buf (truncated to cap). */
qkv_status qkv_bytes(const qkv_engine *eng, size_t *device_bytes);
qkv_status qkv_summary(const qkv_engine *eng, char *buf, size_t cap);

/* Sequence slots.  The reference holds one sequence (src/qwfn_state.h:14-16); slots generalise
 * it.  qkv_seq_reset replaces state::reset / engine::reset (src/qwfn_state.cpp:113-121,
 * src/qwfn_engine.cpp:1055-1066): pages released, n_past = 0, recurrent and conv state zeroed. */
qkv_status qkv_seq_alloc(qkv_engine *eng, int32_t slot);
qkv_status qkv_seq_free(qkv_engine *eng, int32_t slot);
qkv_status qkv_seq_reset(qkv_engine *eng, int32_t slot, void *stream);
qkv_status qkv_seq_length(const qkv_engine *eng, int32_t slot, int32_t *n_past);
/* Make the positions a slot will append next, n_past .. n_tokens-1, writable now (allocating
 * pages, copying a shared page that holds n_past), so the appends touch no host state; n_past is
 * unchanged.  Lets a caller capture decode steps in a CUDA graph.  The reference allocates its
 * cache whole at init (src/qwfn_state.cpp:93-111). */
qkv_status qkv_seq_reserve(qkv_engine *eng, int32_t slot, int32_t n_tokens, void *stream);
/* Page ids of a slot's block table (host copy), for inspection and tests. */
qkv_status qkv_seq_pages(const qkv_engine *eng, int32_t slot, int32_t *pages, int32_t cap, int32_t *n);
qkv_status qkv_page_refcount(const qkv_engine *eng, int32_t page, int32_t *refcount);
qkv_status qkv_pages_free(const qkv_engine *eng, int32_t *n_free);

/* ------------------------------------------------------------------ kernel A -------------- */

/* Quantise n_rows F32 rows of K and V (device, [n_rows][n_head_kv*head_dim]) to q8_0 and write
 * them at positions pos .. pos+n_rows-1 of layer `layer` of `slot`.  Bit-exact with ggml's
 * quantize_row_q8_0.  Pages are allocated on demand; a page shared with a snapshot is copied
 * first (copy-on-write).  pos <= n_past is required; n_past becomes max(n_past, pos+n_rows).
 * Replaces graph_builder::kv_append (src/qwfn_graph.cpp:370-384, ggml_cpy F32 -> Q8_0) and
 * qsa_dec_kv_write (src/qwfn_graph.cpp:612-628, ggml_set_rows). */
qkv_status qkv_append(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos,
                      const float *K, const float *V, int32_t n_rows, void *stream);

/* Projections of the new tokens fused with kernel A: for T <= 4 tokens at positions
 * pos .. pos+T-1 of a slot, K = rope(rms_norm(Wk x) * k_norm) and V = Wv x per KV head are
 * quantised to q8_0 into the cache exactly as qkv_append would store them, and (with Wq) the query
 * Q = rope(rms_norm(Wq x) * q_norm) per query head is written to Q_out for the attention call.
 * Replaces graph_builder::qsa_dec_qkv + qsa_dec_kv_write (src/qwfn_graph.cpp:582-628: the
 * projections, the reference's rms() and rope() helpers, src/qwfn_graph.cpp:125-132, and the
 * set_rows); the F32 K/V rows never reach memory.  x: device F32 [T][n_embd] (n_embd a multiple
 * of 256, T * n_embd <= 12288; 2560 in the model); Wq: device bf16 [2*n_head*head_dim][n_embd], query and gate rows interleaved per
 * head as attn_q.weight is (NULL: no query); Wk, Wv: device bf16 [n_head_kv*head_dim][n_embd];
 * q_norm, k_norm: device F32 [head_dim]; rope: the first rope_dim dims of each head, NEOX pairs,
 * theta_i = p * freq_base^(-2i/rope_dim) (text positions); Q_out: device F32 [T][n_head][head_dim].
 * pos <= n_past; n_past becomes max(n_past, pos+T).  Weight and input pointers 16-byte aligned. */
qkv_status qkv_project_append(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, const float *x,
                              int32_t n_embd, int32_t T, const uint16_t *Wq, const uint16_t *Wk,
                              const uint16_t *Wv, const float *q_norm, const float *k_norm, float rms_eps,
                              int32_t rope_dim, float rope_freq_base, float *Q_out, void *stream);

/* ------------------------------------------------------------------ kernel C -------------- */

/* Decode / MTP-verify attention for n_seq sequences, T (1..4) query tokens each.
 *   slots[n_seq], pos0[n_seq]: HOST arrays; query token t of sequence i sits at position
 *       pos0[i] + t and sees cache cells c <= pos0[i] + t (causal among the T tokens), i.e. the
 *       per-position npast masks of src/qwfn_graph.cpp:671-675 chained as in
 *       src/qwfn_engine.cpp:2266-2281.  The rows of the T tokens must already be appended.
 *   Q:   device F32 [n_seq][T][n_head][head_dim];  out: device F32, same shape.
 *   sel_blocks: NULL for dense attention over cells 0..pos0+T-1, or device int32
 *       [n_seq][n_head_kv][n_sel] 64-token block ids (from qkv_select_blocks; -1 = unused) for
 *       sparse attention over those blocks only, read in place (no gather copy).
 * softmax(scale * QK^T + mask) V with the query converted to q8_0, exact int32 block dots, F32
 * softmax and accumulation -- ggml_flash_attn_ext with GGML_PREC_F32 over the q8_0 cache
 * (src/qwfn_graph.cpp:461-471 and 697-699). */
qkv_status qkv_attn_decode(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                           int32_t n_seq, const float *Q, int32_t T, float scale,
                           const int32_t *sel_blocks, int32_t n_sel, float *out, void *stream);

/* Kernel A fused into kernel C: append the T new K/V rows of each sequence at pos0[i] (device F32
 * [n_seq][T][n_head_kv*head_dim]; bit-exact q8_0 as qkv_append) and run the dense decode of
 * qkv_attn_decode over cells 0..pos0[i]+t, in one launch.  Same position rules as qkv_append
 * (pos0[i] <= n_past; n_past becomes max(n_past, pos0[i]+T)); each slot at most once.  This is
 * the reference's set_rows + flash_attn_ext pair of one decode graph (src/qwfn_graph.cpp:612-628,
 * 697-699) as a single kernel. */
qkv_status qkv_append_attn_decode(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                  int32_t n_seq, const float *K, const float *V, const float *Q, int32_t T,
                                  float scale, float *out, void *stream);

/* ------------------------------------------------------------------ kernel B -------------- */

/* Recompute the per-block key summaries of blocks [b0, b1) of `slot`'s layer `layer` from the
 * q8_0 cache (fp16 mean of the dequantised K rows of each 64-token block, per KV head).  Replaces
 * qsa_dec_index's pooling and engine::qsa_pool_rebuild (src/qwfn_graph.cpp:282-301, 529-552,
 * src/qwfn_engine.cpp:1107-1148) for the synthetic sparse config.  Needs select_block == 64. */
qkv_status qkv_block_summary(qkv_engine *eng, int32_t layer, int32_t slot, int32_t b0, int32_t b1,
                             void *stream);

/* Score the blocks of each sequence against its T query tokens and keep top_k per KV head.
 * Blocks 0 .. nb-1 with nb = ceil((pos0+T)/64) are candidates; block 0 and the last two are
 * always kept (the 1e9 bias of src/qwfn_engine.cpp:1092-1096), the others are ranked by
 * sum over the group's query heads and tokens of relu(q . summary) (src/qwfn_graph.cpp:560-574),
 * ties by lower block index.  idx_out: device int32 [n_seq][n_head_kv][top_k], best first.
 * scores_out: nullable device F32 [n_seq][n_head_kv][max_blocks] (max_blocks = n_ctx/64).
 * Replaces qsa_dec_cells / qsa_top_k (src/qwfn_graph.cpp:556-579, 313-367). */
qkv_status qkv_select_blocks(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                             int32_t n_seq, const float *Q, int32_t T, int32_t top_k,
                             int32_t *idx_out, float *scores_out, void *stream);

/* Raw gather of cache rows in ggml's layout: for each of n_cells positions (device int32),
 * write the K and V q8_0 rows (n_head_kv*head_dim/32*34 bytes each) to K_out / V_out (device).
 * Replaces graph_builder::qsa_gather's raw path (src/qwfn_graph.cpp:632-651). */
qkv_status qkv_gather_rows(qkv_engine *eng, int32_t layer, int32_t slot, const int32_t *cells,
                           int32_t n_cells, void *K_out, void *V_out, void *stream);
/* Contiguous rows pos .. pos+n-1 in ggml's layout (the bytes a ggml view of the cache holds). */
qkv_status qkv_read_rows(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, int32_t n,
                         void *K_out, void *V_out, void *stream);
/* The inverse: store ggml-layout q8_0 rows (device) at pos .. pos+n-1 (allocating pages). */
qkv_status qkv_write_rows(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, int32_t n,
                          const void *K_in, const void *V_in, void *stream);

/* ------------------------------------------------------------------ QSA lightning indexer -- */

/* The model's own sparse-attention selector (src/qwfn_graph.cpp:280-367, 529-579,
 * src/qwfn_engine.cpp:1072-1148), decode path.  Per token the caller supplies the indexer's raw
 * key (F32 [key_len], after k_proj) and its query (F32 [n_head][key_len], after q_proj, q_norm
 * and rope: idx_query, src/qwfn_graph.cpp:303-311); the projections need the model's weights
 * and stay with the caller.  The engine keeps the raw keys as fp16 (the reference's F16
 * idx_cache) and, for every block of `ratio` cells once its last cell is written, the pooled
 * key fp16( rope( rms_norm(mean of the ratio raw keys) * k_norm ) ) at the block's first position
 * (qsa_pool_blocks).  Text positions: the rope sections then all read the same position, so the
 * interleaved multi-section rope is the NEOX-paired rotation of the first rope_dim dims with
 * theta_i = p * freq_base^(-2i/rope_dim) (built as ggml's CPU rope does, by repeated fp32
 * multiplication).  Both live in pages parallel to the KV pages (same page ids), so snapshots,
 * restores and copy-on-write carry them. */
typedef struct qkv_indexer_config {
    int32_t n_head;         /* indexer heads (4)                                                */
    int32_t key_len;        /* 128 (the only value this build provides)                         */
    int32_t ratio;          /* cells per block (4, the only value this build provides)          */
    int32_t top_k;          /* cells kept per token (2048): k_blocks = ceil((top_k+ratio-1)/ratio) */
    int32_t rope_dim;       /* dims rotated (64; even, <= key_len)                              */
    float   rope_freq_base; /* 1e7                                                              */
    float   rms_eps;        /* 1e-6                                                             */
} qkv_indexer_config;
/* Turns the indexer on (once, before any indexer call); k_norm: host F32 [n_layer][key_len]
 * (indexer.k_norm.weight per attention layer), NULL = all ones. */
qkv_status qkv_indexer_enable(qkv_engine *eng, const qkv_indexer_config *cfg, const float *k_norm);
/* Store n_rows raw keys (device F32 [n_rows][key_len]) at positions pos .. pos+n_rows-1 of a
 * slot (pos <= the slot's n_past; its pages must exist: append the K/V rows first) and pool
 * every block whose last cell is among them.  Replaces the indexer-key copy and pooling of
 * qsa_top_k / qsa_dec_index (src/qwfn_graph.cpp:330-336, 529-552). */
qkv_status qkv_idx_append(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, const float *k_raw,
                          int32_t n_rows, void *stream);
/* Block selection for T tokens per sequence at positions pos0[i] .. pos0[i]+T-1 (each token t
 * selects for itself, as the reference's chained verify does).  For the token at position p:
 * whole blocks b < (p+1)/ratio score sum_h relu(fp16(q_h) . pooled_b) (qsa_dec_cells,
 * src/qwfn_graph.cpp:556-579); the block holding p, if incomplete, is always kept (the 1e9
 * bias, src/qwfn_engine.cpp:1092-1096); the best k_blocks blocks in all are kept, ties by lower
 * block index, or every block 0 .. p/ratio when there are no more than k_blocks.  q_idx: device
 * F32 [n_seq][T][n_head][key_len]; blocks_out: device int32 [n_seq][T][k_blocks], ascending
 * block ids, -1 after the n_out_out[i][t] kept ones; scores_out (nullable): device F32
 * [n_seq][T][n_ctx/ratio], the scores of the whole blocks. */
qkv_status qkv_idx_select(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0, int32_t n_seq,
                          const float *q_idx, int32_t T, int32_t *blocks_out, int32_t *n_out_out, float *scores_out,
                          void *stream);
/* Sparse decode with the indexer: select as qkv_idx_select, gather each token's kept cells
 * (those <= its position) into scratch pages, and attend to them with the decode kernel --
 * the reference's qsa_dec_cells + cell mask + raw qsa_gather + ggml_flash_attn_ext
 * (src/qwfn_graph.cpp:653-705).  Q/out as qkv_attn_decode. */
qkv_status qkv_attn_decode_qsa(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                               int32_t n_seq, const float *q_idx, const float *Q, int32_t T, float scale, float *out,
                               void *stream);

/* The indexer's prefill side (graph_builder::sparse_attn with qsa_top_k + qsa_mask,
 * src/qwfn_graph.cpp:313-415, tables of engine::fill_chunk_qsa, src/qwfn_engine.cpp:1276-1320):
 * every query row of the chunk (position pos0 + t) keeps the incomplete block that holds it (if
 * any) and the best k_blocks - 1 (or k_blocks) whole blocks before it by the indexer score, as the
 * decode path does per token (all blocks when there are no more), and attends causally to the
 * kept cells only.  q_idx: device F32 [Tc][n_head_idx][key_len] (the rows' indexer queries);
 * Q: bf16 [Tc][n_head][head_dim] as qkv_attn_prefill.  The chunk's K/V rows (qkv_append) and
 * indexer keys (qkv_idx_append) must be appended first.  blocks_out / n_out (nullable, both or
 * neither): device int32 [Tc][k_blocks] kept block ids ascending and [Tc] counts. */
qkv_status qkv_attn_prefill_qsa(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos0, const float *q_idx,
                                const uint16_t *Q, int32_t Tc, float scale, float *out, int32_t *blocks_out,
                                int32_t *n_out, void *stream);
/* Stored indexer data for tests and snapshots: raw keys of positions pos .. pos+n-1 (device fp16
 * [n][key_len]) and pooled keys of blocks b0 .. b0+n_blk-1 (device fp16 [n_blk][key_len]); either
 * output may be NULL. */
qkv_status qkv_idx_read(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, int32_t n, uint16_t *keys_out,
                        int32_t b0, int32_t n_blk, uint16_t *pooled_out, void *stream);

/* ------------------------------------------------------------------ kernel D -------------- */

/* Chunked causal prefill: Tc query tokens at positions pos0 .. pos0+Tc-1 (their K/V rows
 * already appended) attend to cells 0 .. pos0+t.  Q: device bf16 [Tc][n_head][head_dim] (raw
 * bf16 bits); out: device F32 [Tc][n_head][head_dim].  Replaces the prefill
 * ggml_flash_attn_ext call of graph_builder::sparse_attn (src/qwfn_graph.cpp:417-476) with the
 * dense causal mask built in engine::build_attn_inputs (src/qwfn_engine.cpp:1238-1274). */
qkv_status qkv_attn_prefill(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos0,
                            const uint16_t *Q, int32_t Tc, float scale, float *out, void *stream);

/* ------------------------------------------------------------------ kernel E -------------- */

/* Snapshot of a slot's first n_past positions: its pages are shared (refcounted, no KV bytes
 * move) and the recurrent/conv state is copied device-to-device.  Replaces
 * engine::snapshot_save (src/qwfn_engine.h:296-311, src/qwfn_engine.cpp:988-1027), whose
 * snapshot is a set of host blobs. */
qkv_status qkv_snapshot_save(qkv_engine *eng, int32_t slot, qkv_snapshot **out, void *stream);
/* Restore a snapshot into a slot, keeping its first n_keep positions (n_keep < 0: all).  The
 * slot's old pages are released, the snapshot's pages are shared, a partly kept page is copied
 * on the slot's first write into it, and the recurrent/conv state is copied back.  Replaces
 * engine::snapshot_load (src/qwfn_engine.cpp:1029-1053) and the server's restore_or_reset
 * (tools/qwfn_server.cpp:1380-1404). */
qkv_status qkv_snapshot_restore(qkv_engine *eng, const qkv_snapshot *snap, int32_t slot, int32_t n_keep,
                                void *stream);
/* The same for many slots at once: one batched copy launch for all recurrent state. */
qkv_status qkv_snapshot_restore_many(qkv_engine *eng, const qkv_snapshot *snap, const int32_t *slots,
                                     const int32_t *n_keep, int32_t n, void *stream);
void qkv_snapshot_release(qkv_engine *eng, qkv_snapshot *snap);
qkv_status qkv_snapshot_info(const qkv_snapshot *snap, int32_t *n_past, size_t *host_bytes);
/* Host blobs in the reference's snapshot_parts order (src/qwfn_engine.cpp:987-998): layer by
 * layer (absolute order when attn_interval is set, else attention layers first), an attention
 * layer contributes its first n_past K rows, then V rows (ggml q8_0 layout), then -- with the
 * indexer on -- its n_past raw indexer keys (fp16 [n_past][128]); a recurrent layer its state
 * then its conv history (F32).  The PLE conv state that ends the reference's blob is not held by
 * this engine.  Importing re-pools the indexer's whole blocks.  dst/src are host memory. */
qkv_status qkv_snapshot_to_host(qkv_engine *eng, const qkv_snapshot *snap, void *dst, size_t bytes,
                                void *stream);
qkv_status qkv_snapshot_from_host(qkv_engine *eng, const void *src, size_t bytes, int32_t n_past,
                                  qkv_snapshot **out, void *stream);

/* ------------------------------------------------------------------ saved-sequence store --- */

/* Saved sequences keyed by their token ids, held as device snapshots (shared pages + a device
 * copy of the recurrent state) instead of host blobs.  Replaces the server's saved_seq list and
 * its restore / shared-prefix logic (tools/qwfn_server.cpp:764-800, 1380-1430): at most
 * max_entries sequences (the reference keeps 4) holding at most cap_bytes of device memory
 * (snapshot pages in every layer + recurrent copy; the reference caps host bytes by
 * QWFN_SNAP_MB), least recently used first out.  Bound to one engine; destroy it before the
 * engine. */
typedef struct qkv_store qkv_store;
qkv_status qkv_store_create(qkv_engine *eng, size_t cap_bytes, int32_t max_entries, qkv_store **out);
void qkv_store_destroy(qkv_store *store);
/* Snapshot a slot whose n_past equals n_tok and keep it under tok[0..n_tok) (server save_seq,
 * tools/qwfn_server.cpp:771-780): an entry with equal tokens is replaced; a snapshot above the
 * cap is not kept (*kept = 0, not an error); older entries leave until both limits hold. */
qkv_status qkv_store_save(qkv_store *store, int32_t slot, const int32_t *tok, int32_t n_tok, int32_t *kept,
                          void *stream);
/* Restore into slot the longest saved sequence that prompt[0..n_prompt) strictly extends and make
 * it the most recently used (*n_restored = its length); with none, or if its restore fails,
 * reset the slot (*n_restored = 0).  The server's restore_or_reset after its set-aside step
 * (tools/qwfn_server.cpp:1380-1404, best_saved 782-794); the set-aside is a qkv_store_save. */
qkv_status qkv_store_restore_or_reset(qkv_store *store, int32_t slot, const int32_t *prompt, int32_t n_prompt,
                                      int32_t *n_restored, void *stream);
/* Where a fresh prefill should stop once to save a prefix it shares with a saved sequence
 * (shared_prefix_split, tools/qwfn_server.cpp:1410-1430): the longest common prefix L with any
 * entry if n_consumed < min_prefix, L >= min_prefix, L + 16 < n_prompt, L >= n_consumed + 2 and
 * no entry is exactly that prefix; else 0.  The reference's min_prefix is 2048. */
qkv_status qkv_store_prefix_split(const qkv_store *store, const int32_t *prompt, int32_t n_prompt,
                                  int32_t n_consumed, int32_t min_prefix, int32_t *split_at);
/* Drop the n least recently used entries (e.g. when the page pool runs out). */
qkv_status qkv_store_evict(qkv_store *store, int32_t n);
/* Entries and the device bytes they hold; entry i in LRU order (0 = least recently used). */
qkv_status qkv_store_info(const qkv_store *store, int32_t *n_entries, size_t *bytes);
qkv_status qkv_store_entry(const qkv_store *store, int32_t i, int32_t *n_tok, size_t *bytes);

/* Rewind n_back positions after rejected drafts: restore the recurrent/conv state from
 * rollback snapshot n_back-1 and set n_past -= n_back (cache rows are overwritten later).
 * Replaces engine::rollback_n (src/qwfn_engine.cpp:3629-3660). */
qkv_status qkv_rollback(qkv_engine *eng, int32_t slot, int32_t n_back, void *stream);
/* Declare that rollback snapshots 0..depth-1 of a slot hold the state 1..depth tokens back (the
 * DeltaNet step that wrote them calls this; the reference sets rb_valid_/rb_depth_ in
 * eval_batch after a multi-token step, src/qwfn_engine.cpp:3630-3655). */
qkv_status qkv_rollback_arm(qkv_engine *eng, int32_t slot, int32_t depth);

/* Device pointers of a slot's recurrent state for the (out-of-scope) DeltaNet kernels:
 * kind 0 = state [rec_head_dim, rec_head_dim, rec_n_head] F32, kind 1 = conv [conv_hist,
 * conv_channels] F32; which 0 = live state, 1..n_rollback = rollback snapshot which-1.
 * Replaces state::rs_state / rs_conv (src/qwfn_state.h:55-57). */
qkv_status qkv_state_ptr(qkv_engine *eng, int32_t slot, int32_t rec_layer, int32_t kind, int32_t which,
                         void **ptr, size_t *bytes);

/* Description of a layer's page pool, for k_cache(il)/v_cache(il) style access
 * (src/qwfn_state.h:50-53). */
typedef struct qkv_cache_view {
    void   *pool;          /* device base of the layer's page pool                       */
    size_t  page_bytes;    /* bytes of one page (all KV heads, K and V)                  */
    size_t  tile_bytes;    /* bytes of one 64-token tile of one KV head                  */
    int32_t page_tokens;   /* 256                                                        */
    int32_t tile_tokens;   /* 64                                                         */
    int32_t n_pages;
    int32_t n_head_kv;
    int32_t head_dim;
    const int32_t *block_table;  /* device [n_slots][max_pages_per_seq] page ids, -1 = none */
    int32_t max_pages_per_seq;
} qkv_cache_view;
qkv_status qkv_cache_view_get(const qkv_engine *eng, int32_t layer, qkv_cache_view *view);

/* Allocation-free dense decode.  No counterpart in the reference: it exists for callers that must
 * not allocate device memory -- a custom op inside ggml's graph executor (memory planned ahead by
 * ggml-alloc, nothing may grow mid-graph) or code under an allocator that owns the whole device.
 * Same attention as qkv_attn_decode over a cache described by a qkv_cache_view (from
 * qkv_cache_view_get; block_table has n_slots rows), Q/out device F32 [n_seq][T][n_head][head_dim].
 * The split-K scratch is a fixed 6.05 MiB array compiled into the library (held on every GPU that
 * loads it until exit), so T * n_head / n_head_kv must be <= 32 (else QKV_ERR_UNSUPPORTED).
 * Calls share that array: calls that overlap on the GPU race.  The first call on a device looks
 * up the array's address and should come before any stream capture.  Bounds violations and
 * timed-out waits seen by the kernels are recorded in a status word of the same fixed scratch,
 * which each call clears first: read it with qkv_static_status. */
qkv_status qkv_attn_decode_static(const qkv_cache_view *view, int32_t n_slots, const int32_t *slots,
                                  const int32_t *pos0, int32_t n_seq, int32_t n_head, const float *Q,
                                  int32_t T, float scale, float *out, void *stream);

/* The device status of the last qkv_attn_decode_static call on the current device (same bits as
 * qkv_device_status: 1 bad page, 2 bad index, 4 timed-out wait), read on `stream` (synchronising
 * it) and cleared.  Allocates nothing, like the entry point it reports on.  No counterpart in the
 * reference.  Returns QKV_ERR_DEVICE when the word was non-zero. */
qkv_status qkv_static_status(void *stream, int32_t *code);

/* Reads (and clears) the device status word that checked kernels write on a bounds violation.
 * Synchronises the stream. */
qkv_status qkv_device_status(qkv_engine *eng, void *stream, int32_t *code);

/* Failure-detection tests.  No counterpart in the reference.  Sets the limit of the decode kernels'
 * bounded waits (the tile copies; default 2 s) and, when
 * withhold_unit >= 0, makes the NEXT decode launch of this engine skip the copy of that unit's first
 * tile while still waiting for its bytes: the wait runs out after wait_limit_ns, the kernel sets
 * the timed-out bit (4) of the device status and returns, and the context stays usable.  Nothing
 * faults and nothing hangs.  wait_limit_ns <= 0 restores the default. */
qkv_status qkv_debug_decode_wait(qkv_engine *eng, int64_t wait_limit_ns, int32_t withhold_unit);

/* Numerics test.  No counterpart in the reference.  For every non-negative float x (bit patterns
 * 0 .. 0x7F800000) compares the library's q8_0 block-scale arithmetic -- d = x / 127 and 1 / x as
 * the quantisers of kernels A, C and D compute them -- with the device's IEEE division and
 * reciprocal, and writes the number of differing results.  Synchronous on the current device. */
qkv_status qkv_debug_check_q8_scale(uint64_t *mismatch_div, uint64_t *mismatch_rcp);

/* Kernels this process has launched through the library so far (all engines, all devices). */
qkv_status qkv_launch_count(uint64_t *count);

/* ------------------------------------------------------------------ multi-GPU ------------ */

/* Longest-processing-time partition of n independent sequences over n_ranks GPUs by cost
 * (e.g. context length): owner[i] receives the rank of sequence i.  Sequences never split,
 * so no collective is needed on the attention path. */
qkv_status qkv_shard_lpt(const int64_t *cost, int32_t n, int32_t n_ranks, int32_t *owner);

#ifdef __cplusplus
}
#endif

#endif /* QKV_H */
