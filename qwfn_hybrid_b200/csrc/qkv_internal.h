// qkv_internal.h -- cache layout constants and kernel launch interfaces shared by the engine
// (qkv_engine.cpp) and the kernels (*.cu).  Not part of the public ABI (include/qkv.h).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>

#include "qkv.h"

namespace qkv {

// Kernels launched by this library (qkv_launch_count); bumped by every launch helper.
void count_launches(uint64_t n);

// ---- q8_0 and head geometry ---------------------------------------------------------------
constexpr int HD         = 256;         // head_dim (the only value provided)
constexpr int QK         = 32;          // q8_0 block
constexpr int NBLK       = HD / QK;     // 8 q8_0 blocks per head row
constexpr int ROW_Q8     = NBLK * 34;   // 272 bytes of ggml block_q8_0 per head row

// ---- pages and tiles ------------------------------------------------------------------------
// A page holds 256 positions of one layer.  Per KV head it holds four 64-token tiles, each a
// contiguous 34816-byte record, so that one bulk copy moves everything attention needs for
// 64 tokens of one head:
//   [0, 16384)      K quants, token-major: token t's 256 int8 at t*256, its 16-byte chunks
//                   XOR-swizzled by kswz(t) (bank-conflict-free ldmatrix of 8 token rows)
//   [16384, 32768)  V quants, transposed: dim i's 64 int8 (tokens) at 16384 + i*64, its four
//                   16-byte chunks XOR-swizzled by (i>>1)&3
//   [32768, 33792)  K scales, fp16 [64 tokens][8 blocks]
//   [33792, 34816)  V scales, fp16 [8 blocks][64 tokens]
// Page = [head][tile] records; page bytes = n_head_kv * 4 * 34816 (278528 for two heads, the
// same bytes as 256 ggml q8_0 K and V rows of 544 bytes).
constexpr int PAGE_TOK       = 256;
constexpr int TILE_TOK       = 64;
constexpr int TILES_PER_PAGE = PAGE_TOK / TILE_TOK;
constexpr int TILE_KQ        = 0;
constexpr int TILE_VQ        = 16384;
constexpr int TILE_KD        = 32768;
constexpr int TILE_VD        = 33792;
constexpr int TILE_BYTES     = 34816;

__host__ __device__ __forceinline__ int kswz(int t) { return (((t >> 2) & 3) << 1) | (t & 1); }

#ifdef __CUDACC__
// roundf(v) -- round half away from zero, as ggml's quantize_row_q8_0 rounds -- for |v| <= 128,
// in FP32 adds instead of the conversion pipe (which bounds kernels that round many values):
// with both additions rounded toward zero, rz(rz(|v| + 0.5) + 2^23) = 2^23 + floor(|v| + 0.5)
// exactly, so the integer is the low mantissa bits.  Checked against roundf for every float in
// [-128, 128] (an exhaustive host run of the same two round-toward-zero additions).
__device__ __forceinline__ int round_half_away(float v) {
    const float r = __fadd_rz(__fadd_rz(fabsf(v), 0.5f), 8388608.0f);
    const int mag = __float_as_int(r) - 0x4B000000;
    return v < 0.0f ? -mag : mag;
}
// The same rounding as a float (roundf's value, sign of zero included).
__device__ __forceinline__ float round_half_away_f(float v) {
    const float r = __fadd_rz(__fadd_rz(fabsf(v), 0.5f), 8388608.0f);
    return copysignf(__fadd_rn(r, -8388608.0f), v);
}
// The q8_0 block scale of ggml's quantize_row_q8_0: d = amax / 127 and id = 1 / d (0 when d is 0),
// both correctly rounded, on the FMA pipe instead of the library's division and reciprocal
// sequences (which bound kernels that quantise many blocks):
//  * quotient by the constant 127: q = RN(x c) with c = RN(1/127), the residual x - 127 q exactly
//    by one FMA, then RN(q + residual c) (Markstein's correction step for a constant divisor);
//  * reciprocal: the hardware estimate r0 (rcp.approx), e = 1 - d r0 exactly by one FMA, then
//    RN(r0 + r0 e) (one Newton-Raphson step).
// Inputs outside [2^-100, 2^100] (never met by real activations) take __fdiv_rn / __frcp_rn.  The
// fast paths equal __fdiv_rn(x, 127) and __frcp_rn(x) for every float in that range
// (qkv_debug_check_q8_scale runs the exhaustive comparison on the device).
__device__ __forceinline__ float div127_rn(float x) {
    if (!(x >= 0x1p-100f && x <= 0x1p100f)) return __fdiv_rn(x, 127.0f);
    constexpr float c = 1.0f / 127.0f;
    const float q = __fmul_rn(x, c);
    const float r = __fmaf_rn(-q, 127.0f, x);
    return __fmaf_rn(r, c, q);
}
__device__ __forceinline__ float rcp_rn(float d) {
    if (!(d >= 0x1p-100f && d <= 0x1p100f)) return __frcp_rn(d);
    float r0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(d));
    const float e = __fmaf_rn(-d, r0, 1.0f);
    return __fmaf_rn(r0, e, r0);
}
#endif
// byte offset of K quant (token t, element j) inside a tile
__host__ __device__ __forceinline__ int k_off(int t, int j) {
    return TILE_KQ + t * HD + ((((j >> 4) ^ kswz(t))) << 4) + (j & 15);
}
// byte offset of V quant (element i, token t) inside a tile
__host__ __device__ __forceinline__ int v_off(int i, int t) {
    return TILE_VQ + i * TILE_TOK + ((((t >> 4) ^ ((i >> 1) & 3))) << 4) + (t & 15);
}
__host__ __device__ __forceinline__ int kd_off(int t, int b) { return TILE_KD + (t * NBLK + b) * 2; }
__host__ __device__ __forceinline__ int vd_off(int b, int t) { return TILE_VD + (b * TILE_TOK + t) * 2; }

// Device status word bits (qkv_device_status).
constexpr int32_t ST_BAD_PAGE  = 1;    // a block-table entry was < 0 or >= n_pages
constexpr int32_t ST_BAD_INDEX = 2;    // a cell / block index outside the sequence
constexpr int32_t ST_TIMEOUT   = 4;    // a bounded wait on a tile copy gave up

// ---- kernel A and layout transforms ------------------------------------------------------------
struct PoolRef {
    uint8_t       *pool;          // layer pool base
    const int32_t *bt;            // block-table row of the slot (device)
    int64_t        page_bytes;
    int32_t        n_pages;
    int32_t        max_pages;     // length of the block-table row
    int32_t        n_head_kv;
    int32_t       *status;
};

cudaError_t launch_append(const PoolRef &pr, int32_t pos, const float *K, const float *V, int32_t n_rows,
                          cudaStream_t st);

// Fused projection + rms-norm + rope + q8_0 append for up to PJ_MAX_T tokens (k_project_dot; n_embd a multiple of 256, T * n_embd floats within 48 KiB of shared memory).
constexpr int PJ_MAX_T = 4, PJ_MAX_HALF = 64;
struct ProjectParams {
    PoolRef        pr;            // the slot's pages in the layer's pool
    const float   *x;             // [T][n_embd]
    const uint16_t *Wq, *Wk, *Wv; // bf16 weights, rows of n_embd; Wq: query/gate interleaved per head (nullable)
    const float   *q_norm, *k_norm;   // [HD]
    float         *Q_out;         // [T][n_head][HD] (with Wq)
    int32_t n_embd, T, pos, n_head, n_head_kv, rope_half;
    float   eps;
    float2  cs[PJ_MAX_T][PJ_MAX_HALF];   // {cos, sin} of pair i at position pos + t
};
cudaError_t launch_project(const ProjectParams &p, cudaStream_t st);
// cells == nullptr: rows pos .. pos+n-1
cudaError_t launch_read_rows(const PoolRef &pr, const int32_t *cells, int32_t pos, int32_t n, uint8_t *K_out,
                             uint8_t *V_out, cudaStream_t st);
cudaError_t launch_write_rows(const PoolRef &pr, int32_t pos, int32_t n, const uint8_t *K_in, const uint8_t *V_in,
                              cudaStream_t st);

// ---- kernel E: batched device copies ------------------------------------------------------------
constexpr int COPY_MAX = 64;
struct CopyDesc {
    const uint8_t *src;
    uint8_t       *dst;
    int64_t        bytes;          // multiple of 16, both pointers 16-byte aligned
};
cudaError_t launch_copy_batch(const CopyDesc *descs, int n, int num_sms, cudaStream_t st);

// ---- kernel B ---------------------------------------------------------------------------------
cudaError_t launch_block_summary(const PoolRef &pr, int32_t b0, int32_t b1, uint16_t *summary, int32_t max_blocks,
                                 cudaStream_t st);

constexpr int MAX_SEQ = 64;
struct SelectParams {
    const float    *Q;            // [n_seq][T][n_head][HD]
    const uint16_t *summary;      // layer base: [slot][n_head_kv][max_blocks][HD] fp16
    int32_t        *idx_out;      // [n_seq][n_head_kv][top_k]
    float          *scores;       // [n_seq][n_head_kv][max_blocks]: the caller's scores_out, or engine scratch
    int32_t n_seq, T, n_head, n_head_kv, G, top_k, max_blocks;
    int32_t chunk, rk;            // set by launch_select: candidates per score CTA, rank CTAs per (sequence, head)
    int32_t seq_slot[MAX_SEQ];
    int32_t seq_nblk[MAX_SEQ];    // candidate blocks of each sequence
};
cudaError_t launch_select(const SelectParams &p, cudaStream_t st);

// ---- QSA lightning indexer --------------------------------------------------------------------
// Per attention layer an indexer pool parallel to the KV pool (same page ids).  An indexer page
// holds the raw keys of its 256 positions, fp16 [256][IDX_KEY], then the pooled keys of its 64
// blocks of IDX_R cells, fp16 [64][IDX_KEY].
constexpr int IDX_KEY        = 128;
constexpr int IDX_R          = 4;
constexpr int IDX_BPP        = PAGE_TOK / IDX_R;
constexpr int IDX_RAW_BYTES  = PAGE_TOK * IDX_KEY * 2;
constexpr int IDX_PAGE_BYTES = IDX_RAW_BYTES + IDX_BPP * IDX_KEY * 2;
constexpr int IDX_MAX_HEAD   = 8;
constexpr int IDX_MAX_VSEQ   = 256;   // (sequence, token) pairs per selection launch

struct IdxAppendParams {
    uint8_t       *pool;          // layer indexer pool
    const int32_t *bt;            // block-table row of the slot
    const float   *k_raw;         // [n_rows][IDX_KEY]
    const float   *norm_w;        // [IDX_KEY]
    const float2  *rope;          // [block][rope_half] {cos, sin}
    int32_t       *status;
    int32_t n_pages, max_pages, pos, n_rows, rope_half;
    float   eps;
};
cudaError_t launch_idx_append(const IdxAppendParams &p, cudaStream_t st);
cudaError_t launch_idx_pool(const IdxAppendParams &p, int32_t b_lo, int32_t n_blk, cudaStream_t st);

// One entry per (sequence, token): v = i * T + t; the T entries of a sequence are adjacent.
struct IdxSelectParams {
    const uint8_t *pool;          // layer indexer pool
    const int32_t *bt;            // engine block table [n_slots][max_pages]
    const float   *q;             // [n_v][n_head][IDX_KEY]
    float         *scores;        // [n_v][score_stride]
    int32_t       *blocks;        // [n_v][k_blocks]
    int32_t       *n_out;         // [n_v]
    int32_t       *status;
    int32_t n_v, T, n_head, k_blocks, score_stride, n_pages, max_pages;   // n_v a multiple of T
    int32_t v_slot[IDX_MAX_VSEQ], v_pos[IDX_MAX_VSEQ];
};
cudaError_t launch_idx_select(const IdxSelectParams &p, int32_t max_whole, cudaStream_t st);

// Kept-block bitsets for the sparse prefill: bits[v][words] from blocks[v][k_blocks] / n_out[v].
cudaError_t launch_idx_bits(const int32_t *blocks, const int32_t *n_out, int32_t k_blocks, int32_t n_v, uint32_t *bits,
                            int32_t words, cudaStream_t st);

// ---- kernel C -----------------------------------------------------------------------------------
constexpr int MAX_PAIRS = MAX_SEQ * 8;
struct DecodeParams {
    const uint8_t *pool;
    const int32_t *block_table;   // [n_slots][max_pages]
    const float   *Q;             // [n_seq][T][n_head][HD]
    float         *out;           // [n_seq][T][n_head][HD]
    float         *partial;       // scratch: one record per unit of [nq*HD + 2*nq] floats
    const int32_t *sel;           // nullable [n_seq][n_head_kv][n_sel] block ids
    const float   *Knew, *Vnew;   // nullable [n_seq][T][n_head_kv*HD]: fused append (dense only)
    int32_t       *status;
    int64_t page_bytes;
    int32_t n_pages, max_pages, n_head, n_head_kv, G, T, nq, n_seq, n_sel, n_units;
    int32_t n_merge;              // pairs with more than one unit: plan positions first, pairs 0 .. n_merge-1
    float   scale;
    uint64_t wait_ns;             // limit of every bounded wait (tile copies, the pair barrier)
    int32_t withhold_unit;        // failure tests: this unit's first tile copy is never started (-1: none)
    // QSA mode (grp non-null): sequence i's dense sequence is its kept 4-cell blocks
    // grp[i][0 .. grp_n[i]) (ascending) of the slot's pages; a tile is 16 of them
    const int32_t *grp;
    const int32_t *grp_n;
    int32_t grp_stride;
#ifdef QKV_TIMELINE
    int32_t tl_nopf;              // analysis builds only: no tile prefetch before the dependency wait
#endif
    // per plan position j (sequences ordered by units, largest first):
    int32_t seq_idx[MAX_SEQ];        // the sequence's index in the caller's arrays
    int32_t seq_slot[MAX_SEQ];
    int32_t seq_pos0[MAX_SEQ];
    int32_t seq_tiles[MAX_SEQ];      // tiles of each pair of the sequence
    int32_t seq_units[MAX_SEQ];      // units (CTAs) per pair of the sequence
    int32_t seq_unit0[MAX_SEQ + 1];  // prefix of n_head_kv * seq_units
    int32_t seq_vpos[MAX_SEQ];       // QSA mode: the query's position (every kept cell is <= it)
};
// partial record size in floats for nq query rows: O [nq][HD] unnormalised, m [nq] (log2
// domain), l [nq]
__host__ __device__ __forceinline__ int64_t partial_stride(int nq) { return (int64_t)nq * HD + 2 * nq; }

cudaError_t launch_decode(const DecodeParams &p, cudaStream_t st);   // k_decode, then a merge kernel
int decode_max_nq();
int decode_max_ctas(int nq);       // co-resident CTAs of the decode kernel (0 = unknown)
int decode_merge_max_units();      // units per pair the merge kernel takes
constexpr uint64_t WAIT_NS_DEFAULT = 2000000000ull;   // limit of the decode kernels' bounded waits
// Plans one decode launch of ns sequences (P.n_head_kv, P.nq set; tiles[i] = tiles of each pair of
// sequence i): the per-position arrays, n_units and n_merge.  Units in proportion to tiles, about
// `target` CTAs in all, at least two tiles and at most `umax` units per pair, no more than
// `max_units` (the caller's scratch).
void plan_decode(DecodeParams &P, const int32_t *slots, const int32_t *pos0, const int32_t *tiles, int ns,
                 int64_t target, int64_t umax, int64_t max_units);

// ---- kernel D -----------------------------------------------------------------------------------
// A prefill tile is 128 rows = (128 / G) query tokens x the G q-heads of one KV head.  Two tiles
// of a KV head (query groups 2p, 2p+1: a pair tile) run on a CTA pair whose MMAs cover both.  The
// KV range of a pair tile is cut into segments (contiguous 128-key KV tiles); every pair runs a
// contiguous run of segments.  Each segment leaves two partial records (one per tile: unnormalised
// O, row max, row sums); a second kernel merges the records of every tile and writes the output.
constexpr int PF_ROWS      = 128;
constexpr int PF_KT        = 128;              // keys per KV tile of kernel D
constexpr int PF_MAX_TC    = 4096;             // query tokens per call
constexpr int PF_QTILE     = PF_ROWS * HD * 2; // bytes of one fp16 query tile
// partial record: O as [HD/4 float4 columns][PF_ROWS rows][4] (a warp's rows are adjacent, so the
// epilogue's stores coalesce), then m[PF_ROWS] (log2 domain), then the row sums l[2][PF_ROWS] of
// the two key halves (l = l[0] + l[1])
__host__ __device__ __forceinline__ int64_t pf_part_floats() { return (int64_t)PF_ROWS * HD + 3 * PF_ROWS; }
struct PrefillParams {
    const uint8_t  *pool;
    const int32_t  *bt;           // block-table row of the slot
    const uint16_t *Q;            // bf16 bits [Tc][n_head][HD]
    uint8_t        *qtiles;       // scratch [n_tiles][PF_QTILE]: q8_0-rounded queries, fp16, MMA layout
    float          *out;          // [Tc][n_head][HD]
    float          *partial;      // scratch [parts][pf_part_floats()], one record per segment
    int32_t        *status;
    // the plan, in device memory, or (plan_inline) in the launch's PfPlanInline at int offsets 0
    // (segs), off_tiles (tile_parts), off_cta (cta_seg)
    const int32_t  *cta_seg;      // [n_ctas + 1] first segment of each CTA
    const int4     *segs;         // {tile, kv tile begin, kv tile end, part}
    const int2     *tile_parts;   // {number of parts, first part}
    int32_t plan_inline, off_tiles, off_cta;
    int64_t page_bytes;
    int32_t n_pages, max_pages, n_head, n_head_kv, G, tpt, n_groups, n_tiles, Tc, pos0, n_kv;
    int32_t n_gpairs;             // pairs of query groups per KV head (the plan's pair tiles: kvh * n_gpairs + pair)
    int32_t n_ctas;               // 2 per pair run
    float   scale_log2;           // softmax scale x log2(e)
    // QSA prefill (nullable): per query token of the chunk, qsa_words words of kept indexer blocks
    // (4 cells each, bit b & 31 of word b >> 5); word w covers KV tile w (PF_KT = 32 blocks)
    const uint32_t *qsa_bits;
    int32_t         qsa_words;
};
// A plan of up to PF_PLAN_INLINE ints travels with the launch (kernel parameters), so a call
// needs no host-to-device copy ahead of its kernels.
constexpr int PF_PLAN_INLINE = 2048;
struct alignas(16) PfPlanInline {
    int32_t v[PF_PLAN_INLINE];
};
cudaError_t launch_prefill(const PrefillParams &p, const PfPlanInline &plan, cudaStream_t st);
int prefill_max_pairs();   // co-resident CTA pairs of kernel D (0 = unknown)

// ---- host side shared by the engine and the saved-sequence store (qkv_store.cpp) ---------------
// Sets the engine's last error (qkv_last_error) to msg and returns st.
qkv_status engine_fail(qkv_engine *eng, qkv_status st, const char *msg);
// Device bytes a snapshot holds: its pages in every layer's pool plus its recurrent-state copy
// (counted on host-only engines too, where nothing is allocated).
size_t snapshot_held_bytes(const qkv_snapshot *snap);

}  // namespace qkv
