// qkv_engine.cpp -- host side of the engine: page pool, block tables, sequence slots, snapshots,
// rollback, and the C ABI of include/qkv.h.
//
// The reference keeps one sequence in contiguous per-layer ggml tensors (src/qwfn_state.cpp:
// 48-111) and snapshots by copying their first n_past rows to host blobs (src/qwfn_engine.cpp:
// 988-1053).  Here positions live in 256-token pages drawn from a pool; a slot's block table
// maps page index -> page id (the same id in every layer's pool).  A snapshot shares pages by
// reference count instead of copying them, and a write into a shared page copies it first.
#include "qkv.h"
#include "qkv_internal.h"

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <numeric>
#include <string>
#include <vector>

using namespace qkv;

static std::atomic<uint64_t> g_launches{0};
void qkv::count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

extern "C" qkv_status qkv_launch_count(uint64_t *count) {
    if (!count) return QKV_ERR_INVALID;
    *count = g_launches.load(std::memory_order_relaxed);
    return QKV_OK;
}

struct qkv_snapshot {
    qkv_engine          *eng = nullptr;
    int32_t              n_past = 0;
    std::vector<int32_t> pages;     // shared page ids (one reference each)
    uint8_t             *rec = nullptr;  // device copy of the recurrent / conv state
};

struct qkv_engine {
    qkv_config  cfg{};
    int         device    = -1;
    bool        host_only = true;
    std::string err;
    int         num_sms    = 0;
    int32_t     max_pages  = 0;       // block-table row length
    int32_t     n_pages    = 0;
    int64_t     page_bytes = 0;
    int64_t     rs_bytes = 0, conv_bytes = 0, rec_layer_bytes = 0, rec_slot_bytes = 0;
    int32_t     max_blocks = 0;       // selection blocks per sequence
    int32_t     max_nq     = 0;

    std::vector<int32_t> refcnt;
    std::vector<int32_t> free_pages;  // stack, lowest id on top
    struct Slot {
        bool                 active   = false;
        bool                 dirty    = false;
        int32_t              n_past   = 0;
        int32_t              rb_depth = 0;
        std::vector<int32_t> pages;
    };
    std::vector<Slot>    slots;
    std::vector<int32_t> sum_valid;   // [slot][layer] whole blocks whose summary is current

    std::vector<uint8_t *> pools;     // per layer
    int32_t  *d_bt      = nullptr;    // [n_slots][max_pages]
    uint8_t  *d_rec     = nullptr;    // [n_slots][rec_slot_bytes]
    uint8_t  *d_rb      = nullptr;    // [n_slots][n_rollback][rec_slot_bytes]
    uint16_t *d_summary = nullptr;    // [n_layer][n_slots][n_head_kv][max_blocks][HD]
    float    *d_sel_scores = nullptr; // kernel B1 scratch: [MAX_SEQ][n_head_kv][max_blocks] block scores
    float    *d_partial = nullptr;    // kernel C: per-cluster partial records
    size_t    partial_bytes = 0;
    int32_t  *d_status  = nullptr;
    uint64_t  wait_ns = WAIT_NS_DEFAULT;   // limit of the decode kernels' bounded waits
    int32_t   withhold_unit = -1;     // failure tests: the next decode launch withholds this unit's first tile
    // kernel D scratch, allocated by the first prefill call
    uint8_t  *d_pf_q        = nullptr;    // query tiles
    float    *d_pf_partial  = nullptr;    // split-segment partials
    int32_t  *d_pf_plan     = nullptr;    // segments, tile parts, CTA offsets
    int32_t   pf_max_tiles = 0, pf_max_parts = 0, pf_plan_ints = 0;
    PfPlanInline pf_plan_inline;   // host copy of a small plan, passed with the launch
    size_t    device_bytes = 0;

    // pinned upload ring for block-table rows: a block is reused only after its event fired
    static constexpr int    RING_N     = 32;
    static constexpr size_t RING_BLOCK = 512 * 1024;
    uint8_t    *ring = nullptr;
    cudaEvent_t ring_ev[RING_N]{};
    bool        ring_used[RING_N]{};
    int         ring_next = 0;

    std::vector<qkv_snapshot *> snaps;

    // QSA lightning indexer (qkv_indexer_enable)
    bool                   idx_on = false;
    qkv_indexer_config     icfg{};
    int32_t                k_blocks = 0;      // blocks kept per token
    int32_t                idx_max_blk = 0;   // blocks of n_ctx
    std::vector<uint8_t *> idx_pools;         // per layer, n_pages x IDX_PAGE_BYTES
    float2   *d_rope  = nullptr;              // [idx_max_blk][rope_dim/2] {cos, sin}
    float    *d_knorm = nullptr;              // [n_layer][IDX_KEY]
    // qkv_attn_decode_qsa scratch (grown on demand): scores, kept blocks and their counts
    float    *d_iscore = nullptr;
    int32_t  *d_isel = nullptr, *d_inout = nullptr;
    int32_t   iscratch_v = 0;
    // qkv_attn_prefill_qsa scratch (grown on demand): kept blocks and counts per row, bitsets
    int32_t  *d_psel = nullptr, *d_pnout = nullptr;
    int32_t   psel_rows = 0;
    uint32_t *d_pbits = nullptr;
    int64_t   pbits_words = 0;
};

// ------------------------------------------------------------------------------------ helpers
static qkv_status fail(qkv_engine *eng, qkv_status st, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (eng) eng->err = buf;
    return st;
}
#define CK(eng, call)                                                                              \
    do {                                                                                           \
        const cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess) return fail((eng), QKV_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

static cudaStream_t S(void *stream) { return reinterpret_cast<cudaStream_t>(stream); }

qkv_status qkv::engine_fail(qkv_engine *eng, qkv_status st, const char *msg) { return fail(eng, st, "%s", msg); }

size_t qkv::snapshot_held_bytes(const qkv_snapshot *snap) {
    const qkv_engine *eng = snap->eng;
    return snap->pages.size() * (size_t)eng->page_bytes * eng->cfg.n_layer + (size_t)eng->rec_slot_bytes;
}

static qkv_status use_device(qkv_engine *eng) {
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    int cur = -1;
    CK(eng, cudaGetDevice(&cur));
    if (cur != eng->device) CK(eng, cudaSetDevice(eng->device));
    return QKV_OK;
}

static qkv_status check_slot(qkv_engine *eng, int32_t slot, bool must_be_active = true) {
    if (slot < 0 || slot >= eng->cfg.n_slots) return fail(eng, QKV_ERR_INVALID, "slot %d outside [0, %d)", slot, eng->cfg.n_slots);
    if (must_be_active && !eng->slots[slot].active) return fail(eng, QKV_ERR_STATE, "slot %d is not allocated", slot);
    return QKV_OK;
}
static qkv_status check_layer(qkv_engine *eng, int32_t layer) {
    if (layer < 0 || layer >= eng->cfg.n_layer) return fail(eng, QKV_ERR_INVALID, "layer %d outside [0, %d)", layer, eng->cfg.n_layer);
    return QKV_OK;
}

static void page_ref(qkv_engine *eng, int32_t p) { eng->refcnt[p]++; }
static void page_unref(qkv_engine *eng, int32_t p) {
    if (--eng->refcnt[p] == 0) eng->free_pages.push_back(p);
}
static int32_t page_alloc(qkv_engine *eng) {
    const int32_t p = eng->free_pages.back();
    eng->free_pages.pop_back();
    eng->refcnt[p] = 1;
    return p;
}
static void release_pages(qkv_engine *eng, std::vector<int32_t> &pages) {
    for (int32_t p : pages) page_unref(eng, p);
    pages.clear();
}
static void invalidate_summaries(qkv_engine *eng, int32_t slot, int32_t from_pos) {
    const int32_t blk = from_pos / TILE_TOK;
    for (int l = 0; l < eng->cfg.n_layer; l++) {
        int32_t &v = eng->sum_valid[(size_t)slot * eng->cfg.n_layer + l];
        v = std::min(v, blk);
    }
}

static PoolRef pool_ref(qkv_engine *eng, int32_t layer, const int32_t *bt_row) {
    PoolRef pr;
    pr.pool       = eng->pools[layer];
    pr.bt         = bt_row;
    pr.page_bytes = eng->page_bytes;
    pr.n_pages    = eng->n_pages;
    pr.max_pages  = eng->max_pages;
    pr.n_head_kv  = eng->cfg.n_head_kv;
    pr.status     = eng->d_status;
    return pr;
}

// Reserve a ring block for `bytes` of uploads; returns its host pointer.
static qkv_status ring_block(qkv_engine *eng, int &k, uint8_t *&host) {
    k = eng->ring_next;
    eng->ring_next = (k + 1) % qkv_engine::RING_N;
    if (eng->ring_used[k]) CK(eng, cudaEventSynchronize(eng->ring_ev[k]));
    host = eng->ring + (size_t)k * qkv_engine::RING_BLOCK;
    return QKV_OK;
}

// Upload the block-table rows of all dirty slots (stream-ordered, from pinned staging).
static qkv_status flush_tables(qkv_engine *eng, cudaStream_t st) {
    if (eng->host_only) return QKV_OK;
    const size_t row_bytes = (size_t)eng->max_pages * sizeof(int32_t);
    const size_t per_block = qkv_engine::RING_BLOCK / row_bytes;
    int k = -1;
    uint8_t *host = nullptr;
    size_t used = per_block;
    for (int s = 0; s < eng->cfg.n_slots; s++) {
        qkv_engine::Slot &sl = eng->slots[s];
        if (!sl.dirty) continue;
        if (used == per_block) {
            if (k >= 0) {
                CK(eng, cudaEventRecord(eng->ring_ev[k], st));
                eng->ring_used[k] = true;
            }
            const qkv_status r = ring_block(eng, k, host);
            if (r != QKV_OK) return r;
            used = 0;
        }
        int32_t *row = reinterpret_cast<int32_t *>(host + used * row_bytes);
        std::fill(row, row + eng->max_pages, -1);
        std::copy(sl.pages.begin(), sl.pages.end(), row);
        CK(eng, cudaMemcpyAsync(eng->d_bt + (size_t)s * eng->max_pages, row, row_bytes, cudaMemcpyHostToDevice, st));
        used++;
        sl.dirty = false;
    }
    if (k >= 0) {
        CK(eng, cudaEventRecord(eng->ring_ev[k], st));
        eng->ring_used[k] = true;
    }
    return QKV_OK;
}

// Upload an arbitrary small int32 array (e.g. a snapshot's page list) to a device buffer.
static qkv_status upload_i32(qkv_engine *eng, const std::vector<int32_t> &v, int32_t *dst, cudaStream_t st) {
    size_t off = 0;
    while (off < v.size()) {
        int k = 0;
        uint8_t *host = nullptr;
        const qkv_status r = ring_block(eng, k, host);
        if (r != QKV_OK) return r;
        const size_t n = std::min(v.size() - off, qkv_engine::RING_BLOCK / sizeof(int32_t));
        memcpy(host, v.data() + off, n * sizeof(int32_t));
        CK(eng, cudaMemcpyAsync(dst + off, host, n * sizeof(int32_t), cudaMemcpyHostToDevice, st));
        CK(eng, cudaEventRecord(eng->ring_ev[k], st));
        eng->ring_used[k] = true;
        off += n;
    }
    return QKV_OK;
}

// Make positions [pos, pos+n) of a slot writable: allocate missing pages and copy shared ones
// (all layers of the page) before the caller's write.  All or nothing.
static qkv_status reserve(qkv_engine *eng, int32_t slot, int32_t pos, int32_t n, cudaStream_t st) {
    qkv_engine::Slot &sl = eng->slots[slot];
    const int32_t first = pos / PAGE_TOK, last = (pos + n - 1) / PAGE_TOK;
    if (last >= eng->max_pages) return fail(eng, QKV_ERR_STATE, "context exhausted: position %d >= n_ctx %d", pos + n - 1, eng->cfg.n_ctx);
    size_t need = 0;
    for (int32_t pi = first; pi <= last; pi++)
        if (pi >= (int32_t)sl.pages.size() || eng->refcnt[sl.pages[pi]] > 1) need++;
    if (need > eng->free_pages.size())
        return fail(eng, QKV_ERR_NO_MEMORY, "page pool exhausted: need %zu pages, %zu free", need, eng->free_pages.size());
    std::vector<CopyDesc> cow;
    for (int32_t pi = first; pi <= last; pi++) {
        if (pi >= (int32_t)sl.pages.size()) {
            sl.pages.push_back(page_alloc(eng));
            sl.dirty = true;
        } else if (eng->refcnt[sl.pages[pi]] > 1) {
            const int32_t old = sl.pages[pi], fresh = page_alloc(eng);
            for (int l = 0; l < eng->cfg.n_layer && !eng->host_only; l++)
                cow.push_back(CopyDesc{eng->pools[l] + (int64_t)old * eng->page_bytes,
                                       eng->pools[l] + (int64_t)fresh * eng->page_bytes, eng->page_bytes});
            for (size_t l = 0; l < eng->idx_pools.size() && !eng->host_only; l++)
                cow.push_back(CopyDesc{eng->idx_pools[l] + (int64_t)old * IDX_PAGE_BYTES,
                                       eng->idx_pools[l] + (int64_t)fresh * IDX_PAGE_BYTES, IDX_PAGE_BYTES});
            page_unref(eng, old);
            sl.pages[pi] = fresh;
            sl.dirty = true;
        }
    }
    if (!cow.empty() && !eng->host_only) CK(eng, launch_copy_batch(cow.data(), (int)cow.size(), eng->num_sms, st));
    return QKV_OK;
}

// ------------------------------------------------------------------------------ create/destroy
extern "C" const char *qkv_status_string(qkv_status st) {
    switch (st) {
        case QKV_OK: return "ok";
        case QKV_ERR_INVALID: return "invalid argument";
        case QKV_ERR_NO_MEMORY: return "out of memory";
        case QKV_ERR_CUDA: return "CUDA error";
        case QKV_ERR_STATE: return "invalid state";
        case QKV_ERR_MISMATCH: return "layout mismatch";
        case QKV_ERR_DEVICE: return "device-side error";
        case QKV_ERR_UNSUPPORTED: return "unsupported";
    }
    return "unknown status";
}

extern "C" const char *qkv_last_error(const qkv_engine *eng) { return eng ? eng->err.c_str() : "null engine"; }

static void free_device(qkv_engine *eng) {
    if (eng->host_only) return;
    for (uint8_t *p : eng->pools) cudaFree(p);
    eng->pools.clear();
    cudaFree(eng->d_bt);
    cudaFree(eng->d_rec);
    cudaFree(eng->d_rb);
    cudaFree(eng->d_summary);
    cudaFree(eng->d_sel_scores);
    cudaFree(eng->d_partial);
    cudaFree(eng->d_status);
    cudaFree(eng->d_pf_q);
    cudaFree(eng->d_pf_partial);
    cudaFree(eng->d_pf_plan);
    for (uint8_t *p : eng->idx_pools) cudaFree(p);
    eng->idx_pools.clear();
    cudaFree(eng->d_rope);
    cudaFree(eng->d_knorm);
    cudaFree(eng->d_iscore);
    cudaFree(eng->d_isel);
    cudaFree(eng->d_inout);
    cudaFree(eng->d_psel);
    cudaFree(eng->d_pnout);
    cudaFree(eng->d_pbits);
    if (eng->ring) cudaFreeHost(eng->ring);
    for (auto &ev : eng->ring_ev)
        if (ev) cudaEventDestroy(ev);
}

template <class T>
static qkv_status dalloc(qkv_engine *eng, T *&ptr, size_t bytes, const char *what) {
    if (bytes == 0) return QKV_OK;
    void *p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(eng, QKV_ERR_NO_MEMORY, "cudaMalloc(%s, %.3f GB): %s", what, bytes / 1e9, cudaGetErrorString(e));
    }
    ptr = static_cast<T *>(p);
    eng->device_bytes += bytes;
    return QKV_OK;
}

extern "C" qkv_status qkv_create(const qkv_config *cfg, int device, qkv_engine **out) {
    if (!cfg || !out) return QKV_ERR_INVALID;
    *out = nullptr;
    const qkv_config &c = *cfg;
    if (c.n_layer < 1 || c.n_head < 1 || c.n_head_kv < 1 || c.n_head % c.n_head_kv || c.head_dim != HD ||
        c.n_ctx < 1 || c.n_slots < 1 || c.n_pages < 0 || c.rec_n_layer < 0 || c.n_rollback < 0 || c.n_rollback > 4 ||
        (c.select_block != 0 && c.select_block != TILE_TOK) || c.n_head_kv > 8 || c.n_head / c.n_head_kv > 16 ||
        c.attn_interval < 0 || (c.attn_interval > 0 && (int64_t)c.n_layer * c.attn_interval != c.n_layer + c.rec_n_layer))
        return QKV_ERR_INVALID;
    if (c.rec_n_layer > 0 && (c.rec_head_dim < 1 || c.rec_n_head < 1 || c.conv_channels < 1 || c.conv_hist < 1))
        return QKV_ERR_INVALID;
    qkv_engine *eng = new (std::nothrow) qkv_engine;
    if (!eng) return QKV_ERR_NO_MEMORY;
    eng->cfg       = c;
    eng->device    = device;
    eng->host_only = device < 0;
    eng->max_pages = (c.n_ctx + PAGE_TOK - 1) / PAGE_TOK;
    eng->n_pages   = c.n_pages > 0 ? c.n_pages : c.n_slots * eng->max_pages;
    eng->page_bytes = (int64_t)c.n_head_kv * TILES_PER_PAGE * TILE_BYTES;
    eng->rs_bytes   = (int64_t)c.rec_head_dim * c.rec_head_dim * c.rec_n_head * 4;
    eng->conv_bytes = (int64_t)c.conv_hist * c.conv_channels * 4;
    eng->rs_bytes   = (eng->rs_bytes + 255) / 256 * 256;
    eng->conv_bytes = (eng->conv_bytes + 255) / 256 * 256;
    eng->rec_layer_bytes = c.rec_n_layer > 0 ? eng->rs_bytes + eng->conv_bytes : 0;
    eng->rec_slot_bytes  = eng->rec_layer_bytes * c.rec_n_layer;
    eng->max_blocks = c.select_block ? (c.n_ctx + TILE_TOK - 1) / TILE_TOK : 0;
    eng->max_nq     = 4 * (c.n_head / c.n_head_kv);
    eng->refcnt.assign(eng->n_pages, 0);
    eng->free_pages.resize(eng->n_pages);
    for (int32_t i = 0; i < eng->n_pages; i++) eng->free_pages[i] = eng->n_pages - 1 - i;
    eng->slots.resize(c.n_slots);
    eng->sum_valid.assign((size_t)c.n_slots * c.n_layer, 0);
    if (!eng->host_only) {
        qkv_status r = QKV_OK;
        cudaError_t e = cudaSetDevice(device);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&eng->num_sms, cudaDevAttrMultiProcessorCount, device);
        if (e != cudaSuccess) {
            r = fail(eng, QKV_ERR_CUDA, "device %d: %s", device, cudaGetErrorString(e));
        }
        eng->pools.assign(c.n_layer, nullptr);
        for (int l = 0; l < c.n_layer && r == QKV_OK; l++)
            r = dalloc(eng, eng->pools[l], (size_t)eng->n_pages * eng->page_bytes, "page pool");
        if (r == QKV_OK) r = dalloc(eng, eng->d_bt, (size_t)c.n_slots * eng->max_pages * 4, "block table");
        if (r == QKV_OK) r = dalloc(eng, eng->d_rec, (size_t)c.n_slots * eng->rec_slot_bytes, "recurrent state");
        if (r == QKV_OK) r = dalloc(eng, eng->d_rb, (size_t)c.n_slots * c.n_rollback * eng->rec_slot_bytes, "rollback state");
        if (r == QKV_OK)
            r = dalloc(eng, eng->d_summary, (size_t)c.n_layer * c.n_slots * c.n_head_kv * eng->max_blocks * HD * 2,
                       "block summaries");
        if (r == QKV_OK && eng->max_blocks > 0)
            r = dalloc(eng, eng->d_sel_scores, (size_t)MAX_SEQ * c.n_head_kv * eng->max_blocks * sizeof(float),
                       "block scores");
        if (r == QKV_OK) {
            // one record per unit: at most one wave of co-resident CTAs plus one unit per pair of
            // a launch, for the widest query group of each kernel instance
            size_t need = 0;
            for (int nq = 8; nq <= std::min((eng->max_nq + 7) & ~7, decode_max_nq()); nq += 8) {
                const int ctas = decode_max_ctas(nq);
                const size_t max_units = (size_t)(ctas > 0 ? ctas : eng->num_sms * 8) + (size_t)MAX_SEQ * c.n_head_kv;
                need = std::max(need, max_units * (size_t)partial_stride(nq) * sizeof(float));
            }
            eng->partial_bytes = need;
            r = dalloc(eng, eng->d_partial, eng->partial_bytes, "split-K partials");
        }
        if (r == QKV_OK) r = dalloc(eng, eng->d_status, 256, "status");
        if (r == QKV_OK) {
            e = cudaMallocHost(&eng->ring, (size_t)qkv_engine::RING_N * qkv_engine::RING_BLOCK);
            for (int i = 0; i < qkv_engine::RING_N && e == cudaSuccess; i++)
                e = cudaEventCreateWithFlags(&eng->ring_ev[i], cudaEventDisableTiming);
            if (e != cudaSuccess) r = fail(eng, QKV_ERR_CUDA, "pinned upload ring: %s", cudaGetErrorString(e));
        }
        if (r == QKV_OK) {
            e = cudaMemset(eng->d_bt, 0xff, (size_t)c.n_slots * eng->max_pages * 4);
            if (e == cudaSuccess && eng->d_rec) e = cudaMemset(eng->d_rec, 0, (size_t)c.n_slots * eng->rec_slot_bytes);
            if (e == cudaSuccess) e = cudaMemset(eng->d_status, 0, 256);
            if (e == cudaSuccess) e = cudaDeviceSynchronize();
            if (e != cudaSuccess) r = fail(eng, QKV_ERR_CUDA, "init: %s", cudaGetErrorString(e));
        }
        if (r != QKV_OK) {
            free_device(eng);
            delete eng;
            return r;
        }
    }
    *out = eng;
    return QKV_OK;
}

extern "C" void qkv_destroy(qkv_engine *eng) {
    if (!eng) return;
    if (!eng->host_only) {
        cudaSetDevice(eng->device);
        cudaDeviceSynchronize();
        for (qkv_snapshot *s : eng->snaps) cudaFree(s->rec);
    }
    for (qkv_snapshot *s : eng->snaps) delete s;
    free_device(eng);
    delete eng;
}

extern "C" qkv_status qkv_bytes(const qkv_engine *eng, size_t *device_bytes) {
    if (!eng || !device_bytes) return QKV_ERR_INVALID;
    *device_bytes = eng->device_bytes;
    return QKV_OK;
}

extern "C" qkv_status qkv_summary(const qkv_engine *eng, char *buf, size_t cap) {
    if (!eng || !buf || cap == 0) return QKV_ERR_INVALID;
    const double kv = (double)eng->n_pages * eng->page_bytes * eng->cfg.n_layer;
    snprintf(buf, cap,
             "qkv engine on %s: %d attention layers, %d pages x %d tokens (%.3f GB q8_0 KV), %d slots, "
             "recurrent %.1f MB/slot, %.3f GB on the device",
             eng->host_only ? "host only" : "cuda", eng->cfg.n_layer, eng->n_pages, PAGE_TOK, kv / 1e9,
             eng->cfg.n_slots, eng->rec_slot_bytes / 1e6, eng->device_bytes / 1e9);
    return QKV_OK;
}

// ---------------------------------------------------------------------------------- slots
extern "C" qkv_status qkv_seq_alloc(qkv_engine *eng, int32_t slot) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot, false);
    if (r != QKV_OK) return r;
    qkv_engine::Slot &sl = eng->slots[slot];
    if (sl.active) return fail(eng, QKV_ERR_STATE, "slot %d is already allocated", slot);
    sl.active = true;
    sl.n_past = 0;
    sl.rb_depth = 0;
    sl.pages.clear();
    sl.dirty = true;
    invalidate_summaries(eng, slot, 0);
    return QKV_OK;
}

extern "C" qkv_status qkv_seq_free(qkv_engine *eng, int32_t slot) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    qkv_engine::Slot &sl = eng->slots[slot];
    release_pages(eng, sl.pages);
    sl.active = false;
    sl.n_past = 0;
    sl.rb_depth = 0;
    sl.dirty = true;
    return QKV_OK;
}

extern "C" qkv_status qkv_seq_reset(qkv_engine *eng, int32_t slot, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    qkv_engine::Slot &sl = eng->slots[slot];
    release_pages(eng, sl.pages);
    sl.n_past = 0;
    sl.rb_depth = 0;
    sl.dirty = true;
    invalidate_summaries(eng, slot, 0);
    if (eng->host_only || eng->rec_slot_bytes == 0) return QKV_OK;
    if ((r = use_device(eng)) != QKV_OK) return r;
    CK(eng, cudaMemsetAsync(eng->d_rec + (size_t)slot * eng->rec_slot_bytes, 0, eng->rec_slot_bytes, S(stream)));
    return QKV_OK;
}

extern "C" qkv_status qkv_seq_length(const qkv_engine *eng, int32_t slot, int32_t *n_past) {
    if (!eng || !n_past || slot < 0 || slot >= eng->cfg.n_slots) return QKV_ERR_INVALID;
    *n_past = eng->slots[slot].n_past;
    return QKV_OK;
}

extern "C" qkv_status qkv_seq_reserve(qkv_engine *eng, int32_t slot, int32_t n_tokens, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    if (n_tokens < 0 || n_tokens > eng->cfg.n_ctx) return fail(eng, QKV_ERR_INVALID, "reserve %d of n_ctx %d", n_tokens, eng->cfg.n_ctx);
    const int32_t from = eng->slots[slot].n_past;
    if (n_tokens <= from) return QKV_OK;
    if (!eng->host_only && (r = use_device(eng)) != QKV_OK) return r;
    if ((r = reserve(eng, slot, from, n_tokens - from, S(stream))) != QKV_OK) return r;
    return flush_tables(eng, S(stream));
}

extern "C" qkv_status qkv_seq_pages(const qkv_engine *eng, int32_t slot, int32_t *pages, int32_t cap, int32_t *n) {
    if (!eng || !n || slot < 0 || slot >= eng->cfg.n_slots || (cap > 0 && !pages)) return QKV_ERR_INVALID;
    const auto &pg = eng->slots[slot].pages;
    *n = (int32_t)pg.size();
    for (int32_t i = 0; i < cap && i < (int32_t)pg.size(); i++) pages[i] = pg[i];
    return QKV_OK;
}

extern "C" qkv_status qkv_page_refcount(const qkv_engine *eng, int32_t page, int32_t *refcount) {
    if (!eng || !refcount || page < 0 || page >= eng->n_pages) return QKV_ERR_INVALID;
    *refcount = eng->refcnt[page];
    return QKV_OK;
}

extern "C" qkv_status qkv_pages_free(const qkv_engine *eng, int32_t *n_free) {
    if (!eng || !n_free) return QKV_ERR_INVALID;
    *n_free = (int32_t)eng->free_pages.size();
    return QKV_OK;
}

// ------------------------------------------------------------------------------------ append
extern "C" qkv_status qkv_append(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, const float *K,
                                 const float *V, int32_t n_rows, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    qkv_engine::Slot &sl = eng->slots[slot];
    if (n_rows < 1 || !K || !V) return fail(eng, QKV_ERR_INVALID, "append: %d rows, K=%p V=%p", n_rows, (const void *)K, (const void *)V);
    if (pos < 0 || pos > sl.n_past) return fail(eng, QKV_ERR_INVALID, "append at %d: slot %d holds %d positions", pos, slot, sl.n_past);
    if ((int64_t)pos + n_rows > eng->cfg.n_ctx) return fail(eng, QKV_ERR_STATE, "context exhausted: %d + %d > n_ctx %d", pos, n_rows, eng->cfg.n_ctx);
    if (!eng->host_only && (r = use_device(eng)) != QKV_OK) return r;
    if ((r = reserve(eng, slot, pos, n_rows, S(stream))) != QKV_OK) return r;
    if (eng->host_only) {
        sl.n_past = std::max(sl.n_past, pos + n_rows);
        invalidate_summaries(eng, slot, pos);
        return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: pages reserved, no rows written");
    }
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    CK(eng, launch_append(pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages), pos, K, V, n_rows, S(stream)));
    sl.n_past = std::max(sl.n_past, pos + n_rows);
    invalidate_summaries(eng, slot, pos);
    return QKV_OK;
}

extern "C" qkv_status qkv_project_append(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, const float *x,
                                         int32_t n_embd, int32_t T, const uint16_t *Wq, const uint16_t *Wk,
                                         const uint16_t *Wv, const float *q_norm, const float *k_norm, float rms_eps,
                                         int32_t rope_dim, float rope_freq_base, float *Q_out, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    auto aligned = [](const void *ptr) { return ((uintptr_t)ptr & 15) == 0; };
    if (!x || !Wk || !Wv || !k_norm || (Wq && (!q_norm || !Q_out)) || T < 1 || T > PJ_MAX_T || n_embd < 256 ||
        n_embd % 256 || (size_t)T * n_embd * 4 > 48 * 1024 || rope_dim < 0 || rope_dim % 2 || rope_dim / 2 > PJ_MAX_HALF ||
        !(rope_freq_base > 0.f) || !(rms_eps >= 0.f) || !aligned(x) || !aligned(Wk) || !aligned(Wv) ||
        (Wq && !aligned(Wq)))
        return fail(eng, QKV_ERR_INVALID, "project_append: T %d (1..%d), n_embd %d (multiple of 256, T * n_embd <= 12288), rope_dim %d, "
                    "null or unaligned pointer", T, PJ_MAX_T, n_embd, rope_dim);
    qkv_engine::Slot &sl = eng->slots[slot];
    if (pos < 0 || pos > sl.n_past || (int64_t)pos + T > eng->cfg.n_ctx)
        return fail(eng, QKV_ERR_INVALID, "project_append at %d: slot %d holds %d, n_ctx %d", pos, slot, sl.n_past, eng->cfg.n_ctx);
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    if ((r = reserve(eng, slot, pos, T, st)) != QKV_OK) return r;
    if ((r = flush_tables(eng, st)) != QKV_OK) return r;
    ProjectParams p;
    memset(&p, 0, sizeof p);
    p.pr = pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages);
    p.x = x;
    p.Wq = Wq;
    p.Wk = Wk;
    p.Wv = Wv;
    p.q_norm = q_norm;
    p.k_norm = k_norm;
    p.Q_out = Q_out;
    p.n_embd = n_embd;
    p.T = T;
    p.pos = pos;
    p.n_head = eng->cfg.n_head;
    p.n_head_kv = eng->cfg.n_head_kv;
    p.rope_half = rope_dim / 2;
    p.eps = rms_eps;
    // angles as ggml's CPU rope cache builds them: theta_0 = p, one fp32 multiplication per pair
    const float theta_scale = powf(rope_freq_base, -2.0f / (float)std::max(rope_dim, 1));
    for (int t = 0; t < T; t++) {
        float th = (float)(pos + t);
        for (int i = 0; i < rope_dim / 2; i++) {
            p.cs[t][i] = make_float2(cosf(th), sinf(th));
            th *= theta_scale;
        }
    }
    CK(eng, launch_project(p, st));
    sl.n_past = std::max(sl.n_past, pos + T);
    invalidate_summaries(eng, slot, pos);
    return QKV_OK;
}

// ------------------------------------------------------------------------------------ decode
// Plan one launch of kernel C for sequences [base, base+ns): every pair (sequence, KV head) is
// cut into units in proportion to its tiles (plan_decode) so that about a wave of CTAs carries
// equal work.
// Where kernel C reads from: by default the layer's pool through the engine's block table; the
// indexer path points it at dense scratch copies of the kept cells instead.
// QSA mode of a decode launch: sequence i attends to its kept 4-cell blocks blocks[i][0 .. n_out[i])
// (device arrays, ascending) of its slot; pos0[i] + 1 is the number of kept cells and vpos[i] the
// query's position.
struct DecodeGroups {
    const int32_t *blocks, *n_out;
    int32_t        stride;
    const int32_t *vpos;   // host [ns]
};

static qkv_status decode_launch(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0, int ns,
                                const float *Q, int32_t T, float scale, const int32_t *sel, int32_t n_sel,
                                const float *Knew, const float *Vnew, float *out, cudaStream_t st,
                                const DecodeGroups *grp = nullptr) {
    const int H = eng->cfg.n_head_kv, G = eng->cfg.n_head / H;
    DecodeParams P;
    memset(&P, 0, sizeof P);
    P.pool = eng->pools[layer];
    P.block_table = eng->d_bt;
    P.Q = Q;
    P.out = out;
    P.partial = eng->d_partial;
    P.sel = sel;
    P.Knew = Knew;
    P.Vnew = Vnew;
    P.status = eng->d_status;
    P.page_bytes = eng->page_bytes;
    P.n_pages = eng->n_pages;
    P.max_pages = eng->max_pages;
    P.n_head = eng->cfg.n_head;
    P.n_head_kv = H;
    P.G = G;
    P.T = T;
    P.nq = T * G;
    P.n_seq = ns;
    P.n_sel = n_sel;
    P.scale = scale;
    P.wait_ns = eng->wait_ns;
    P.withhold_unit = eng->withhold_unit;
    eng->withhold_unit = -1;   // one launch only
    if (grp) {
        P.grp = grp->blocks;
        P.grp_n = grp->n_out;
        P.grp_stride = grp->stride;
    }
    std::vector<int32_t> tiles(ns);
    for (int i = 0; i < ns; i++) tiles[i] = sel ? n_sel : (pos0[i] + T + TILE_TOK - 1) / TILE_TOK;
    const int max_ctas = decode_max_ctas(T * G);
    const int64_t target = max_ctas > 0 ? max_ctas : (int64_t)eng->num_sms * 2;
    plan_decode(P, slots, pos0, tiles.data(), ns, target, decode_merge_max_units(),
                (int64_t)(eng->partial_bytes / (partial_stride(P.nq) * sizeof(float))));
    if (grp)
        for (int j = 0; j < ns; j++) P.seq_vpos[j] = grp->vpos[P.seq_idx[j]];
    if ((size_t)P.n_units * partial_stride(P.nq) * sizeof(float) > eng->partial_bytes)
        return fail(eng, QKV_ERR_NO_MEMORY, "decode: split-K scratch too small for %d units", P.n_units);
    CK(eng, launch_decode(P, st));
    return QKV_OK;
}

static qkv_status decode_common(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                int32_t n_seq, const float *Q, int32_t T, float scale, const int32_t *sel_blocks,
                                int32_t n_sel, const float *Knew, const float *Vnew, float *out, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK) return r;
    if (!slots || !pos0 || n_seq < 1 || !Q || !out || T < 1 || T > 4)
        return fail(eng, QKV_ERR_INVALID, "decode: n_seq %d, T %d (1..4), null pointer", n_seq, T);
    if (sel_blocks && n_sel < 1) return fail(eng, QKV_ERR_INVALID, "decode: n_sel %d with a selection", n_sel);
    const bool fused = Knew != nullptr;
    if (fused && (!Vnew || sel_blocks)) return fail(eng, QKV_ERR_INVALID, "fused append needs K and V and dense attention");
    const int G = eng->cfg.n_head / eng->cfg.n_head_kv;
    if (T * G > decode_max_nq()) return fail(eng, QKV_ERR_UNSUPPORTED, "decode: %d query rows per KV head (max %d)", T * G, decode_max_nq());
    for (int i = 0; i < n_seq; i++) {
        if ((r = check_slot(eng, slots[i])) != QKV_OK) return r;
        for (int j = 0; j < i; j++)
            if (fused && slots[j] == slots[i]) return fail(eng, QKV_ERR_INVALID, "fused append: slot %d twice", slots[i]);
        const int32_t n_past = eng->slots[slots[i]].n_past;
        if (fused) {
            if (pos0[i] < 0 || pos0[i] > n_past || (int64_t)pos0[i] + T > eng->cfg.n_ctx)
                return fail(eng, QKV_ERR_INVALID, "fused append at %d: slot %d holds %d (n_ctx %d)", pos0[i], slots[i], n_past, eng->cfg.n_ctx);
        } else if (pos0[i] < 0 || pos0[i] + T > n_past) {
            return fail(eng, QKV_ERR_INVALID, "decode: sequence %d queries positions %d..%d but slot %d holds %d", i, pos0[i],
                        pos0[i] + T - 1, slots[i], n_past);
        }
    }
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    if (fused) {
        // reserve every sequence's rows first: a failure leaves no sequence half-appended
        size_t need = 0;
        for (int i = 0; i < n_seq; i++) {
            const qkv_engine::Slot &sl = eng->slots[slots[i]];
            for (int32_t pi = pos0[i] / PAGE_TOK; pi <= (pos0[i] + T - 1) / PAGE_TOK; pi++)
                if (pi >= (int32_t)sl.pages.size() || eng->refcnt[sl.pages[pi]] > 1) need++;
        }
        if (need > eng->free_pages.size())
            return fail(eng, QKV_ERR_NO_MEMORY, "page pool exhausted: need %zu pages, %zu free", need, eng->free_pages.size());
        for (int i = 0; i < n_seq; i++)
            if ((r = reserve(eng, slots[i], pos0[i], T, st)) != QKV_OK) return r;
    }
    if ((r = flush_tables(eng, st)) != QKV_OK) return r;
    const int H = eng->cfg.n_head_kv;
    const size_t qrow = (size_t)T * eng->cfg.n_head * HD, krow = (size_t)T * H * HD;
    for (int base = 0; base < n_seq; base += MAX_SEQ) {
        const int ns = std::min(MAX_SEQ, n_seq - base);
        if ((r = decode_launch(eng, layer, slots + base, pos0 + base, ns, Q + base * qrow, T, scale,
                               sel_blocks ? sel_blocks + (size_t)base * H * n_sel : nullptr, n_sel,
                               fused ? Knew + base * krow : nullptr, fused ? Vnew + base * krow : nullptr,
                               out + base * qrow, st)) != QKV_OK)
            return r;
    }
    if (fused)
        for (int i = 0; i < n_seq; i++) {
            qkv_engine::Slot &sl = eng->slots[slots[i]];
            sl.n_past = std::max(sl.n_past, pos0[i] + T);
            invalidate_summaries(eng, slots[i], pos0[i]);
        }
    return QKV_OK;
}

extern "C" qkv_status qkv_attn_decode(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                      int32_t n_seq, const float *Q, int32_t T, float scale,
                                      const int32_t *sel_blocks, int32_t n_sel, float *out, void *stream) {
    return decode_common(eng, layer, slots, pos0, n_seq, Q, T, scale, sel_blocks, n_sel, nullptr, nullptr, out, stream);
}

extern "C" qkv_status qkv_append_attn_decode(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                             int32_t n_seq, const float *K, const float *V, const float *Q, int32_t T,
                                             float scale, float *out, void *stream) {
    if (!K || !V) return eng ? fail(eng, QKV_ERR_INVALID, "fused append: null K or V") : QKV_ERR_INVALID;
    return decode_common(eng, layer, slots, pos0, n_seq, Q, T, scale, nullptr, 0, K, V, out, stream);
}

// ---------------------------------------------------------------------- QSA lightning indexer
extern "C" qkv_status qkv_indexer_enable(qkv_engine *eng, const qkv_indexer_config *cfg, const float *k_norm) {
    if (!eng || !cfg) return QKV_ERR_INVALID;
    const qkv_indexer_config &c = *cfg;
    if (eng->idx_on) return fail(eng, QKV_ERR_STATE, "indexer already enabled");
    if (c.n_head < 1 || c.n_head > IDX_MAX_HEAD || c.key_len != IDX_KEY || c.ratio != IDX_R || c.top_k < 1 ||
        c.rope_dim < 0 || c.rope_dim % 8 || c.rope_dim > IDX_KEY || !(c.rope_freq_base > 0.f) || !(c.rms_eps >= 0.f))
        return fail(eng, QKV_ERR_INVALID,
                    "indexer: n_head %d (1..%d), key_len %d (%d), ratio %d (%d), top_k %d, rope_dim %d (multiple of 8, <= %d)",
                    c.n_head, IDX_MAX_HEAD, c.key_len, IDX_KEY, c.ratio, IDX_R, c.top_k, c.rope_dim, IDX_KEY);
    eng->icfg = c;
    eng->k_blocks = (c.top_k + c.ratio - 1 + c.ratio - 1) / c.ratio;   // ceil(width / ratio), engine.cpp:687
    eng->idx_max_blk = (eng->cfg.n_ctx + IDX_R - 1) / IDX_R;
    if (eng->host_only) {
        eng->idx_on = true;
        return QKV_OK;
    }
    qkv_status r = use_device(eng);
    if (r != QKV_OK) return r;
    eng->idx_pools.assign(eng->cfg.n_layer, nullptr);
    for (int l = 0; l < eng->cfg.n_layer && r == QKV_OK; l++) {
        r = dalloc(eng, eng->idx_pools[l], (size_t)eng->n_pages * IDX_PAGE_BYTES, "indexer pool");
        if (r == QKV_OK) CK(eng, cudaMemset(eng->idx_pools[l], 0, (size_t)eng->n_pages * IDX_PAGE_BYTES));
    }
    // rope table of the block positions p = 4b: theta_0 = p, theta_{i+1} = theta_i * freq_base^(-2/rope_dim)
    // in fp32, as ggml's CPU rope cache is built (one multiplication per pair)
    const int half = c.rope_dim / 2;
    std::vector<float2> tab((size_t)eng->idx_max_blk * std::max(half, 1));
    const float theta_scale = powf(c.rope_freq_base, -2.0f / (float)std::max(c.rope_dim, 1));
    for (int32_t b = 0; b < eng->idx_max_blk; b++) {
        float th = (float)(b * IDX_R);
        for (int i = 0; i < half; i++) {
            tab[(size_t)b * half + i] = make_float2(cosf(th), sinf(th));
            th *= theta_scale;
        }
    }
    std::vector<float> w((size_t)eng->cfg.n_layer * IDX_KEY, 1.0f);
    if (k_norm) memcpy(w.data(), k_norm, w.size() * sizeof(float));
    if (r == QKV_OK) r = dalloc(eng, eng->d_rope, tab.size() * sizeof(float2), "indexer rope table");
    if (r == QKV_OK) r = dalloc(eng, eng->d_knorm, w.size() * sizeof(float), "indexer norm weights");
    if (r != QKV_OK) return r;
    CK(eng, cudaMemcpy(eng->d_rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
    CK(eng, cudaMemcpy(eng->d_knorm, w.data(), w.size() * sizeof(float), cudaMemcpyHostToDevice));
    eng->idx_on = true;
    return QKV_OK;
}

static qkv_status idx_check(qkv_engine *eng, int32_t layer) {
    if (!eng) return QKV_ERR_INVALID;
    if (!eng->idx_on) return fail(eng, QKV_ERR_STATE, "indexer not enabled (qkv_indexer_enable)");
    return check_layer(eng, layer);
}

extern "C" qkv_status qkv_idx_append(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, const float *k_raw,
                                     int32_t n_rows, void *stream) {
    qkv_status r;
    if ((r = idx_check(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    if (n_rows < 1 || !k_raw || ((uintptr_t)k_raw & 15))
        return fail(eng, QKV_ERR_INVALID, "idx_append: %d rows, keys %p (16-byte aligned)", n_rows, (const void *)k_raw);
    const qkv_engine::Slot &sl = eng->slots[slot];
    if (pos < 0 || pos > sl.n_past || (int64_t)pos + n_rows > eng->cfg.n_ctx)
        return fail(eng, QKV_ERR_INVALID, "idx_append at %d (+%d): slot %d holds %d, n_ctx %d", pos, n_rows, slot, sl.n_past,
                    eng->cfg.n_ctx);
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    if ((r = reserve(eng, slot, pos, n_rows, st)) != QKV_OK) return r;
    if ((r = flush_tables(eng, st)) != QKV_OK) return r;
    IdxAppendParams p;
    p.pool = eng->idx_pools[layer];
    p.bt = eng->d_bt + (size_t)slot * eng->max_pages;
    p.k_raw = k_raw;
    p.norm_w = eng->d_knorm + (size_t)layer * IDX_KEY;
    p.rope = eng->d_rope;
    p.status = eng->d_status;
    p.n_pages = eng->n_pages;
    p.max_pages = eng->max_pages;
    p.pos = pos;
    p.n_rows = n_rows;
    p.rope_half = eng->icfg.rope_dim / 2;
    p.eps = eng->icfg.rms_eps;
    CK(eng, launch_idx_append(p, st));
    return QKV_OK;
}

// Validate (sequence, token) entries: every position already appended to its slot.
static qkv_status idx_entries(qkv_engine *eng, const int32_t *slots, const int32_t *pos0, int32_t n_seq, int32_t T,
                              const void *q) {
    if (!slots || !pos0 || !q || n_seq < 1 || T < 1 || T > 4)
        return fail(eng, QKV_ERR_INVALID, "indexer: n_seq %d, T %d (1..4), null pointer", n_seq, T);
    for (int i = 0; i < n_seq; i++) {
        qkv_status r = check_slot(eng, slots[i]);
        if (r != QKV_OK) return r;
        if (pos0[i] < 0 || pos0[i] + T > eng->slots[slots[i]].n_past)
            return fail(eng, QKV_ERR_INVALID, "indexer: sequence %d positions %d..%d but slot %d holds %d", i, pos0[i],
                        pos0[i] + T - 1, slots[i], eng->slots[slots[i]].n_past);
    }
    return QKV_OK;
}

// Scores + top-k for entries [v0, v0 + nv) of n_seq x T (entry v = i * T + t).
static qkv_status idx_select_chunk(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0, int32_t T,
                                   int32_t v0, int32_t nv, const float *q_idx, int32_t *blocks, int32_t *n_out,
                                   float *scores, int32_t score_stride, cudaStream_t st) {
    IdxSelectParams p;
    memset(&p, 0, sizeof p);
    p.pool = eng->idx_pools[layer];
    p.bt = eng->d_bt;
    p.q = q_idx + (size_t)v0 * eng->icfg.n_head * IDX_KEY;
    p.scores = scores;
    p.blocks = blocks;
    p.n_out = n_out;
    p.status = eng->d_status;
    p.n_v = nv;
    p.T = T;
    p.n_head = eng->icfg.n_head;
    p.k_blocks = eng->k_blocks;
    p.score_stride = score_stride;
    p.n_pages = eng->n_pages;
    p.max_pages = eng->max_pages;
    int32_t max_whole = 0;
    for (int k = 0; k < nv; k++) {
        const int v = v0 + k;
        p.v_slot[k] = slots[v / T];
        p.v_pos[k] = pos0[v / T] + v % T;
        max_whole = std::max(max_whole, (p.v_pos[k] + 1) / IDX_R);
    }
    CK(eng, launch_idx_select(p, max_whole, st));
    return QKV_OK;
}

static qkv_status idx_scratch(qkv_engine *eng, int32_t nv) {
    if (nv <= eng->iscratch_v) return QKV_OK;
    cudaFree(eng->d_iscore);
    cudaFree(eng->d_isel);
    cudaFree(eng->d_inout);
    eng->d_iscore = nullptr;
    eng->d_isel = eng->d_inout = nullptr;
    eng->iscratch_v = 0;
    qkv_status r = dalloc(eng, eng->d_iscore, (size_t)nv * eng->idx_max_blk * sizeof(float), "indexer scores");
    if (r == QKV_OK) r = dalloc(eng, eng->d_isel, (size_t)nv * eng->k_blocks * sizeof(int32_t), "indexer blocks");
    if (r == QKV_OK) r = dalloc(eng, eng->d_inout, (size_t)nv * sizeof(int32_t), "indexer counts");
    if (r == QKV_OK) eng->iscratch_v = nv;
    return r;
}

extern "C" qkv_status qkv_idx_select(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                     int32_t n_seq, const float *q_idx, int32_t T, int32_t *blocks_out, int32_t *n_out_out,
                                     float *scores_out, void *stream) {
    qkv_status r;
    if ((r = idx_check(eng, layer)) != QKV_OK || (r = idx_entries(eng, slots, pos0, n_seq, T, q_idx)) != QKV_OK) return r;
    if (!blocks_out || !n_out_out) return fail(eng, QKV_ERR_INVALID, "idx_select: null output");
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    if ((r = flush_tables(eng, st)) != QKV_OK) return r;
    const int32_t n_v = n_seq * T;
    const int32_t step = IDX_MAX_VSEQ / T * T;   // whole sequences per launch
    if (!scores_out && (r = idx_scratch(eng, std::min(n_v, step))) != QKV_OK) return r;
    for (int32_t v0 = 0; v0 < n_v; v0 += step) {
        const int32_t nv = std::min(step, n_v - v0);
        float *sc = scores_out ? scores_out + (size_t)v0 * eng->idx_max_blk : eng->d_iscore;
        if ((r = idx_select_chunk(eng, layer, slots, pos0, T, v0, nv, q_idx, blocks_out + (size_t)v0 * eng->k_blocks,
                                  n_out_out + v0, sc, eng->idx_max_blk, st)) != QKV_OK)
            return r;
    }
    return QKV_OK;
}

extern "C" qkv_status qkv_attn_decode_qsa(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                          int32_t n_seq, const float *q_idx, const float *Q, int32_t T, float scale,
                                          float *out, void *stream) {
    qkv_status r;
    if ((r = idx_check(eng, layer)) != QKV_OK || (r = idx_entries(eng, slots, pos0, n_seq, T, q_idx)) != QKV_OK) return r;
    if (!Q || !out) return fail(eng, QKV_ERR_INVALID, "decode_qsa: null Q or out");
    if (eng->cfg.n_head / eng->cfg.n_head_kv > decode_max_nq())
        return fail(eng, QKV_ERR_UNSUPPORTED, "decode_qsa: %d query heads per KV head", eng->cfg.n_head / eng->cfg.n_head_kv);
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    if ((r = flush_tables(eng, st)) != QKV_OK) return r;
    // entries go through in chunks of MAX_SEQ (one selection and one decode launch each), reusing
    // the scratch; the decode reads each entry's kept blocks in place (QSA mode)
    if ((r = idx_scratch(eng, MAX_SEQ)) != QKV_OK) return r;
    const int32_t n_v = n_seq * T, K = eng->k_blocks;
    const size_t qrow = (size_t)eng->cfg.n_head * HD;
    const int32_t step = MAX_SEQ / T * T;   // whole sequences per launch
    for (int32_t v0 = 0; v0 < n_v; v0 += step) {
        const int32_t nv = std::min(step, n_v - v0);
        if ((r = idx_select_chunk(eng, layer, slots, pos0, T, v0, nv, q_idx, eng->d_isel, eng->d_inout, eng->d_iscore,
                                  eng->idx_max_blk, st)) != QKV_OK)
            return r;
        int32_t vslot[MAX_SEQ], vlast[MAX_SEQ], vpos[MAX_SEQ];
        for (int k = 0; k < nv; k++) {
            const int v = v0 + k;
            const int32_t p = pos0[v / T] + v % T, b_last = p / IDX_R, whole = (p + 1) / IDX_R;
            const int32_t tail = b_last >= whole ? 1 : 0;
            // kept cells: every block (cells 0 .. p), or k_blocks blocks with the tail's cells up
            // to p last
            const int32_t len = b_last + 1 <= K ? p + 1 : IDX_R * (K - tail) + (tail ? p - IDX_R * b_last + 1 : 0);
            vslot[k] = slots[v / T];
            vlast[k] = len - 1;
            vpos[k] = p;
        }
        const DecodeGroups grp{eng->d_isel, eng->d_inout, K, vpos};
        if ((r = decode_launch(eng, layer, vslot, vlast, nv, Q + (size_t)v0 * qrow, 1, scale, nullptr, 0, nullptr, nullptr,
                               out + (size_t)v0 * qrow, st, &grp)) != QKV_OK)
            return r;
    }
    return QKV_OK;
}

extern "C" qkv_status qkv_idx_read(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, int32_t n,
                                   uint16_t *keys_out, int32_t b0, int32_t n_blk, uint16_t *pooled_out, void *stream) {
    qkv_status r;
    if ((r = idx_check(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    const qkv_engine::Slot &sl = eng->slots[slot];
    const int64_t have = (int64_t)sl.pages.size() * PAGE_TOK;
    if ((keys_out && (pos < 0 || n < 0 || pos + (int64_t)n > have)) ||
        (pooled_out && (b0 < 0 || n_blk < 0 || (int64_t)(b0 + n_blk) * IDX_R > have)))
        return fail(eng, QKV_ERR_INVALID, "idx_read: positions %d+%d / blocks %d+%d outside the slot's %lld pages", pos, n, b0,
                    n_blk, (long long)sl.pages.size());
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    const uint8_t *pool = eng->idx_pools[layer];
    for (int32_t c = pos; keys_out && c < pos + n;) {   // runs within one page
        const int32_t run = std::min(pos + n - c, PAGE_TOK - (c & (PAGE_TOK - 1)));
        const uint8_t *src = pool + (int64_t)sl.pages[c / PAGE_TOK] * IDX_PAGE_BYTES + (int64_t)(c & (PAGE_TOK - 1)) * IDX_KEY * 2;
        CK(eng, cudaMemcpyAsync(keys_out + (size_t)(c - pos) * IDX_KEY, src, (size_t)run * IDX_KEY * 2, cudaMemcpyDeviceToDevice, st));
        c += run;
    }
    for (int32_t b = b0; pooled_out && b < b0 + n_blk;) {
        const int32_t run = std::min(b0 + n_blk - b, IDX_BPP - (b & (IDX_BPP - 1)));
        const uint8_t *src = pool + (int64_t)sl.pages[b / IDX_BPP] * IDX_PAGE_BYTES + IDX_RAW_BYTES +
                             (int64_t)(b & (IDX_BPP - 1)) * IDX_KEY * 2;
        CK(eng, cudaMemcpyAsync(pooled_out + (size_t)(b - b0) * IDX_KEY, src, (size_t)run * IDX_KEY * 2, cudaMemcpyDeviceToDevice, st));
        b += run;
    }
    return QKV_OK;
}

// --------------------------------------------------------------------------------- selection
static qkv_status refresh_summaries(qkv_engine *eng, int32_t layer, int32_t slot, int32_t nb_whole, cudaStream_t st) {
    int32_t &v = eng->sum_valid[(size_t)slot * eng->cfg.n_layer + layer];
    if (v >= nb_whole) return QKV_OK;
    uint16_t *sum = eng->d_summary + ((size_t)layer * eng->cfg.n_slots + slot) * eng->cfg.n_head_kv * eng->max_blocks * HD;
    CK(eng, launch_block_summary(pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages), v, nb_whole, sum,
                                 eng->max_blocks, st));
    v = nb_whole;
    return QKV_OK;
}

extern "C" qkv_status qkv_block_summary(qkv_engine *eng, int32_t layer, int32_t slot, int32_t b0, int32_t b1,
                                        void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    if (!eng->cfg.select_block) return fail(eng, QKV_ERR_UNSUPPORTED, "engine created with select_block = 0");
    const int32_t whole = eng->slots[slot].n_past / TILE_TOK;
    if (b0 < 0 || b1 < b0 || b1 > whole) return fail(eng, QKV_ERR_INVALID, "summary blocks [%d, %d) outside the %d whole blocks", b0, b1, whole);
    if ((r = use_device(eng)) != QKV_OK) return r;
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    uint16_t *sum = eng->d_summary + ((size_t)layer * eng->cfg.n_slots + slot) * eng->cfg.n_head_kv * eng->max_blocks * HD;
    CK(eng, launch_block_summary(pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages), b0, b1, sum,
                                 eng->max_blocks, S(stream)));
    int32_t &v = eng->sum_valid[(size_t)slot * eng->cfg.n_layer + layer];
    if (b0 <= v) v = std::max(v, b1);
    return QKV_OK;
}

extern "C" qkv_status qkv_select_blocks(qkv_engine *eng, int32_t layer, const int32_t *slots, const int32_t *pos0,
                                        int32_t n_seq, const float *Q, int32_t T, int32_t top_k, int32_t *idx_out,
                                        float *scores_out, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK) return r;
    if (!eng->cfg.select_block) return fail(eng, QKV_ERR_UNSUPPORTED, "engine created with select_block = 0");
    if (!slots || !pos0 || n_seq < 1 || !Q || !idx_out || T < 1 || T > 4 || top_k < 3)
        return fail(eng, QKV_ERR_INVALID, "select: n_seq %d, T %d, top_k %d (>= 3)", n_seq, T, top_k);
    for (int i = 0; i < n_seq; i++) {
        if ((r = check_slot(eng, slots[i])) != QKV_OK) return r;
        if (pos0[i] < 0 || pos0[i] + T > eng->slots[slots[i]].n_past)
            return fail(eng, QKV_ERR_INVALID, "select: sequence %d positions beyond slot %d", i, slots[i]);
    }
    if ((r = use_device(eng)) != QKV_OK) return r;
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    const int G = eng->cfg.n_head / eng->cfg.n_head_kv;
    for (int base = 0; base < n_seq; base += MAX_SEQ) {
        const int ns = std::min(MAX_SEQ, n_seq - base);
        SelectParams P;
        memset(&P, 0, sizeof P);
        P.Q = Q + (size_t)base * T * eng->cfg.n_head * HD;
        P.summary = eng->d_summary + (size_t)layer * eng->cfg.n_slots * eng->cfg.n_head_kv * eng->max_blocks * HD;
        P.idx_out = idx_out + (size_t)base * eng->cfg.n_head_kv * top_k;
        P.scores = scores_out ? scores_out + (size_t)base * eng->cfg.n_head_kv * eng->max_blocks : eng->d_sel_scores;
        P.n_seq = ns;
        P.T = T;
        P.n_head = eng->cfg.n_head;
        P.n_head_kv = eng->cfg.n_head_kv;
        P.G = G;
        P.top_k = top_k;
        P.max_blocks = eng->max_blocks;
        for (int i = 0; i < ns; i++) {
            const int32_t slot = slots[base + i], n_kv = pos0[base + i] + T;
            const int32_t nb = (n_kv + TILE_TOK - 1) / TILE_TOK;
            P.seq_slot[i] = slot;
            P.seq_nblk[i] = nb;
            // scored blocks are 1 .. nb-3: whole blocks, summaries refreshed lazily
            if ((r = refresh_summaries(eng, layer, slot, std::max(0, nb - 2), S(stream))) != QKV_OK) return r;
        }
        CK(eng, launch_select(P, S(stream)));
    }
    return QKV_OK;
}

// ---------------------------------------------------------------------------- row transforms
static qkv_status rows_common(qkv_engine *eng, int32_t layer, int32_t slot, int32_t n) {
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    if (n < 0) return fail(eng, QKV_ERR_INVALID, "negative row count");
    return use_device(eng);
}

extern "C" qkv_status qkv_gather_rows(qkv_engine *eng, int32_t layer, int32_t slot, const int32_t *cells, int32_t n_cells,
                                      void *K_out, void *V_out, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = rows_common(eng, layer, slot, n_cells);
    if (r != QKV_OK) return r;
    if (n_cells == 0) return QKV_OK;
    if (!cells || !K_out || !V_out) return fail(eng, QKV_ERR_INVALID, "gather: null pointer");
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    CK(eng, launch_read_rows(pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages), cells, 0, n_cells,
                             static_cast<uint8_t *>(K_out), static_cast<uint8_t *>(V_out), S(stream)));
    return QKV_OK;
}

extern "C" qkv_status qkv_read_rows(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, int32_t n, void *K_out,
                                    void *V_out, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = rows_common(eng, layer, slot, n);
    if (r != QKV_OK) return r;
    if (pos < 0 || pos + n > eng->slots[slot].n_past)
        return fail(eng, QKV_ERR_INVALID, "read rows %d..%d: slot %d holds %d", pos, pos + n - 1, slot, eng->slots[slot].n_past);
    if (n == 0) return QKV_OK;
    if (!K_out || !V_out) return fail(eng, QKV_ERR_INVALID, "read rows: null pointer");
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    CK(eng, launch_read_rows(pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages), nullptr, pos, n,
                             static_cast<uint8_t *>(K_out), static_cast<uint8_t *>(V_out), S(stream)));
    return QKV_OK;
}

extern "C" qkv_status qkv_write_rows(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos, int32_t n,
                                     const void *K_in, const void *V_in, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = rows_common(eng, layer, slot, n);
    if (r != QKV_OK) return r;
    qkv_engine::Slot &sl = eng->slots[slot];
    if (pos < 0 || pos > sl.n_past || (int64_t)pos + n > eng->cfg.n_ctx)
        return fail(eng, QKV_ERR_INVALID, "write rows at %d: slot %d holds %d (n_ctx %d)", pos, slot, sl.n_past, eng->cfg.n_ctx);
    if (n == 0) return QKV_OK;
    if (!K_in || !V_in) return fail(eng, QKV_ERR_INVALID, "write rows: null pointer");
    if ((r = reserve(eng, slot, pos, n, S(stream))) != QKV_OK) return r;
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    CK(eng, launch_write_rows(pool_ref(eng, layer, eng->d_bt + (size_t)slot * eng->max_pages), pos, n,
                              static_cast<const uint8_t *>(K_in), static_cast<const uint8_t *>(V_in), S(stream)));
    sl.n_past = std::max(sl.n_past, pos + n);
    invalidate_summaries(eng, slot, pos);
    return QKV_OK;
}

// ---------------------------------------------------------------------------------- prefill
// Plan for kernel D.  Tiles are (KV head, group of 128/G query tokens); two groups of a KV head
// (2p, 2p+1) form a pair tile, run by a CTA pair, which needs 128-key KV tiles 0 .. nk-1 (causal:
// up to the pair's last query position).  The flattened sequence of all (pair tile, KV tile)
// items is cut into n_runs equal runs, one per CTA pair; each run is a list of segments, and every
// segment is one part of its pair tile (parts of a pair tile consecutive, in KV order), with the
// partial records 2 part + 0 and 2 part + 1 of its two tiles.
struct PfPlan {
    std::vector<int32_t> segs;        // 4 per segment: pair tile, kt0, kt1, part
    std::vector<int32_t> tile_parts;  // 2 per pair tile: parts, first part
    std::vector<int32_t> cta_seg;     // n_runs + 1
    int32_t n_parts = 0;
};
// Greedy cut of the flattened (pair tile, KV tile) sequence into runs of cost <= budget, where a
// run pays PF_SEG_COST KV tiles for every segment after its first (the finished segment's
// epilogue and the next query tiles).  Returns the runs used; with `segs`, records the segments
// {pair tile, kt0, kt1} and the run starts.
constexpr double PF_SEG_COST = 2.5;
static int pf_cut(const std::vector<int32_t> &nk, double budget, std::vector<int32_t> *segs,
                  std::vector<int32_t> *run_seg) {
    int runs = 0;
    size_t t = 0;
    int off = 0;
    while (t < nk.size()) {
        if (run_seg) run_seg->push_back((int32_t)(segs->size() / 4));
        runs++;
        double left = budget;
        bool first = true;
        while (t < nk.size()) {
            const double avail = left - (first ? 0.0 : PF_SEG_COST);
            int n = (int)std::floor(avail + 1e-9);
            if (n < 1) {
                if (!first) break;
                n = 1;   // a run takes at least one KV tile
            }
            n = std::min(n, nk[t] - off);
            if (segs) segs->insert(segs->end(), {(int32_t)t, off, off + n, -1});
            left = avail - n;
            first = false;
            off += n;
            if (off == nk[t]) {
                t++;
                off = 0;
            }
        }
    }
    return runs;
}

// Plan of one launch: the smallest run budget whose greedy cut fits n_runs runs (binary search;
// the cut may need fewer), then every segment's part index (parts of a pair tile consecutive, in
// KV order).
static void pf_build(const std::vector<int32_t> &nk, int64_t W, int &n_runs, PfPlan &pl) {
    const int n_tiles = (int)nk.size();
    double lo = (double)W / n_runs, hi = lo + 2 * PF_SEG_COST + 2;
    while (pf_cut(nk, hi, nullptr, nullptr) > n_runs) hi *= 1.5;
    for (int i = 0; i < 40 && hi - lo > 0.01; i++) {
        const double mid = 0.5 * (lo + hi);
        if (pf_cut(nk, mid, nullptr, nullptr) <= n_runs) hi = mid;
        else lo = mid;
    }
    pl.segs.clear();
    pl.cta_seg.clear();
    n_runs = pf_cut(nk, hi, &pl.segs, &pl.cta_seg);
    std::vector<int32_t> count(n_tiles, 0);
    for (size_t i = 0; i < pl.segs.size(); i += 4) count[pl.segs[i]]++;
    pl.cta_seg.push_back((int32_t)(pl.segs.size() / 4));
    pl.tile_parts.assign(2 * n_tiles, 0);
    pl.n_parts = 0;
    for (int i = 0; i < n_tiles; i++) {
        pl.tile_parts[2 * i] = count[i];
        pl.tile_parts[2 * i + 1] = pl.n_parts;
        pl.n_parts += count[i];
    }
    std::vector<int32_t> next(n_tiles, 0);
    for (size_t i = 0; i < pl.segs.size(); i += 4) {
        const int tile = pl.segs[i];
        pl.segs[i + 3] = pl.tile_parts[2 * tile + 1] + next[tile]++;
    }
}

static qkv_status pf_scratch(qkv_engine *eng) {
    if (eng->d_pf_q) return QKV_OK;
    const int G = eng->cfg.n_head / eng->cfg.n_head_kv, tpt = PF_ROWS / G;
    eng->pf_max_tiles = eng->cfg.n_head_kv * ((PF_MAX_TC + tpt - 1) / tpt);
    eng->pf_max_parts = eng->pf_max_tiles + eng->num_sms;   // every run boundary adds at most one segment
    eng->pf_plan_ints = 4 * (eng->pf_max_tiles + eng->num_sms) + 2 * eng->pf_max_tiles + eng->num_sms + 1;
    qkv_status r = dalloc(eng, eng->d_pf_q, (size_t)eng->pf_max_tiles * PF_QTILE, "prefill query tiles");
    if (r == QKV_OK)
        r = dalloc(eng, eng->d_pf_partial, (size_t)2 * eng->pf_max_parts * pf_part_floats() * 4, "prefill partials");
    if (r == QKV_OK) r = dalloc(eng, eng->d_pf_plan, (size_t)eng->pf_plan_ints * 4, "prefill plan");
    if (r != QKV_OK) {
        cudaFree(eng->d_pf_q);
        cudaFree(eng->d_pf_partial);
        cudaFree(eng->d_pf_plan);
        eng->d_pf_q = nullptr;
        eng->d_pf_partial = nullptr;
        eng->d_pf_plan = nullptr;
    }
    return r;
}

// Kernel D over the chunk's Tc queries; with qsa_bits (sparse prefill) each query sees only the
// kept indexer blocks of its row (qsa_words words per row).
static qkv_status prefill_run(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos0, const uint16_t *Q, int32_t Tc,
                              float scale, float *out, const uint32_t *qsa_bits, int32_t qsa_words, void *stream) {
    qkv_status r;
    if ((r = check_layer(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    const int H = eng->cfg.n_head_kv, G = eng->cfg.n_head / H;
    if (!Q || !out || Tc < 1 || Tc > PF_MAX_TC || pos0 < 0 || !std::isfinite(scale))
        return fail(eng, QKV_ERR_INVALID, "prefill: Q=%p out=%p Tc=%d (1..%d) pos0=%d", (const void *)Q, (void *)out, Tc,
                    PF_MAX_TC, pos0);
    if (PF_ROWS % G) return fail(eng, QKV_ERR_UNSUPPORTED, "prefill: q-heads per KV head %d must divide %d", G, PF_ROWS);
    const qkv_engine::Slot &sl = eng->slots[slot];
    if ((int64_t)pos0 + Tc > sl.n_past)
        return fail(eng, QKV_ERR_STATE, "prefill: positions %d..%d not appended (slot %d holds %d)", pos0, pos0 + Tc - 1,
                    slot, sl.n_past);
    if ((r = use_device(eng)) != QKV_OK) return r;
    if ((r = pf_scratch(eng)) != QKV_OK) return r;
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;

    const int tpt = PF_ROWS / G, n_groups = (Tc + tpt - 1) / tpt, n_tiles = H * n_groups;
    const int n_gpairs = (n_groups + 1) / 2, n_ptiles = H * n_gpairs;
    std::vector<int32_t> nk(n_ptiles);
    int64_t W = 0;
    for (int t = 0; t < n_ptiles; t++) {
        const int gp = t % n_gpairs, last_tok = std::min((2 * gp + 2) * tpt, Tc) - 1;
        nk[t] = (pos0 + last_tok) / PF_KT + 1;
        W += nk[t];
    }
    PfPlan pl;
    int max_pairs = prefill_max_pairs();
    if (max_pairs <= 0) max_pairs = eng->num_sms / 2;
    int n_runs = (int)std::min<int64_t>(max_pairs, W);
    pf_build(nk, W, n_runs, pl);   // may use fewer runs
    if (pl.n_parts > eng->pf_max_parts)
        return fail(eng, QKV_ERR_NO_MEMORY, "prefill plan: %d parts (max %d)", pl.n_parts, eng->pf_max_parts);
    std::vector<int32_t> ints;
    ints.reserve(pl.segs.size() + pl.tile_parts.size() + pl.cta_seg.size());
    ints.insert(ints.end(), pl.segs.begin(), pl.segs.end());
    const size_t off_tiles = ints.size();
    ints.insert(ints.end(), pl.tile_parts.begin(), pl.tile_parts.end());
    const size_t off_cta = ints.size();
    ints.insert(ints.end(), pl.cta_seg.begin(), pl.cta_seg.end());
    // small plans travel with the launch; larger ones are uploaded ahead of the kernels
    const bool inline_plan = ints.size() <= (size_t)PF_PLAN_INLINE;
    if (!inline_plan) {
        if ((int64_t)ints.size() > eng->pf_plan_ints)
            return fail(eng, QKV_ERR_NO_MEMORY, "prefill plan: %zu ints", ints.size());
        if ((r = upload_i32(eng, ints, eng->d_pf_plan, S(stream))) != QKV_OK) return r;
    } else {
        std::copy(ints.begin(), ints.end(), eng->pf_plan_inline.v);
    }

    PrefillParams P;
    memset(&P, 0, sizeof P);
    P.pool = eng->pools[layer];
    P.bt = eng->d_bt + (size_t)slot * eng->max_pages;
    P.Q = Q;
    P.qtiles = eng->d_pf_q;
    P.out = out;
    P.partial = eng->d_pf_partial;
    P.status = eng->d_status;
    P.segs = reinterpret_cast<const int4 *>(eng->d_pf_plan);
    P.tile_parts = reinterpret_cast<const int2 *>(eng->d_pf_plan + off_tiles);
    P.cta_seg = eng->d_pf_plan + off_cta;
    P.plan_inline = inline_plan;
    P.off_tiles = (int32_t)off_tiles;
    P.off_cta = (int32_t)off_cta;
    P.page_bytes = eng->page_bytes;
    P.n_pages = eng->n_pages;
    P.max_pages = eng->max_pages;
    P.n_head = eng->cfg.n_head;
    P.n_head_kv = H;
    P.G = G;
    P.tpt = tpt;
    P.n_groups = n_groups;
    P.n_gpairs = n_gpairs;
    P.n_tiles = n_tiles;
    P.Tc = Tc;
    P.pos0 = pos0;
    P.n_kv = pos0 + Tc;
    P.n_ctas = 2 * n_runs;
    P.scale_log2 = scale * 1.4426950408889634f;
    P.qsa_bits = qsa_bits;
    P.qsa_words = qsa_words;
    CK(eng, launch_prefill(P, eng->pf_plan_inline, S(stream)));
    return QKV_OK;
}

extern "C" qkv_status qkv_attn_prefill(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos0, const uint16_t *Q,
                                       int32_t Tc, float scale, float *out, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    return prefill_run(eng, layer, slot, pos0, Q, Tc, scale, out, nullptr, 0, stream);
}

extern "C" qkv_status qkv_attn_prefill_qsa(qkv_engine *eng, int32_t layer, int32_t slot, int32_t pos0, const float *q_idx,
                                           const uint16_t *Q, int32_t Tc, float scale, float *out, int32_t *blocks_out,
                                           int32_t *n_out_out, void *stream) {
    qkv_status r;
    if ((r = idx_check(eng, layer)) != QKV_OK || (r = check_slot(eng, slot)) != QKV_OK) return r;
    if (!q_idx || !Q || !out || Tc < 1 || Tc > PF_MAX_TC || pos0 < 0 || (!blocks_out) != (!n_out_out))
        return fail(eng, QKV_ERR_INVALID, "prefill_qsa: Tc %d (1..%d), pos0 %d, null pointer", Tc, PF_MAX_TC, pos0);
    if ((int64_t)pos0 + Tc > eng->slots[slot].n_past)
        return fail(eng, QKV_ERR_STATE, "prefill_qsa: positions %d..%d not appended (slot %d holds %d)", pos0, pos0 + Tc - 1,
                    slot, eng->slots[slot].n_past);
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine: no device work");
    if ((r = use_device(eng)) != QKV_OK) return r;
    cudaStream_t st = S(stream);
    if ((r = flush_tables(eng, st)) != QKV_OK) return r;
    // the rows' kept blocks: the decode selection for every query row (groups of 4 rows share the
    // pooled-key loads), IDX_MAX_VSEQ rows per launch
    const int32_t K = eng->k_blocks, words = (pos0 + Tc - 1) / PF_KT + 1;
    if ((r = idx_scratch(eng, IDX_MAX_VSEQ)) != QKV_OK) return r;
    int32_t *sel = blocks_out, *nout = n_out_out;
    if (!sel) {
        if (eng->psel_rows < Tc) {
            cudaFree(eng->d_psel);
            cudaFree(eng->d_pnout);
            eng->d_psel = eng->d_pnout = nullptr;
            eng->psel_rows = 0;
            if ((r = dalloc(eng, eng->d_psel, (size_t)PF_MAX_TC * K * sizeof(int32_t), "prefill kept blocks")) != QKV_OK ||
                (r = dalloc(eng, eng->d_pnout, (size_t)PF_MAX_TC * sizeof(int32_t), "prefill kept counts")) != QKV_OK)
                return r;
            eng->psel_rows = PF_MAX_TC;
        }
        sel = eng->d_psel;
        nout = eng->d_pnout;
    }
    if ((int64_t)Tc * words > eng->pbits_words) {
        cudaFree(eng->d_pbits);
        eng->d_pbits = nullptr;
        eng->pbits_words = 0;
        const int64_t need = (int64_t)PF_MAX_TC * ((eng->cfg.n_ctx + PF_KT - 1) / PF_KT);
        if ((r = dalloc(eng, eng->d_pbits, (size_t)need * sizeof(uint32_t), "prefill kept-block bitsets")) != QKV_OK) return r;
        eng->pbits_words = need;
    }
    const size_t qrow = (size_t)eng->icfg.n_head * IDX_KEY;
    for (int32_t v0 = 0; v0 < Tc; v0 += IDX_MAX_VSEQ) {
        const int32_t nv = std::min<int32_t>(IDX_MAX_VSEQ, Tc - v0);
        for (const int32_t T : {4, 1}) {
            const int32_t a = T == 4 ? 0 : nv / 4 * 4, n = T == 4 ? nv / 4 * 4 : nv - nv / 4 * 4;
            if (n == 0) continue;
            std::vector<int32_t> slots(n / T, slot), pos(n / T);
            for (int32_t k = 0; k < n / T; k++) pos[k] = pos0 + v0 + a + T * k;
            if ((r = idx_select_chunk(eng, layer, slots.data(), pos.data(), T, 0, n, q_idx + (size_t)(v0 + a) * qrow,
                                      sel + (size_t)(v0 + a) * K, nout + v0 + a, eng->d_iscore, eng->idx_max_blk, st)) !=
                QKV_OK)
                return r;
        }
    }
    CK(eng, launch_idx_bits(sel, nout, K, Tc, eng->d_pbits, words, st));
    return prefill_run(eng, layer, slot, pos0, Q, Tc, scale, out, eng->d_pbits, words, stream);
}

// -------------------------------------------------------------------------------- snapshots
static qkv_status rec_copy(qkv_engine *eng, const std::vector<CopyDesc> &d, cudaStream_t st) {
    if (d.empty() || eng->host_only) return QKV_OK;
    CK(eng, launch_copy_batch(d.data(), (int)d.size(), eng->num_sms, st));
    return QKV_OK;
}

extern "C" qkv_status qkv_snapshot_save(qkv_engine *eng, int32_t slot, qkv_snapshot **out, void *stream) {
    if (!eng || !out) return QKV_ERR_INVALID;
    *out = nullptr;
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    if (!eng->host_only && (r = use_device(eng)) != QKV_OK) return r;
    qkv_snapshot *snap = new (std::nothrow) qkv_snapshot;
    if (!snap) return fail(eng, QKV_ERR_NO_MEMORY, "snapshot: host allocation");
    const qkv_engine::Slot &sl = eng->slots[slot];
    snap->eng = eng;
    snap->n_past = sl.n_past;
    if (!eng->host_only && eng->rec_slot_bytes > 0) {
        r = dalloc(eng, snap->rec, eng->rec_slot_bytes, "snapshot recurrent state");
        if (r != QKV_OK) {
            delete snap;
            return r;
        }
        eng->device_bytes -= eng->rec_slot_bytes;  // snapshots are reported separately
        r = rec_copy(eng, {CopyDesc{eng->d_rec + (size_t)slot * eng->rec_slot_bytes, snap->rec, eng->rec_slot_bytes}},
                     S(stream));
        if (r != QKV_OK) {
            cudaFree(snap->rec);
            delete snap;
            return r;
        }
    }
    const int32_t np = (sl.n_past + PAGE_TOK - 1) / PAGE_TOK;
    snap->pages.assign(sl.pages.begin(), sl.pages.begin() + np);
    for (int32_t p : snap->pages) page_ref(eng, p);
    eng->snaps.push_back(snap);
    *out = snap;
    return QKV_OK;
}

static qkv_status restore_one(qkv_engine *eng, const qkv_snapshot *snap, int32_t slot, int32_t n_keep,
                              std::vector<CopyDesc> &copies) {
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    if (n_keep < 0) n_keep = snap->n_past;
    if (n_keep > snap->n_past) return fail(eng, QKV_ERR_INVALID, "restore keeps %d of a %d-position snapshot", n_keep, snap->n_past);
    qkv_engine::Slot &sl = eng->slots[slot];
    // take the new references before dropping the old ones: restoring a slot's own snapshot
    const int32_t np = (n_keep + PAGE_TOK - 1) / PAGE_TOK;
    for (int32_t i = 0; i < np; i++) page_ref(eng, snap->pages[i]);
    release_pages(eng, sl.pages);
    sl.pages.assign(snap->pages.begin(), snap->pages.begin() + np);
    sl.n_past = n_keep;
    sl.rb_depth = 0;
    sl.dirty = true;
    invalidate_summaries(eng, slot, 0);
    if (snap->rec) copies.push_back(CopyDesc{snap->rec, eng->d_rec + (size_t)slot * eng->rec_slot_bytes, eng->rec_slot_bytes});
    return QKV_OK;
}

extern "C" qkv_status qkv_snapshot_restore(qkv_engine *eng, const qkv_snapshot *snap, int32_t slot, int32_t n_keep,
                                           void *stream) {
    return qkv_snapshot_restore_many(eng, snap, &slot, &n_keep, 1, stream);
}

extern "C" qkv_status qkv_snapshot_restore_many(qkv_engine *eng, const qkv_snapshot *snap, const int32_t *slots,
                                                const int32_t *n_keep, int32_t n, void *stream) {
    if (!eng || !snap || !slots || n < 0) return QKV_ERR_INVALID;
    if (snap->eng != eng) return fail(eng, QKV_ERR_MISMATCH, "snapshot belongs to another engine");
    qkv_status r;
    if (!eng->host_only && (r = use_device(eng)) != QKV_OK) return r;
    for (int i = 0; i < n; i++) {   // validate everything before changing anything
        if ((r = check_slot(eng, slots[i])) != QKV_OK) return r;
        const int32_t k = n_keep ? n_keep[i] : -1;
        if (k > snap->n_past) return fail(eng, QKV_ERR_INVALID, "restore keeps %d of a %d-position snapshot", k, snap->n_past);
    }
    std::vector<CopyDesc> copies;
    for (int i = 0; i < n; i++)
        if ((r = restore_one(eng, snap, slots[i], n_keep ? n_keep[i] : -1, copies)) != QKV_OK) return r;
    if ((r = flush_tables(eng, S(stream))) != QKV_OK) return r;
    return rec_copy(eng, copies, S(stream));
}

extern "C" void qkv_snapshot_release(qkv_engine *eng, qkv_snapshot *snap) {
    if (!eng || !snap || snap->eng != eng) return;
    auto it = std::find(eng->snaps.begin(), eng->snaps.end(), snap);
    if (it == eng->snaps.end()) return;
    eng->snaps.erase(it);
    for (int32_t p : snap->pages) page_unref(eng, p);
    if (snap->rec && !eng->host_only) {
        cudaSetDevice(eng->device);
        cudaDeviceSynchronize();   // a restore may still be reading it
        cudaFree(snap->rec);
    }
    delete snap;
}

extern "C" qkv_status qkv_snapshot_info(const qkv_snapshot *snap, int32_t *n_past, size_t *host_bytes) {
    if (!snap) return QKV_ERR_INVALID;
    const qkv_engine *eng = snap->eng;
    if (n_past) *n_past = snap->n_past;
    if (host_bytes)
        *host_bytes = (size_t)eng->cfg.n_layer * 2 * snap->n_past * eng->cfg.n_head_kv * ROW_Q8 +
                      (eng->idx_on ? (size_t)eng->cfg.n_layer * snap->n_past * IDX_KEY * 2 : 0) +
                      (size_t)eng->cfg.rec_n_layer * ((size_t)eng->cfg.rec_head_dim * eng->cfg.rec_head_dim * eng->cfg.rec_n_head * 4 +
                                                      (size_t)eng->cfg.conv_hist * eng->cfg.conv_channels * 4);
    return QKV_OK;
}

// Layer order of a host blob: {attention?, index} per absolute layer (snapshot_parts walks the
// model's layers in order), or attention layers first when no interval is configured.
static std::vector<std::pair<bool, int>> blob_layers(const qkv_engine *eng) {
    std::vector<std::pair<bool, int>> o;
    const int A = eng->cfg.n_layer, R = eng->cfg.rec_n_layer, I = eng->cfg.attn_interval;
    if (I > 0) {
        for (int il = 0; il < A + R; il++)
            o.push_back((il + 1) % I == 0 ? std::make_pair(true, il / I) : std::make_pair(false, il - (il + 1) / I));
    } else {
        for (int a = 0; a < A; a++) o.push_back({true, a});
        for (int r = 0; r < R; r++) o.push_back({false, r});
    }
    return o;
}

// Raw indexer keys of positions 0 .. n-1 between the pages of `pages` and host memory, one copy
// per page run.
static qkv_status idx_rows_copy(qkv_engine *eng, int layer, const std::vector<int32_t> &pages, int32_t n, uint8_t *host,
                                bool to_host, cudaStream_t st) {
    for (int32_t c = 0; c < n; c += PAGE_TOK) {
        const int32_t run = std::min(PAGE_TOK, n - c);
        uint8_t *dev = eng->idx_pools[layer] + (int64_t)pages[c / PAGE_TOK] * IDX_PAGE_BYTES;
        uint8_t *h = host + (size_t)c * IDX_KEY * 2;
        CK(eng, cudaMemcpyAsync(to_host ? (void *)h : (void *)dev, to_host ? (const void *)dev : (const void *)h,
                                (size_t)run * IDX_KEY * 2, to_host ? cudaMemcpyDeviceToHost : cudaMemcpyHostToDevice, st));
    }
    return QKV_OK;
}

extern "C" qkv_status qkv_snapshot_to_host(qkv_engine *eng, const qkv_snapshot *snap, void *dst, size_t bytes,
                                           void *stream) {
    if (!eng || !snap || !dst) return QKV_ERR_INVALID;
    if (snap->eng != eng) return fail(eng, QKV_ERR_MISMATCH, "snapshot belongs to another engine");
    size_t need = 0;
    qkv_snapshot_info(snap, nullptr, &need);
    if (bytes != need) return fail(eng, QKV_ERR_MISMATCH, "host blob is %zu bytes, snapshot needs %zu", bytes, need);
    qkv_status r = use_device(eng);
    if (r != QKV_OK) return r;
    cudaStream_t st = S(stream);
    const size_t rows = (size_t)snap->n_past * eng->cfg.n_head_kv * ROW_Q8;
    uint8_t *out = static_cast<uint8_t *>(dst);
    uint8_t *stage = nullptr;
    int32_t *d_pages = nullptr;
    if ((r = dalloc(eng, stage, std::max<size_t>(2 * rows, 16), "snapshot staging")) != QKV_OK) return r;
    eng->device_bytes -= std::max<size_t>(2 * rows, 16);
    if ((r = dalloc(eng, d_pages, std::max<size_t>(snap->pages.size(), 1) * 4, "snapshot pages")) != QKV_OK) {
        cudaFree(stage);
        return r;
    }
    eng->device_bytes -= std::max<size_t>(snap->pages.size(), 1) * 4;
    auto done = [&](qkv_status s) {
        cudaStreamSynchronize(st);
        cudaFree(stage);
        cudaFree(d_pages);
        return s;
    };
    if ((r = upload_i32(eng, snap->pages, d_pages, st)) != QKV_OK) return done(r);
    const size_t rs = (size_t)eng->cfg.rec_head_dim * eng->cfg.rec_head_dim * eng->cfg.rec_n_head * 4;
    const size_t cv = (size_t)eng->cfg.conv_hist * eng->cfg.conv_channels * 4;
    for (const auto &[attn, l] : blob_layers(eng)) {
        if (attn) {
            if (snap->n_past == 0) continue;
            if (launch_read_rows(pool_ref(eng, l, d_pages), nullptr, 0, snap->n_past, stage, stage + rows, st) != cudaSuccess ||
                cudaMemcpyAsync(out, stage, 2 * rows, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                cudaStreamSynchronize(st) != cudaSuccess)
                return done(fail(eng, QKV_ERR_CUDA, "snapshot export of layer %d: %s", l, cudaGetErrorString(cudaGetLastError())));
            out += 2 * rows;
            if (eng->idx_on) {
                if ((r = idx_rows_copy(eng, l, snap->pages, snap->n_past, out, true, st)) != QKV_OK) return done(r);
                out += (size_t)snap->n_past * IDX_KEY * 2;
            }
        } else {
            const uint8_t *base = snap->rec + (size_t)l * eng->rec_layer_bytes;
            if (cudaMemcpyAsync(out, base, rs, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                cudaMemcpyAsync(out + rs, base + eng->rs_bytes, cv, cudaMemcpyDeviceToHost, st) != cudaSuccess)
                return done(fail(eng, QKV_ERR_CUDA, "snapshot export of recurrent layer %d", l));
            out += rs + cv;
        }
    }
    return done(QKV_OK);
}

extern "C" qkv_status qkv_snapshot_from_host(qkv_engine *eng, const void *src, size_t bytes, int32_t n_past,
                                             qkv_snapshot **out, void *stream) {
    if (!eng || !src || !out || n_past < 0) return QKV_ERR_INVALID;
    *out = nullptr;
    if (n_past > eng->cfg.n_ctx) return fail(eng, QKV_ERR_MISMATCH, "snapshot of %d positions exceeds n_ctx %d", n_past, eng->cfg.n_ctx);
    qkv_status r = use_device(eng);
    if (r != QKV_OK) return r;
    qkv_snapshot probe;
    probe.eng = eng;
    probe.n_past = n_past;
    size_t need = 0;
    qkv_snapshot_info(&probe, nullptr, &need);
    if (bytes != need) return fail(eng, QKV_ERR_MISMATCH, "host blob is %zu bytes, %d positions need %zu", bytes, n_past, need);
    const int32_t np = (n_past + PAGE_TOK - 1) / PAGE_TOK;
    if ((size_t)np > eng->free_pages.size()) return fail(eng, QKV_ERR_NO_MEMORY, "page pool exhausted");
    qkv_snapshot *snap = new (std::nothrow) qkv_snapshot;
    if (!snap) return fail(eng, QKV_ERR_NO_MEMORY, "snapshot: host allocation");
    snap->eng = eng;
    snap->n_past = n_past;
    for (int32_t i = 0; i < np; i++) snap->pages.push_back(page_alloc(eng));
    cudaStream_t st = S(stream);
    const size_t rows = (size_t)n_past * eng->cfg.n_head_kv * ROW_Q8;
    uint8_t *stage = nullptr;
    int32_t *d_pages = nullptr;
    auto undo = [&](qkv_status s) {
        cudaStreamSynchronize(st);
        cudaFree(stage);
        cudaFree(d_pages);
        for (int32_t p : snap->pages) page_unref(eng, p);
        cudaFree(snap->rec);
        delete snap;
        return s;
    };
    if ((r = dalloc(eng, stage, std::max<size_t>(2 * rows, 16), "snapshot staging")) != QKV_OK) return undo(r);
    eng->device_bytes -= std::max<size_t>(2 * rows, 16);
    if ((r = dalloc(eng, d_pages, std::max<size_t>(np, 1) * 4, "snapshot pages")) != QKV_OK) return undo(r);
    eng->device_bytes -= std::max<size_t>(np, 1) * 4;
    if (eng->rec_slot_bytes > 0) {
        if ((r = dalloc(eng, snap->rec, eng->rec_slot_bytes, "snapshot recurrent state")) != QKV_OK) return undo(r);
        eng->device_bytes -= eng->rec_slot_bytes;
        CK(eng, cudaMemsetAsync(snap->rec, 0, eng->rec_slot_bytes, st));
    }
    if ((r = upload_i32(eng, snap->pages, d_pages, st)) != QKV_OK) return undo(r);
    const uint8_t *in = static_cast<const uint8_t *>(src);
    const size_t rs = (size_t)eng->cfg.rec_head_dim * eng->cfg.rec_head_dim * eng->cfg.rec_n_head * 4;
    const size_t cv = (size_t)eng->cfg.conv_hist * eng->cfg.conv_channels * 4;
    for (const auto &[attn, l] : blob_layers(eng)) {
        if (attn) {
            if (n_past == 0) continue;
            if (cudaMemcpyAsync(stage, in, 2 * rows, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                launch_write_rows(pool_ref(eng, l, d_pages), 0, n_past, stage, stage + rows, st) != cudaSuccess ||
                cudaStreamSynchronize(st) != cudaSuccess)
                return undo(fail(eng, QKV_ERR_CUDA, "snapshot import of layer %d", l));
            in += 2 * rows;
            if (eng->idx_on) {   // raw keys, then the whole blocks pooled again
                if ((r = idx_rows_copy(eng, l, snap->pages, n_past, const_cast<uint8_t *>(in), false, st)) != QKV_OK)
                    return undo(r);
                IdxAppendParams p;
                memset(&p, 0, sizeof p);
                p.pool = eng->idx_pools[l];
                p.bt = d_pages;
                p.norm_w = eng->d_knorm + (size_t)l * IDX_KEY;
                p.rope = eng->d_rope;
                p.status = eng->d_status;
                p.n_pages = eng->n_pages;
                p.max_pages = np;
                p.rope_half = eng->icfg.rope_dim / 2;
                p.eps = eng->icfg.rms_eps;
                if (launch_idx_pool(p, 0, n_past / IDX_R, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
                    return undo(fail(eng, QKV_ERR_CUDA, "snapshot import: pooling indexer keys of layer %d", l));
                in += (size_t)n_past * IDX_KEY * 2;
            }
        } else {
            uint8_t *base = snap->rec + (size_t)l * eng->rec_layer_bytes;
            if (cudaMemcpyAsync(base, in, rs, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaMemcpyAsync(base + eng->rs_bytes, in + rs, cv, cudaMemcpyHostToDevice, st) != cudaSuccess)
                return undo(fail(eng, QKV_ERR_CUDA, "snapshot import of recurrent layer %d", l));
            in += rs + cv;
        }
    }
    cudaStreamSynchronize(st);
    cudaFree(stage);
    cudaFree(d_pages);
    eng->snaps.push_back(snap);
    *out = snap;
    return QKV_OK;
}

// --------------------------------------------------------------------------------- rollback
extern "C" qkv_status qkv_rollback_arm(qkv_engine *eng, int32_t slot, int32_t depth) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    if (depth < 0 || depth > eng->cfg.n_rollback)
        return fail(eng, QKV_ERR_INVALID, "rollback depth %d outside [0, %d]", depth, eng->cfg.n_rollback);
    eng->slots[slot].rb_depth = depth;
    return QKV_OK;
}

extern "C" qkv_status qkv_rollback(qkv_engine *eng, int32_t slot, int32_t n_back, void *stream) {
    if (!eng) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot);
    if (r != QKV_OK) return r;
    qkv_engine::Slot &sl = eng->slots[slot];
    if (n_back < 1 || n_back > sl.rb_depth)
        return fail(eng, QKV_ERR_STATE, "rollback: no snapshot of the state %d tokens back (depth %d)", n_back, sl.rb_depth);
    if (n_back > sl.n_past) return fail(eng, QKV_ERR_STATE, "rollback of %d past position 0", n_back);
    if (!eng->host_only) {
        if ((r = use_device(eng)) != QKV_OK) return r;
        if (eng->rec_slot_bytes > 0) {
            const uint8_t *src = eng->d_rb + ((size_t)slot * eng->cfg.n_rollback + (n_back - 1)) * eng->rec_slot_bytes;
            if ((r = rec_copy(eng, {CopyDesc{src, eng->d_rec + (size_t)slot * eng->rec_slot_bytes, eng->rec_slot_bytes}},
                              S(stream))) != QKV_OK)
                return r;
        }
    }
    sl.n_past -= n_back;
    sl.rb_depth = 0;
    invalidate_summaries(eng, slot, sl.n_past);
    return QKV_OK;
}

extern "C" qkv_status qkv_state_ptr(qkv_engine *eng, int32_t slot, int32_t rec_layer, int32_t kind, int32_t which,
                                    void **ptr, size_t *bytes) {
    if (!eng || !ptr) return QKV_ERR_INVALID;
    qkv_status r = check_slot(eng, slot, false);
    if (r != QKV_OK) return r;
    if (rec_layer < 0 || rec_layer >= eng->cfg.rec_n_layer || kind < 0 || kind > 1 || which < 0 || which > eng->cfg.n_rollback)
        return fail(eng, QKV_ERR_INVALID, "state_ptr: layer %d kind %d which %d", rec_layer, kind, which);
    if (eng->host_only) return fail(eng, QKV_ERR_UNSUPPORTED, "host-only engine has no device state");
    uint8_t *base = which == 0 ? eng->d_rec + (size_t)slot * eng->rec_slot_bytes
                               : eng->d_rb + ((size_t)slot * eng->cfg.n_rollback + (which - 1)) * eng->rec_slot_bytes;
    base += (size_t)rec_layer * eng->rec_layer_bytes + (kind ? eng->rs_bytes : 0);
    *ptr = base;
    if (bytes)
        *bytes = kind ? (size_t)eng->cfg.conv_hist * eng->cfg.conv_channels * 4
                      : (size_t)eng->cfg.rec_head_dim * eng->cfg.rec_head_dim * eng->cfg.rec_n_head * 4;
    return QKV_OK;
}

extern "C" qkv_status qkv_cache_view_get(const qkv_engine *eng, int32_t layer, qkv_cache_view *view) {
    if (!eng || !view || layer < 0 || layer >= eng->cfg.n_layer) return QKV_ERR_INVALID;
    view->pool = eng->host_only ? nullptr : eng->pools[layer];
    view->page_bytes = (size_t)eng->page_bytes;
    view->tile_bytes = TILE_BYTES;
    view->page_tokens = PAGE_TOK;
    view->tile_tokens = TILE_TOK;
    view->n_pages = eng->n_pages;
    view->n_head_kv = eng->cfg.n_head_kv;
    view->head_dim = HD;
    view->block_table = eng->d_bt;
    view->max_pages_per_seq = eng->max_pages;
    return QKV_OK;
}

extern "C" qkv_status qkv_debug_decode_wait(qkv_engine *eng, int64_t wait_limit_ns, int32_t withhold_unit) {
    if (!eng) return QKV_ERR_INVALID;
    eng->wait_ns = wait_limit_ns > 0 ? (uint64_t)wait_limit_ns : WAIT_NS_DEFAULT;
    eng->withhold_unit = withhold_unit >= 0 ? withhold_unit : -1;
    return QKV_OK;
}

extern "C" qkv_status qkv_device_status(qkv_engine *eng, void *stream, int32_t *code) {
    if (!eng || !code) return QKV_ERR_INVALID;
    qkv_status r = use_device(eng);
    if (r != QKV_OK) return r;
    int32_t h = 0;
    CK(eng, cudaMemcpyAsync(&h, eng->d_status, 4, cudaMemcpyDeviceToHost, S(stream)));
    CK(eng, cudaStreamSynchronize(S(stream)));
    CK(eng, cudaMemsetAsync(eng->d_status, 0, 4, S(stream)));
    *code = h;
    return h ? fail(eng, QKV_ERR_DEVICE, "device status 0x%x (1 = bad page, 2 = bad index, 4 = timed-out wait)", h) : QKV_OK;
}

// ------------------------------------------------------------------------------- multi-GPU
extern "C" qkv_status qkv_shard_lpt(const int64_t *cost, int32_t n, int32_t n_ranks, int32_t *owner) {
    if (n < 0 || n_ranks < 1 || (n > 0 && (!cost || !owner))) return QKV_ERR_INVALID;
    std::vector<int32_t> order(n);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return cost[a] > cost[b]; });
    std::vector<int64_t> load(n_ranks, 0);
    for (int32_t i : order) {
        int32_t best = 0;
        for (int32_t k = 1; k < n_ranks; k++)
            if (load[k] < load[best]) best = k;
        owner[i] = best;
        load[best] += cost[i];
    }
    return QKV_OK;
}
