/* qkv.hpp -- header-only C++ facade over the C ABI in qkv.h, shaped like the reference engine's own
 * state and snapshot interface so its callers change types, not logic.
 *
 *   qwfn::state            (src/qwfn_state.h:39-69)   -> qkv::state
 *   qwfn::state_config     (src/qwfn_state.h:28-37)   -> qkv_config (+ qkv::layer_map)
 *   engine::state_snapshot (src/qwfn_engine.h:293-309) -> qkv::state_snapshot
 *   engine::snapshot_save / snapshot_load / reset / rollback_n
 *                          (src/qwfn_engine.h:310-312, src/qwfn_engine.cpp:988-1066, 3629-3660)
 *
 * Error convention as in the reference: bool + std::string &err where the reference has one,
 * bool alone for snapshot_save/load.  Nothing here aborts.  Layer indices are the reference's
 * ABSOLUTE indices (0..n_layer-1): attention layers map to the engine's attention-layer index,
 * the others to its recurrent-state index, as hparams::is_attn_layer splits them
 * (src/qwfn_hparams.h:29-30, 85-87).  One sequence slot per facade (the reference holds one
 * sequence); several facades can share one engine through different slots.
 */
#ifndef QKV_HPP
#define QKV_HPP

#include "qkv.h"

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

namespace qkv {

/* Which absolute layers carry a q8_0 K/V cache: (il + 1) % full_attention_interval == 0, the
 * rest are recurrent (Gated DeltaNet) layers whose state rides in snapshots. */
struct layer_map {
    uint32_t n_layer = 48;
    uint32_t full_attention_interval = 4;

    bool is_attn_layer(uint32_t il) const {
        return il < n_layer && full_attention_interval > 0 && (il + 1) % full_attention_interval == 0;
    }
    /* engine attention-layer index of absolute layer il, -1 for a recurrent layer */
    int32_t attn_index(uint32_t il) const {
        return is_attn_layer(il) ? (int32_t)(il / full_attention_interval) : -1;
    }
    /* engine recurrent-layer index of absolute layer il, -1 for an attention layer */
    int32_t rec_index(uint32_t il) const {
        if (il >= n_layer || is_attn_layer(il)) return -1;
        return full_attention_interval > 0 ? (int32_t)(il - (il + 1) / full_attention_interval) : (int32_t)il;
    }
    uint32_t n_attn() const { return full_attention_interval > 0 ? n_layer / full_attention_interval : 0; }
    uint32_t n_rec() const { return n_layer - n_attn(); }
};

/* A saved sequence: the first n_past positions' pages (shared, refcounted) plus a device copy
 * of the recurrent state.  Copies of a state_snapshot share one engine snapshot, released with
 * the last copy; the engine must outlive it. */
struct state_snapshot {
    int32_t n_past = 0;
    std::shared_ptr<qkv_snapshot> handle;

    bool empty() const { return !handle; }
    /* bytes the snapshot's host blob (qkv_snapshot_to_host) would take: the reference's
     * state_snapshot::bytes() (src/qwfn_engine.h:302-306). */
    size_t bytes() const {
        size_t b = 0;
        if (handle) qkv_snapshot_info(handle.get(), nullptr, &b);
        return b;
    }
};

class state {
public:
    state() = default;
    ~state() { destroy(); }
    state(const state &) = delete;
    state &operator=(const state &) = delete;

    /* Creates the engine (device < 0: host-only, no kernels) and allocates this facade's slot.
     * cfg.n_layer must equal map.n_attn() and cfg.rec_n_layer map.n_rec() (a recurrent-state-less
     * engine, rec_n_layer 0, is allowed).  Replaces state::init (src/qwfn_state.cpp:21-46). */
    bool init(const layer_map &map, const qkv_config &cfg, int device, std::string &err) {
        destroy();
        if (cfg.n_layer != (int32_t)map.n_attn() || (cfg.rec_n_layer != 0 && cfg.rec_n_layer != (int32_t)map.n_rec())) {
            err = "qkv::state::init: the config's layer counts do not match the layer map";
            return false;
        }
        qkv_config c = cfg;   // host blobs in the model's layer order unless the caller chose one
        if (c.attn_interval == 0 && c.rec_n_layer > 0 &&
            (int64_t)c.n_layer * map.full_attention_interval == (int64_t)c.n_layer + c.rec_n_layer)
            c.attn_interval = (int32_t)map.full_attention_interval;
        qkv_engine *e = nullptr;
        qkv_status st = qkv_create(&c, device, &e);
        if (st != QKV_OK) {
            err = std::string("qkv_create: ") + qkv_status_string(st);
            return false;
        }
        eng_ = e;
        owned_ = true;
        if (!attach_slot(map, 0, err)) return false;
        n_ctx_ = (uint32_t)cfg.n_ctx;
        return true;
    }

    /* Uses an existing engine's slot (allocating it); the engine stays the caller's. */
    bool init_shared(qkv_engine *eng, const layer_map &map, int32_t slot, std::string &err) {
        destroy();
        if (!eng) { err = "qkv::state::init_shared: null engine"; return false; }
        eng_ = eng;
        owned_ = false;
        return attach_slot(map, slot, err);
    }

    /* Attention layers: a description of the layer's page pool (K and V live in the same pages,
     * so k_cache and v_cache return the same view); nullptr for recurrent layers, as the
     * reference's accessors return null there (src/qwfn_state.h:50-53). */
    const qkv_cache_view *k_cache(uint32_t il) const {
        const int32_t a = map_.attn_index(il);
        return a >= 0 && (size_t)a < views_.size() ? &views_[a] : nullptr;
    }
    const qkv_cache_view *v_cache(uint32_t il) const { return k_cache(il); }

    /* Recurrent layers: device F32 [rec_head_dim, rec_head_dim, rec_n_head] and [conv_hist,
     * conv_channels] of this slot's live state; nullptr for attention layers, a host-only engine
     * or an engine without recurrent state (src/qwfn_state.h:55-57). */
    void *rs_state(uint32_t il) const { return rec_ptr(il, 0); }
    void *rs_conv(uint32_t il) const { return rec_ptr(il, 1); }

    /* Releases the slot's pages, zeroes its recurrent state, rewinds to position 0: the
     * reference's state::reset + engine::reset (src/qwfn_state.cpp:113-121,
     * src/qwfn_engine.cpp:1055-1066). */
    void reset(void *stream = nullptr) {
        if (eng_) qkv_seq_reset(eng_, slot_, stream);
    }

    size_t bytes() const {
        size_t b = 0;
        if (eng_) qkv_bytes(eng_, &b);
        return b;
    }
    std::string summary() const {
        char buf[512] = {0};
        if (eng_ && qkv_summary(eng_, buf, sizeof buf) == QKV_OK) return buf;
        return "qkv state: not initialised";
    }
    /* positions per sequence (for init_shared: the block table's capacity, a multiple of 256) */
    uint32_t n_ctx() const { return n_ctx_; }
    int32_t n_past() const {
        int32_t n = 0;
        if (eng_) qkv_seq_length(eng_, slot_, &n);
        return n;
    }

    /* engine::snapshot_save (src/qwfn_engine.cpp:1001-1027): false, with s left empty, when the
     * engine cannot take the snapshot. */
    bool snapshot_save(state_snapshot &s, void *stream = nullptr) {
        s = state_snapshot{};
        qkv_snapshot *h = nullptr;
        if (!eng_ || qkv_snapshot_save(eng_, slot_, &h, stream) != QKV_OK) return false;
        qkv_engine *e = eng_;
        s.handle = std::shared_ptr<qkv_snapshot>(h, [e](qkv_snapshot *p) { qkv_snapshot_release(e, p); });
        qkv_snapshot_info(h, &s.n_past, nullptr);
        return true;
    }
    /* engine::snapshot_load (src/qwfn_engine.cpp:1029-1053): false on an empty snapshot or one
     * that does not fit this engine. */
    bool snapshot_load(const state_snapshot &s, void *stream = nullptr) {
        if (!eng_ || !s.handle) return false;
        return qkv_snapshot_restore(eng_, s.handle.get(), slot_, -1, stream) == QKV_OK;
    }
    /* engine::rollback_n (src/qwfn_engine.cpp:3629-3660). */
    bool rollback_n(int32_t n_back, std::string &err, void *stream = nullptr) {
        if (!eng_) { err = "qkv::state: not initialised"; return false; }
        if (qkv_rollback(eng_, slot_, n_back, stream) != QKV_OK) {
            err = qkv_last_error(eng_);
            return false;
        }
        return true;
    }

    qkv_engine *engine() const { return eng_; }
    int32_t slot() const { return slot_; }
    const layer_map &layers() const { return map_; }

private:
    bool attach_slot(const layer_map &map, int32_t slot, std::string &err) {
        map_ = map;
        slot_ = slot;
        if (qkv_seq_alloc(eng_, slot) != QKV_OK) {
            err = std::string("qkv_seq_alloc: ") + qkv_last_error(eng_);
            destroy();
            return false;
        }
        slot_held_ = true;
        views_.assign(map.n_attn(), qkv_cache_view{});
        for (uint32_t a = 0; a < map.n_attn(); a++) {
            if (qkv_cache_view_get(eng_, (int32_t)a, &views_[a]) != QKV_OK) {
                err = "qkv_cache_view_get failed";
                destroy();
                return false;
            }
        }
        n_ctx_ = views_.empty() ? 0u : (uint32_t)views_[0].max_pages_per_seq * (uint32_t)views_[0].page_tokens;
        return true;
    }
    void *rec_ptr(uint32_t il, int32_t kind) const {
        const int32_t r = map_.rec_index(il);
        void *p = nullptr;
        if (r < 0 || !eng_ || qkv_state_ptr(eng_, slot_, r, kind, 0, &p, nullptr) != QKV_OK) return nullptr;
        return p;
    }
    void destroy() {
        if (eng_ && slot_held_) qkv_seq_free(eng_, slot_);
        if (eng_ && owned_) qkv_destroy(eng_);
        eng_ = nullptr;
        owned_ = false;
        slot_held_ = false;
        views_.clear();
    }

    qkv_engine *eng_ = nullptr;
    bool owned_ = false, slot_held_ = false;
    int32_t slot_ = 0;
    uint32_t n_ctx_ = 0;
    layer_map map_;
    std::vector<qkv_cache_view> views_;
};

}  // namespace qkv

#endif  // QKV_HPP
