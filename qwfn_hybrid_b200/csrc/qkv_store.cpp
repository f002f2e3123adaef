// qkv_store.cpp -- saved sequences kept on the device, keyed by token ids (the reference server's
// saved_seq list, restore_or_reset and shared_prefix_split, tools/qwfn_server.cpp:764-800,
// 1380-1430).  A saved sequence is an engine snapshot: its pages stay shared and refcounted and its
// recurrent state is a device copy, so saving and restoring move no KV bytes and no host blob.
#include "qkv.h"
#include "qkv_internal.h"

#include <algorithm>
#include <cstdio>
#include <new>
#include <vector>

namespace {
struct Entry {
    std::vector<int32_t> tok;
    qkv_snapshot        *snap  = nullptr;
    size_t               bytes = 0;
};
}  // namespace

struct qkv_store {
    qkv_engine        *eng = nullptr;
    size_t             cap = 0;
    int32_t            max_entries = 0;
    std::vector<Entry> saved;   // least recently used first

    size_t total() const {
        size_t t = 0;
        for (const Entry &e : saved) t += e.bytes;
        return t;
    }
    void drop(size_t i) {
        qkv_snapshot_release(eng, saved[i].snap);
        saved.erase(saved.begin() + (std::ptrdiff_t)i);
    }
};

static qkv_status bad(qkv_store *s, const char *msg) {
    return s && s->eng ? qkv::engine_fail(s->eng, QKV_ERR_INVALID, msg) : QKV_ERR_INVALID;
}

extern "C" qkv_status qkv_store_create(qkv_engine *eng, size_t cap_bytes, int32_t max_entries, qkv_store **out) {
    if (!eng || !out || max_entries < 1) return QKV_ERR_INVALID;
    qkv_store *s = new (std::nothrow) qkv_store;
    if (!s) return QKV_ERR_NO_MEMORY;
    s->eng = eng;
    s->cap = cap_bytes;
    s->max_entries = max_entries;
    *out = s;
    return QKV_OK;
}

extern "C" void qkv_store_destroy(qkv_store *store) {
    if (!store) return;
    while (!store->saved.empty()) store->drop(store->saved.size() - 1);
    delete store;
}

extern "C" qkv_status qkv_store_save(qkv_store *store, int32_t slot, const int32_t *tok, int32_t n_tok, int32_t *kept,
                                     void *stream) {
    if (!store || !kept || n_tok < 0 || (n_tok > 0 && !tok)) return bad(store, "store_save: bad arguments");
    *kept = 0;
    int32_t n_past = -1;
    qkv_status r = qkv_seq_length(store->eng, slot, &n_past);
    if (r != QKV_OK) return bad(store, "store_save: no such slot");
    if (n_past != n_tok) {
        char msg[128];
        snprintf(msg, sizeof msg, "store_save: %d tokens for a slot holding %d positions", n_tok, n_past);
        return bad(store, msg);
    }
    Entry e;
    e.tok.assign(tok, tok + n_tok);
    if ((r = qkv_snapshot_save(store->eng, slot, &e.snap, stream)) != QKV_OK) return r;
    e.bytes = qkv::snapshot_held_bytes(e.snap);
    if (e.bytes > store->cap) {   // larger than the whole budget on its own: released at once
        qkv_snapshot_release(store->eng, e.snap);
        return QKV_OK;
    }
    // an entry with the same token list gives way to the new one, which goes to the most recent
    // end; then the least recently used entries leave until the count and the bytes fit
    for (size_t k = 0; k < store->saved.size(); k++)
        if (store->saved[k].tok == e.tok) {
            store->drop(k);
            break;
        }
    store->saved.push_back(std::move(e));
    size_t total = store->total();
    while (store->saved.size() > (size_t)store->max_entries || total > store->cap) {
        total -= store->saved.front().bytes;
        store->drop(0);
    }
    *kept = 1;
    return QKV_OK;
}

// Index of the entry whose token list is a proper prefix of `prompt` and has the most tokens (the
// server's best_saved), or -1 when no entry qualifies.
static int best_saved(const qkv_store *s, const int32_t *prompt, int32_t n) {
    int best = -1;
    for (size_t k = 0; k < s->saved.size(); k++) {
        const std::vector<int32_t> &t = s->saved[k].tok;
        if ((int64_t)t.size() < n && std::equal(t.begin(), t.end(), prompt) &&
            (best < 0 || t.size() > s->saved[(size_t)best].tok.size()))
            best = (int)k;
    }
    return best;
}

extern "C" qkv_status qkv_store_restore_or_reset(qkv_store *store, int32_t slot, const int32_t *prompt,
                                                 int32_t n_prompt, int32_t *n_restored, void *stream) {
    if (!store || !n_restored || n_prompt < 0 || (n_prompt > 0 && !prompt))
        return bad(store, "store_restore_or_reset: bad arguments");
    *n_restored = 0;
    const int best = best_saved(store, prompt, n_prompt);
    if (best >= 0 && qkv_snapshot_restore(store->eng, store->saved[(size_t)best].snap, slot, -1, stream) == QKV_OK) {
        *n_restored = (int32_t)store->saved[(size_t)best].tok.size();
        std::rotate(store->saved.begin() + best, store->saved.begin() + best + 1, store->saved.end());
        return QKV_OK;
    }
    return qkv_seq_reset(store->eng, slot, stream);
}

extern "C" qkv_status qkv_store_prefix_split(const qkv_store *store, const int32_t *prompt, int32_t n_prompt,
                                             int32_t n_consumed, int32_t min_prefix, int32_t *split_at) {
    if (!store || !split_at || n_prompt < 0 || (n_prompt > 0 && !prompt) || n_consumed < 0 || min_prefix < 0)
        return QKV_ERR_INVALID;
    *split_at = 0;
    if (n_consumed >= min_prefix) return QKV_OK;
    // L: the longest run of leading tokens the prompt shares with any entry
    size_t L = 0;
    for (const Entry &e : store->saved) {
        const size_t m = std::min(e.tok.size(), (size_t)n_prompt);
        size_t l = 0;
        while (l < m && e.tok[l] == prompt[l]) l++;
        L = std::max(L, l);
    }
    bool have = false;   // some entry ends exactly where the shared run ends
    for (const Entry &e : store->saved) have |= e.tok.size() == L && std::equal(e.tok.begin(), e.tok.end(), prompt);
    if (L >= (size_t)min_prefix && L + 16 < (size_t)n_prompt && L >= (size_t)n_consumed + 2 && !have)
        *split_at = (int32_t)L;
    return QKV_OK;
}

extern "C" qkv_status qkv_store_evict(qkv_store *store, int32_t n) {
    if (!store || n < 0) return QKV_ERR_INVALID;
    for (int32_t i = 0; i < n && !store->saved.empty(); i++) store->drop(0);
    return QKV_OK;
}

extern "C" qkv_status qkv_store_info(const qkv_store *store, int32_t *n_entries, size_t *bytes) {
    if (!store) return QKV_ERR_INVALID;
    if (n_entries) *n_entries = (int32_t)store->saved.size();
    if (bytes) *bytes = store->total();
    return QKV_OK;
}

extern "C" qkv_status qkv_store_entry(const qkv_store *store, int32_t i, int32_t *n_tok, size_t *bytes) {
    if (!store || i < 0 || (size_t)i >= store->saved.size()) return QKV_ERR_INVALID;
    if (n_tok) *n_tok = (int32_t)store->saved[(size_t)i].tok.size();
    if (bytes) *bytes = store->saved[(size_t)i].bytes;
    return QKV_OK;
}
