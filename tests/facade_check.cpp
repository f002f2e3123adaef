// Exercises the C++ facade include/qkv.hpp the way the reference engine's callers use qwfn::state
// and engine::snapshot_save/load/rollback_n (src/qwfn_state.h:46-69, src/qwfn_engine.h:293-312).
// argv[1] = device: < 0 runs on a host-only engine (page tables, refcounts, snapshots; no kernels),
// >= 0 also moves recurrent state and cache rows on that GPU.  Prints "facade ok" and exits 0, or
// names the first failed check and exits 1.
#include "qkv.hpp"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <set>
#include <vector>

static int g_fail = 0;
#define CHECK(c)                                                     \
    do {                                                             \
        if (!(c)) {                                                  \
            std::fprintf(stderr, "check failed line %d: %s\n", __LINE__, #c); \
            g_fail = 1;                                              \
            return 1;                                                \
        }                                                            \
    } while (0)

static int layer_map_checks() {
    const qkv::layer_map m;   // the model: 48 layers, every 4th attention
    CHECK(m.n_attn() == 12 && m.n_rec() == 36);
    std::set<int32_t> att, rec;
    for (uint32_t il = 0; il < m.n_layer; il++) {
        const int32_t a = m.attn_index(il), r = m.rec_index(il);
        CHECK((a >= 0) != (r >= 0));
        CHECK(m.is_attn_layer(il) == ((il + 1) % 4 == 0));
        if (a >= 0) att.insert(a); else rec.insert(r);
    }
    CHECK(att.size() == 12 && *att.begin() == 0 && *att.rbegin() == 11);
    CHECK(rec.size() == 36 && *rec.begin() == 0 && *rec.rbegin() == 35);
    CHECK(m.attn_index(3) == 0 && m.attn_index(47) == 11 && m.rec_index(4) == 3 && m.rec_index(48) == -1);
    return 0;
}

int main(int argc, char **argv) {
    const int device = argc > 1 ? std::atoi(argv[1]) : -1;
    if (layer_map_checks()) return 1;

    const qkv::layer_map map{8, 4};      // attention at 3 and 7, six recurrent layers
    qkv_config cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cfg.n_layer = 2; cfg.n_head = 16; cfg.n_head_kv = 2; cfg.head_dim = 256;
    cfg.n_ctx = 4096; cfg.n_slots = 2;
    cfg.rec_n_layer = 6; cfg.rec_head_dim = 16; cfg.rec_n_head = 2;
    cfg.conv_channels = 32; cfg.conv_hist = 3; cfg.n_rollback = 2;

    std::string err;
    {
        qkv::state bad;
        qkv_config c2 = cfg;
        c2.n_layer = 3;
        CHECK(!bad.init(map, c2, device, err) && !err.empty());
    }

    qkv::state st;
    err.clear();
    CHECK(st.init(map, cfg, device, err));
    CHECK(st.n_ctx() == 4096 && st.n_past() == 0 && st.slot() == 0);
    CHECK(st.k_cache(3) != nullptr && st.k_cache(7) != nullptr && st.k_cache(0) == nullptr && st.k_cache(8) == nullptr);
    CHECK(st.v_cache(3) == st.k_cache(3));
    CHECK(st.k_cache(3)->page_tokens == 256 && st.k_cache(3)->head_dim == 256 && st.k_cache(3)->n_head_kv == 2);
    CHECK(st.summary().find("qkv engine") == 0);
    CHECK(st.rs_state(3) == nullptr);                      // attention layer: no recurrent state
    if (device < 0) {
        CHECK(st.rs_state(0) == nullptr && st.k_cache(3)->pool == nullptr);
    } else {
        CHECK(st.rs_state(0) != nullptr && st.rs_conv(6) != nullptr && st.rs_state(0) != st.rs_state(1));
        CHECK(st.k_cache(3)->pool != nullptr && st.k_cache(3)->pool != st.k_cache(7)->pool && st.bytes() > 0);
    }

    // 300 rows into both attention layers (zeros on a GPU; host-only engines reserve the pages and
    // report that no rows were written)
    const int n_rows = 300;
    static float host_dummy[1];
    float *K = host_dummy;                                // never read by a host-only engine
    if (device >= 0) {
        CHECK(cudaSetDevice(device) == cudaSuccess);
        CHECK(cudaMalloc(&K, (size_t)n_rows * 512 * sizeof(float)) == cudaSuccess);
        CHECK(cudaMemset(K, 0, (size_t)n_rows * 512 * sizeof(float)) == cudaSuccess);
    }
    for (int32_t a = 0; a < 2; a++) {
        const qkv_status s = qkv_append(st.engine(), a, st.slot(), 0, K, K, n_rows, nullptr);
        CHECK(s == (device < 0 ? QKV_ERR_UNSUPPORTED : QKV_OK));
    }
    CHECK(st.n_past() == n_rows);

    std::vector<float> pattern(16 * 16 * 2), back(pattern.size(), -1.f);
    for (size_t i = 0; i < pattern.size(); i++) pattern[i] = (float)i + 0.5f;
    if (device >= 0)
        CHECK(cudaMemcpy(st.rs_state(5), pattern.data(), pattern.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess);

    qkv::state_snapshot snap;
    CHECK(snap.empty() && snap.bytes() == 0);
    CHECK(st.snapshot_save(snap));
    CHECK(!snap.empty() && snap.n_past == n_rows);
    CHECK(snap.bytes() == (size_t)2 * 2 * n_rows * 2 * 272 + (size_t)6 * (16 * 16 * 2 * 4 + 3 * 32 * 4));
    int32_t pages[16], n_pg = 0, rc = 0;
    CHECK(qkv_seq_pages(st.engine(), st.slot(), pages, 16, &n_pg) == QKV_OK && n_pg == 2);
    CHECK(qkv_page_refcount(st.engine(), pages[0], &rc) == QKV_OK && rc == 2);   // slot + snapshot

    st.reset();
    CHECK(st.n_past() == 0);
    if (device >= 0) {
        CHECK(cudaMemcpy(back.data(), st.rs_state(5), back.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
        CHECK(back[7] == 0.f);                            // reset zeroes the recurrent state
    }
    CHECK(st.snapshot_load(snap));
    CHECK(st.n_past() == n_rows);
    if (device >= 0) {
        CHECK(cudaDeviceSynchronize() == cudaSuccess);
        CHECK(cudaMemcpy(back.data(), st.rs_state(5), back.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
        CHECK(std::memcmp(back.data(), pattern.data(), back.size() * 4) == 0);
    }

    // a second facade on the same engine, another slot, restoring the same snapshot
    {
        qkv::state other;
        CHECK(other.init_shared(st.engine(), map, 1, err));
        CHECK(other.n_ctx() >= 4096 && other.k_cache(7) != nullptr);
        CHECK(other.snapshot_load(snap) && other.n_past() == n_rows);
        CHECK(qkv_page_refcount(st.engine(), pages[0], &rc) == QKV_OK && rc == 3);
    }   // its slot is freed, the engine stays
    CHECK(qkv_page_refcount(st.engine(), pages[0], &rc) == QKV_OK && rc == 2);

    // rollback: refused until the recurrent step arms it, then rewinds n_past
    err.clear();
    CHECK(!st.rollback_n(1, err) && err.find("rollback") != std::string::npos);
    CHECK(qkv_rollback_arm(st.engine(), st.slot(), 2) == QKV_OK);
    CHECK(st.rollback_n(2, err) && st.n_past() == n_rows - 2);

    {
        qkv::state_snapshot copy = snap;                  // shared handle
        snap = qkv::state_snapshot{};
        CHECK(!copy.empty() && copy.n_past == n_rows);
    }   // last copy gone: the snapshot's page references are dropped
    CHECK(qkv_page_refcount(st.engine(), pages[0], &rc) == QKV_OK && rc == 1);
    CHECK(!st.snapshot_load(snap));                       // empty snapshot

    if (device >= 0) cudaFree(K);
    std::printf("facade ok (device %d)\n", device);
    return g_fail;
}
