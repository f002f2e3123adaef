// Drives include/qkv_ggml.hpp the way a ggml custom op in the reference's graph would: operands
// shaped as sparse_attn / sparse_attn_decode build them (src/qwfn_graph.cpp:454-471, 653-705).
// argv[1] = device.  < 0: a host-only engine; every malformed view is rejected with a message.
// >= 0: also on that GPU -- a 2-chunk prefill (kv_append + causal attention, bf16 queries) and a
// fused 3-token decode step through the adapter, each compared with the C oracle
// (oracle/qkv_oracle.c) within atol 2e-3 + rtol 1e-3.  Prints "ggml shim ok" and exits 0, or
// names the first failed check and exits 1.
#include "qkv_ggml.hpp"
#include "../oracle/qkv_oracle.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

using qkv::ggml::tensor;
namespace G = qkv::ggml;

#define CHECK(c)                                                                  \
    do {                                                                          \
        if (!(c)) {                                                               \
            std::fprintf(stderr, "check failed line %d: %s\n", __LINE__, #c);     \
            return 1;                                                             \
        }                                                                         \
    } while (0)

static constexpr int HD = 256, NH = 16, NKV = 2, KVD = NKV * HD;

static std::vector<float> normals(uint64_t seed, size_t n) {
    std::mt19937_64 g(seed);
    std::normal_distribution<float> d(0.0f, 1.0f);
    std::vector<float> v(n);
    for (auto &x : v) x = d(g);
    return v;
}
static uint16_t to_bf16(float f) {   // round to nearest even
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
static float from_bf16(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
template <typename T>
static T *dev_copy(const std::vector<T> &h) {
    T *d = nullptr;
    if (cudaMalloc(&d, h.size() * sizeof(T)) != cudaSuccess) return nullptr;
    cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice);
    return d;
}
static bool close_to(const std::vector<float> &got, const std::vector<float> &ref, const char *what) {
    double worst = 0;
    size_t bad = 0;
    for (size_t i = 0; i < got.size(); i++) {
        const double e = std::fabs((double)got[i] - ref[i]);
        worst = std::max(worst, e);
        if (!(e <= 2e-3 + 1e-3 * std::fabs((double)ref[i]))) bad++;
    }
    std::printf("%s: max err %.3e, %zu of %zu outside\n", what, worst, bad, got.size());
    return bad == 0;
}

// Every malformed operand is refused before anything is launched (works on a host-only engine).
static int rejections(qkv_engine *eng, const qkv_config &cfg) {
    std::string err;
    int32_t dummy[4];
    const int T = 3;
    tensor Q = G::make(G::TYPE_F32, dummy, HD, NH, T);   // roped query [hd, n_head, T]
    tensor q = G::permute_0213(Q);
    tensor k = G::cache_view(dummy, HD, 100 + T, NKV), v = k;
    tensor dst = G::make(G::TYPE_F32, dummy, HD, NH, T);
    tensor kn = G::make(G::TYPE_F32, dummy, KVD, T), vn = kn;
    G::attn_params p;
    // a query that is not the permuted view
    CHECK(!G::attn_decode(eng, cfg, Q, k, v, &kn, &vn, dst, p, err) && err.find("q:") == 0);
    tensor qb = q;
    qb.type = G::TYPE_F16;
    CHECK(!G::attn_decode(eng, cfg, qb, k, v, &kn, &vn, dst, p, err) && err.find("q:") == 0);
    // a cache view with other strides (e.g. head-major) or type
    tensor kh = k;
    std::swap(kh.nb[1], kh.nb[2]);
    CHECK(!G::attn_decode(eng, cfg, q, kh, v, &kn, &vn, dst, p, err) && err.find("k/v:") == 0);
    tensor kf = k;
    kf.type = G::TYPE_F16;
    CHECK(!G::attn_decode(eng, cfg, q, kf, v, &kn, &vn, dst, p, err) && err.find("k/v:") == 0);
    // k and v of different lengths; more than 4 tokens; dst not contiguous
    tensor v2 = G::cache_view(dummy, HD, 100 + T + 1, NKV);
    CHECK(!G::attn_decode(eng, cfg, q, k, v2, &kn, &vn, dst, p, err));
    tensor Q5 = G::make(G::TYPE_F32, dummy, HD, NH, 5);
    tensor d5 = G::make(G::TYPE_F32, dummy, HD, NH, 5);
    tensor k5 = G::cache_view(dummy, HD, 105, NKV);
    CHECK(!G::attn_decode(eng, cfg, G::permute_0213(Q5), k5, k5, nullptr, nullptr, d5, p, err));
    tensor dp = G::permute_0213(dst);
    CHECK(!G::attn_decode(eng, cfg, q, k, v, &kn, &vn, dp, p, err) && err.find("dst") == 0);
    // only one of the new rows; new rows of the wrong size
    CHECK(!G::attn_decode(eng, cfg, q, k, v, &kn, nullptr, dst, p, err));
    tensor kn2 = G::make(G::TYPE_F32, dummy, KVD, T + 1);
    CHECK(!G::attn_decode(eng, cfg, q, k, v, &kn2, &vn, dst, p, err) && err.find("new K/V") == 0);
    // positions the slot does not hold: its cache is empty, the step claims 100 before it
    CHECK(!G::attn_decode(eng, cfg, q, k, v, &kn, &vn, dst, p, err));
    // prefill: F32 queries (the dense path takes bf16)
    CHECK(!G::attn_prefill(eng, cfg, q, k, v, kn, vn, dst, p, err) && err.find("q:") == 0);
    return 0;
}

static int on_device(qkv_engine *eng, const qkv_config &cfg) {
    std::string err;
    const int C = 512, N0 = 2 * C, T = 3;   // two prefill chunks, then a verify step
    G::attn_params p;
    p.layer = 1;
    p.slot = 0;
    p.scale = 1.0f / 16.0f;
    std::vector<float> Kf = normals(1, (size_t)(N0 + T) * KVD), Vf = normals(2, (size_t)(N0 + T) * KVD);
    std::vector<float> Qp = normals(3, (size_t)N0 * NH * HD), Qd = normals(4, (size_t)T * NH * HD);
    std::vector<uint16_t> Qb(Qp.size());
    for (size_t i = 0; i < Qp.size(); i++) Qb[i] = to_bf16(Qp[i]);
    float *dK = dev_copy(Kf), *dV = dev_copy(Vf), *dQd = dev_copy(Qd);
    uint16_t *dQb = dev_copy(Qb);
    float *dOut = nullptr;
    CHECK(dK && dV && dQd && dQb && cudaMalloc(&dOut, (size_t)N0 * NH * HD * 4) == cudaSuccess);
    // prefill, chunk by chunk, as sparse_attn does per chunk: ggml_cast(Q, BF16), permute, the cache
    // views over n_past + Tc cells, the chunk's K/V rows
    for (int c = 0; c < N0 / C; c++) {
        tensor Q = G::make(G::TYPE_BF16, dQb + (size_t)c * C * NH * HD, HD, NH, C);
        tensor kv = G::cache_view(nullptr, HD, (int64_t)(c + 1) * C, NKV);
        tensor kn = G::make(G::TYPE_F32, dK + (size_t)c * C * KVD, HD, NKV, C);
        tensor vn = G::make(G::TYPE_F32, dV + (size_t)c * C * KVD, HD, NKV, C);
        tensor dst = G::make(G::TYPE_F32, dOut + (size_t)c * C * NH * HD, HD, NH, C);
        if (!G::attn_prefill(eng, cfg, G::permute_0213(Q), kv, kv, kn, vn, dst, p, err)) {
            std::fprintf(stderr, "prefill chunk %d: %s\n", c, err.c_str());
            return 1;
        }
    }
    // the decode step: set_rows of the 3 rows + flash_attn_ext over n_kv = N0 + 3
    float *dOd = nullptr;
    CHECK(cudaMalloc(&dOd, (size_t)T * NH * HD * 4) == cudaSuccess);
    {
        tensor Q = G::make(G::TYPE_F32, dQd, HD, NH, T);
        tensor kv = G::cache_view(nullptr, HD, N0 + T, NKV);
        tensor kn = G::make(G::TYPE_F32, dK + (size_t)N0 * KVD, KVD, T);
        tensor vn = G::make(G::TYPE_F32, dV + (size_t)N0 * KVD, KVD, T);
        tensor dst = G::make(G::TYPE_F32, dOd, HD, NH, T);
        if (!G::attn_decode(eng, cfg, G::permute_0213(Q), kv, kv, &kn, &vn, dst, p, err)) {
            std::fprintf(stderr, "decode: %s\n", err.c_str());
            return 1;
        }
    }
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    int32_t status = -1;
    CHECK(qkv_device_status(eng, nullptr, &status) == QKV_OK && status == 0);
    // the cache rows as ggml holds them, then the oracle
    const int N = N0 + T, row = NKV * HD / 32 * 34;
    uint8_t *dKr = nullptr, *dVr = nullptr;
    CHECK(cudaMalloc(&dKr, (size_t)N * row) == cudaSuccess && cudaMalloc(&dVr, (size_t)N * row) == cudaSuccess);
    CHECK(qkv_read_rows(eng, p.layer, p.slot, 0, N, dKr, dVr, nullptr) == QKV_OK);
    std::vector<uint8_t> Kr((size_t)N * row), Vr((size_t)N * row), Kq((size_t)N * row), Vq((size_t)N * row);
    CHECK(cudaMemcpy(Kr.data(), dKr, Kr.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(cudaMemcpy(Vr.data(), dVr, Vr.size(), cudaMemcpyDeviceToHost) == cudaSuccess);
    orc_quantize_rows_q8_0(Kf.data(), Kq.data(), N, KVD, 0);
    orc_quantize_rows_q8_0(Vf.data(), Vq.data(), N, KVD, 0);
    CHECK(Kr == Kq && Vr == Vq);   // every row the adapter wrote, bit-exact
    std::vector<float> got_p((size_t)N0 * NH * HD), got_d((size_t)T * NH * HD);
    CHECK(cudaMemcpy(got_p.data(), dOut, got_p.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(cudaMemcpy(got_d.data(), dOd, got_d.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    std::vector<float> qv(Qb.size());
    for (size_t i = 0; i < Qb.size(); i++) qv[i] = from_bf16(Qb[i]);
    std::vector<int32_t> pos(N0);
    for (int i = 0; i < N0; i++) pos[i] = i;
    std::vector<float> ref_p(got_p.size()), ref_d(got_d.size());
    orc_attn_q8_0(qv.data(), N0, NH, NKV, HD, Kq.data(), Vq.data(), nullptr, N0, pos.data(), p.scale, ref_p.data(), 0);
    const int32_t pd[T] = {N0, N0 + 1, N0 + 2};
    orc_attn_q8_0(Qd.data(), T, NH, NKV, HD, Kq.data(), Vq.data(), nullptr, N, pd, p.scale, ref_d.data(), 0);
    CHECK(close_to(got_p, ref_p, "prefill through the adapter"));
    CHECK(close_to(got_d, ref_d, "decode through the adapter"));
    cudaFree(dK); cudaFree(dV); cudaFree(dQd); cudaFree(dQb); cudaFree(dOut); cudaFree(dOd); cudaFree(dKr); cudaFree(dVr);
    return 0;
}

int main(int argc, char **argv) {
    const int device = argc > 1 ? std::atoi(argv[1]) : -1;
    qkv_config cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cfg.n_layer = 2; cfg.n_head = NH; cfg.n_head_kv = NKV; cfg.head_dim = HD;
    cfg.n_ctx = 2048; cfg.n_slots = 1;
    qkv_engine *eng = nullptr;
    CHECK(qkv_create(&cfg, device, &eng) == QKV_OK);
    CHECK(qkv_seq_alloc(eng, 0) == QKV_OK);
    int rc = rejections(eng, cfg);
    if (!rc && device >= 0) rc = on_device(eng, cfg);
    qkv_destroy(eng);
    if (!rc) std::printf("ggml shim ok (device %d)\n", device);
    return rc;
}
