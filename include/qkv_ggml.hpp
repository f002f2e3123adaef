/* qkv_ggml.hpp -- header-only adapter from the reference's ggml attention nodes to the C ABI.
 *
 * The reference builds, per full-attention layer, a q8_0 cache write followed by
 * ggml_flash_attn_ext(q, k, v, mask, 1/sqrt(hd), 0, 0) with F32 accumulation:
 *   decode : qsa_dec_kv_write's ggml_set_rows + the flash_attn_ext of sparse_attn_decode
 *            (src/qwfn_graph.cpp:612-628, 697-699)
 *   prefill: kv_append's ggml_cpy + the flash_attn_ext of sparse_attn
 *            (src/qwfn_graph.cpp:370-384, 454-471)
 * with q = ggml_permute(Q, 0, 2, 1, 3) of the roped F32 query [hd, n_head, T] and k/v the cache
 * views ggml_view_3d(cache, hd, n_kv, n_head_kv, row_size(kv_dim), row_size(hd), 0)
 * (src/qwfn_graph.cpp:458-464).  A ggml custom op (ggml_map_custom3 and friends) that replaces
 * those nodes receives exactly these tensors; this header checks that they are the views the
 * reference builds and calls qkv_append_attn_decode / qkv_attn_decode / qkv_append /
 * qkv_attn_prefill on them.  ggml itself is not needed: `tensor` mirrors the ggml_tensor fields
 * the adapter reads (type, ne, nb, data), and a custom-op callback fills one from each operand.
 *
 * The cache views carry no usable data pointer here -- the cache lives in the engine's pages --
 * only their shape: n_kv = k.ne[1] must be the sequence's positions after the step
 * (n_past + T, src/qwfn_graph.cpp:426), which fixes where the step's rows go and what they see.
 * The causal kq_mask of the reference (src/qwfn_engine.cpp:1238-1274) is what the kernels apply
 * implicitly: query t of the step sees cells 0 .. n_past + t.
 *
 * Error convention as the reference's: bool + std::string &err, nothing aborts.
 */
#ifndef QKV_GGML_HPP
#define QKV_GGML_HPP

#include "qkv.h"

#include <cstdint>
#include <string>

namespace qkv {
namespace ggml {

/* ggml's type ids (enum ggml_type, ggml.h) of the operand types involved. */
enum : int32_t { TYPE_F32 = 0, TYPE_F16 = 1, TYPE_Q8_0 = 8, TYPE_BF16 = 30 };

/* The fields of a ggml_tensor the adapter reads: element type, extents ne[0..3] (ne[0] fastest)
 * and byte strides nb[0..3], and the device address. */
struct tensor {
    int32_t type = TYPE_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    size_t  nb[4] = {0, 0, 0, 0};
    void   *data = nullptr;
};

/* A contiguous tensor of `type` with extents ne0..ne3 (what ggml_new_tensor_4d makes). */
inline tensor make(int32_t type, void *data, int64_t ne0, int64_t ne1 = 1, int64_t ne2 = 1, int64_t ne3 = 1) {
    tensor t;
    t.type = type;
    t.data = data;
    t.ne[0] = ne0; t.ne[1] = ne1; t.ne[2] = ne2; t.ne[3] = ne3;
    const size_t es = type == TYPE_F32 ? 4 : 2;
    t.nb[0] = es;
    t.nb[1] = es * (size_t)ne0;
    t.nb[2] = t.nb[1] * (size_t)ne1;
    t.nb[3] = t.nb[2] * (size_t)ne2;
    return t;
}

/* ggml_permute(t, 0, 2, 1, 3): swap axes 1 and 2 (a view; no data moves). */
inline tensor permute_0213(const tensor &t) {
    tensor p = t;
    p.ne[1] = t.ne[2]; p.ne[2] = t.ne[1];
    p.nb[1] = t.nb[2]; p.nb[2] = t.nb[1];
    return p;
}

/* The K or V cache view of src/qwfn_graph.cpp:458-464 for n_kv positions: q8_0 [hd, n_kv,
 * n_head_kv] with token stride row_size(kv_dim) and head stride row_size(hd).  data: any
 * address that identifies the cache (the adapter does not read it). */
inline tensor cache_view(void *data, int64_t head_dim, int64_t n_kv, int64_t n_head_kv) {
    tensor t;
    t.type = TYPE_Q8_0;
    t.data = data;
    t.ne[0] = head_dim; t.ne[1] = n_kv; t.ne[2] = n_head_kv; t.ne[3] = 1;
    const size_t head_row = (size_t)head_dim / 32 * 34;   // ggml_row_size(Q8_0, hd)
    t.nb[0] = 34;                                          // ggml_type_size(Q8_0)
    t.nb[1] = head_row * (size_t)n_head_kv;               // ggml_row_size(Q8_0, kv_dim)
    t.nb[2] = head_row;
    t.nb[3] = t.nb[1] * (size_t)n_kv;
    return t;
}

/* The op's parameters: the engine layer (the attention layer's index in the engine) and slot,
 * the scale the graph passes (1/sqrt(hd) in the reference), the device stream. */
struct attn_params {
    int32_t layer = 0;
    int32_t slot = 0;
    float   scale = 0.0625f;
    void   *stream = nullptr;
};

namespace detail {
inline bool fail(std::string &err, const char *what) {
    err = what;
    return false;
}
inline bool status(qkv_engine *eng, qkv_status st, std::string &err) {
    if (st == QKV_OK) return true;
    err = std::string(qkv_status_string(st)) + ": " + qkv_last_error(eng);
    return false;
}
/* q = permute(Q [hd, n_head, T]) of element size es: ne [hd, T, n_head], head stride hd*es, token
 * stride n_head*hd*es -- the memory of a contiguous [T][n_head][hd] array, the C ABI's layout. */
inline bool query_ok(const tensor &q, int32_t type, size_t es, int64_t hd, std::string &err) {
    if (q.type != type || !q.data) return fail(err, "q: wrong type or no data");
    if (q.ne[0] != hd || q.ne[3] != 1) return fail(err, "q: ne[0] must be head_dim and ne[3] 1");
    if (q.nb[0] != es || q.nb[2] != es * (size_t)hd || q.nb[1] != es * (size_t)hd * (size_t)q.ne[2])
        return fail(err, "q: not the permuted [hd, n_head, T] query view (make it contiguous first)");
    return true;
}
inline bool cache_ok(const tensor &k, int64_t hd, int64_t n_head_kv, std::string &err) {
    const tensor want = cache_view(nullptr, hd, k.ne[1], n_head_kv);
    if (k.type != TYPE_Q8_0) return fail(err, "k/v: the cache must be q8_0");
    for (int i = 0; i < 3; i++)
        if (k.ne[i] != want.ne[i] || k.nb[i] != want.nb[i])
            return fail(err, "k/v: not the cache view [hd, n_kv, n_head_kv] of src/qwfn_graph.cpp:458-464");
    return true;
}
/* new rows: F32 [kv_dim, T] or [hd, n_head_kv, T], contiguous */
inline bool rows_ok(const tensor &r, int64_t kv_dim, int64_t T, std::string &err) {
    if (r.type != TYPE_F32 || !r.data) return fail(err, "new K/V rows: F32 with data");
    const int64_t n = r.ne[0] * r.ne[1] * r.ne[2] * r.ne[3];
    if (n != kv_dim * T || r.nb[0] != 4 || r.nb[1] != 4 * (size_t)r.ne[0] || r.nb[2] != r.nb[1] * (size_t)r.ne[1])
        return fail(err, "new K/V rows: contiguous F32 [kv_dim, T]");
    return true;
}
inline bool dst_ok(const tensor &d, int64_t hd, int64_t n_head, int64_t T, std::string &err) {
    if (d.type != TYPE_F32 || !d.data || d.ne[0] != hd || d.ne[1] != n_head || d.ne[2] != T || d.ne[3] != 1)
        return fail(err, "dst: F32 [hd, n_head, T] (flash_attn_ext's result)");
    if (d.nb[0] != 4 || d.nb[1] != 4 * (size_t)hd || d.nb[2] != 4 * (size_t)hd * (size_t)n_head)
        return fail(err, "dst: must be contiguous");
    return true;
}
inline bool seq_len(qkv_engine *eng, int32_t slot, int32_t &n, std::string &err) {
    return status(eng, qkv_seq_length(eng, slot, &n), err);
}
}  // namespace detail

/* Decode / MTP verify: the step's T (1..4) query tokens at positions n_kv - T .. n_kv - 1.
 * With k_new and v_new (F32 [kv_dim, T], the roped K and the V of the step) the rows are
 * quantised into the cache and attended in one launch, as set_rows + flash_attn_ext do;
 * without them the rows must already be in the cache. */
inline bool attn_decode(qkv_engine *eng, const qkv_config &cfg, const tensor &q, const tensor &k, const tensor &v,
                        const tensor *k_new, const tensor *v_new, tensor &dst, const attn_params &p, std::string &err) {
    using namespace detail;
    if (!eng) return fail(err, "null engine");
    const int64_t hd = cfg.head_dim, nh = cfg.n_head, nh_kv = cfg.n_head_kv;
    if (!query_ok(q, TYPE_F32, 4, hd, err) || !cache_ok(k, hd, nh_kv, err) || !cache_ok(v, hd, nh_kv, err)) return false;
    const int64_t T = q.ne[1];
    if (q.ne[2] != nh) return fail(err, "q: ne[2] must be n_head");
    if (T < 1 || T > 4) return fail(err, "decode: 1..4 query tokens per step");
    if (k.ne[1] != v.ne[1]) return fail(err, "k and v views of different lengths");
    if (!dst_ok(dst, hd, nh, T, err)) return false;
    const int64_t n_kv = k.ne[1], pos0 = n_kv - T;
    if (pos0 < 0) return fail(err, "decode: n_kv shorter than the step");
    int32_t n_past = 0;
    if (!seq_len(eng, p.slot, n_past, err)) return false;
    const int32_t slot = p.slot, pos = (int32_t)pos0;
    if ((k_new != nullptr) != (v_new != nullptr)) return fail(err, "decode: both new K and new V, or neither");
    if (k_new) {
        if (!rows_ok(*k_new, hd * nh_kv, T, err) || !rows_ok(*v_new, hd * nh_kv, T, err)) return false;
        if (pos0 > n_past) return fail(err, "decode: the step's first position is past the cache's end");
        return status(eng,
                      qkv_append_attn_decode(eng, p.layer, &slot, &pos, 1, static_cast<const float *>(k_new->data),
                                             static_cast<const float *>(v_new->data),
                                             static_cast<const float *>(q.data), (int32_t)T, p.scale,
                                             static_cast<float *>(dst.data), p.stream),
                      err);
    }
    if (n_kv > n_past) return fail(err, "decode: n_kv exceeds the positions in the cache");
    return status(eng,
                  qkv_attn_decode(eng, p.layer, &slot, &pos, 1, static_cast<const float *>(q.data), (int32_t)T,
                                  p.scale, nullptr, 0, static_cast<float *>(dst.data), p.stream),
                  err);
}

/* Prefill chunk: kv_append's ggml_cpy of the chunk's F32 K and V rows into the cache at
 * n_past, then the causal flash_attn_ext of its Tc queries over all n_kv = n_past + Tc cells.
 * q must be BF16 (a ggml_cast of the roped query before the permute), the type the dense tcgen05
 * path takes. */
inline bool attn_prefill(qkv_engine *eng, const qkv_config &cfg, const tensor &q, const tensor &k, const tensor &v,
                         const tensor &k_new, const tensor &v_new, tensor &dst, const attn_params &p, std::string &err) {
    using namespace detail;
    if (!eng) return fail(err, "null engine");
    const int64_t hd = cfg.head_dim, nh = cfg.n_head, nh_kv = cfg.n_head_kv;
    if (!query_ok(q, TYPE_BF16, 2, hd, err) || !cache_ok(k, hd, nh_kv, err) || !cache_ok(v, hd, nh_kv, err)) return false;
    const int64_t Tc = q.ne[1];
    if (q.ne[2] != nh) return fail(err, "q: ne[2] must be n_head");
    if (k.ne[1] != v.ne[1]) return fail(err, "k and v views of different lengths");
    if (!dst_ok(dst, hd, nh, Tc, err) || !rows_ok(k_new, hd * nh_kv, Tc, err) || !rows_ok(v_new, hd * nh_kv, Tc, err))
        return false;
    const int64_t pos0 = k.ne[1] - Tc;
    int32_t n_past = 0;
    if (!seq_len(eng, p.slot, n_past, err)) return false;
    if (pos0 < 0 || pos0 > n_past) return fail(err, "prefill: the chunk does not continue the cache");
    if (!status(eng, qkv_append(eng, p.layer, p.slot, (int32_t)pos0, static_cast<const float *>(k_new.data),
                                static_cast<const float *>(v_new.data), (int32_t)Tc, p.stream), err))
        return false;
    return status(eng, qkv_attn_prefill(eng, p.layer, p.slot, (int32_t)pos0, static_cast<const uint16_t *>(q.data),
                                        (int32_t)Tc, p.scale, static_cast<float *>(dst.data), p.stream),
                  err);
}

}  // namespace ggml
}  // namespace qkv

#endif  // QKV_GGML_HPP
