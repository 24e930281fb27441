// evk_ai_dispatch.h — shape logic of the evk::ai operators, written once over
// a table of C-ABI entry points.  The product (evk_ai.cpp) instantiates it
// with libevkcu; the oracle's reference-test harness instantiates it with the
// CPU oracle, so both see identical argument derivation.
//
// Each op derives its arguments from Tensor shapes exactly as the reference
// host code does (evk_ai.cpp lines cited per function) and reports a failing
// status through Backend::fail, which the product makes fatal (the reference
// fails fast through assert / EVK_ASSERT).
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "evkcu.h"

namespace evk_b200 {

struct Backend {
    void* (*stream)();
    void (*fail)(int status, const char* op);
    int (*matmul)(const void*, const void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, uint64_t, uint64_t,
                  uint64_t, uint32_t, int, void*);
    int (*flash_attention)(const void*, const void*, const void*, void*, uint32_t, uint32_t, uint32_t, uint32_t,
                           uint32_t, float, uint32_t, int, void*);
    int (*single_query_attention)(const void*, const void*, const void*, void*, uint32_t, uint32_t, uint32_t,
                                  uint32_t, uint32_t, uint32_t, float, int, void*);
    int (*rms_norm)(const void*, void*, const void*, uint32_t, uint32_t, float, int, void*);
    int (*rope)(const void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, float, int, void*);
    int (*gelu)(const void*, void*, uint64_t, int, void*);
    int (*softmax)(const void*, void*, uint32_t, uint32_t, float, int, void*);
    int (*add)(const void*, const void*, void*, uint64_t, int, void*);
    int (*scale)(void*, uint64_t, float, int, void*);
    int (*zero)(void*, uint64_t, int, void*);
    int (*causal_mask)(void*, uint32_t, uint32_t, int, void*);
    int (*embed)(const void*, const void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, int, void*);
    int (*greedy_sample)(const void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, int,
                         void*);
    // training side
    int (*relu)(const void*, void*, uint64_t, int, void*);
    int (*relu_backward)(const void*, const void*, void*, uint64_t, int, void*);
    int (*gelu_backward)(const void*, const void*, void*, uint64_t, int, void*);
    int (*softmax_backward)(const void*, const void*, void*, uint32_t, uint32_t, float, int, void*);
    int (*rms_norm_backward)(const void*, const void*, void*, uint32_t, uint32_t, float, int, void*);
    int (*rope_backward)(const void*, void*, uint32_t, uint32_t, uint32_t, float, int, void*);
    int (*embed_backward)(const void*, const void*, void*, uint32_t, uint32_t, uint32_t, uint32_t, int, void*);
    int (*position_add)(const void*, const void*, void*, uint32_t, uint32_t, uint32_t, int, void*);
    int (*position_add_backward)(const void*, void*, void*, uint32_t, uint32_t, uint32_t, int, void*);
    int (*sum_batch)(const void*, void*, uint32_t, uint64_t, int, void*);
    int (*sgd)(void*, const void*, uint64_t, float, int, void*);
    int (*adam)(void*, const void*, void*, void*, uint64_t, uint32_t, float, float, float, float, int, void*);
    int (*mse_loss)(const void*, const void*, void*, void*, uint64_t, int, void*);
    int (*cross_entropy_loss)(const void*, const void*, void*, void*, uint32_t, uint32_t, uint32_t, int, void*);
    int (*flash_attention_bwd)(const void*, const void*, const void*, const void*, const void*, void*, void*, void*,
                               uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, float, uint32_t, int, void*);
};

template <class T>
inline const void* dptr(T& t) {
    return reinterpret_cast<const void*>(t.buffer.GetReference());
}
template <class T>
inline void* dmut(T& t) {
    return reinterpret_cast<void*>(t.buffer.GetReference());
}

inline void check(const Backend& be, int st, const char* op) {
    if (st != EVKCU_OK) be.fail(st, op);
}

// evk_ai.cpp:254-330: batch = max of the leading-dims products of A, B, C;
// logical dims from the transpose flags; a batch extent of 1 broadcasts
// (stride 0) an input; C is never broadcast.
template <class T>
void matmul(const Backend& be, T& a, T& b, T& c, bool ta, bool tb, bool acc, int dtype = EVKCU_F16) {
    if (a.shape.rank() < 2 || b.shape.rank() < 2 || c.shape.rank() < 2) return be.fail(EVKCU_BAD_SHAPE, "matmul: rank < 2");
    const uint32_t batchA = a.shape.rank() >= 3 ? a.shape.batch_size(2) : 1u;
    const uint32_t batchB = b.shape.rank() >= 3 ? b.shape.batch_size(2) : 1u;
    const uint32_t batchC = c.shape.rank() >= 3 ? c.shape.batch_size(2) : 1u;
    const uint32_t batch = std::max({batchA, batchB, batchC});
    const uint32_t a_rows = ta ? a.shape[-1] : a.shape[-2], a_cols = ta ? a.shape[-2] : a.shape[-1];
    const uint32_t b_rows = tb ? b.shape[-1] : b.shape[-2], b_cols = tb ? b.shape[-2] : b.shape[-1];
    if (a_cols != b_rows || c.shape[-2] != a_rows || c.shape[-1] != b_cols ||
        (batchA != batch && batchA != 1u) || (batchB != batch && batchB != 1u) || batchC != batch)
        return be.fail(EVKCU_BAD_SHAPE, "matmul: incompatible shapes");
    const uint64_t eA = (uint64_t)a.shape[-2] * a.shape[-1], eB = (uint64_t)b.shape[-2] * b.shape[-1];
    const uint64_t eC = (uint64_t)c.shape[-2] * c.shape[-1];
    const uint64_t sA = (batchA == 1u && batch > 1u) ? 0 : eA;
    const uint64_t sB = (batchB == 1u && batch > 1u) ? 0 : eB;
    const uint32_t flags = (ta ? EVKCU_MM_TRANSPOSE_A : 0u) | (tb ? EVKCU_MM_TRANSPOSE_B : 0u) | (acc ? EVKCU_MM_ACC_C : 0u);
    check(be, be.matmul(dptr(a), dptr(b), dmut(c), batch, a_rows, a_cols, b_cols, sA, sB, eC, flags, dtype, be.stream()),
          "matmul");
}

// evk_ai.cpp:332-369: Q, O (B, N, D = H*Dh); K, V (B, N, Dh); scale 1/sqrt(Dh).
template <class T>
void flash_attention(const Backend& be, T& q, T& k, T& v, T& o, int dtype = EVKCU_F16) {
    if (q.shape.rank() != 3 || k.shape.rank() != 3 || v.shape.rank() != 3 || o.shape.rank() != 3)
        return be.fail(EVKCU_BAD_SHAPE, "flash_attention: tensors must be rank 3");
    const uint32_t B = q.shape[0], N = q.shape[1], D = q.shape[2], Dh = k.shape[2];
    if (k.shape[0] != B || k.shape[1] != N || v.shape[0] != B || v.shape[1] != N || v.shape[2] != Dh ||
        o.shape[0] != B || o.shape[1] != N || o.shape[2] != D || Dh == 0 || D % Dh != 0)
        return be.fail(EVKCU_BAD_SHAPE, "flash_attention: incompatible shapes");
    const uint32_t H = D / Dh;
    check(be, be.flash_attention(dptr(q), dptr(k), dptr(v), dmut(o), B, N, H, 1, Dh, 1.0f / std::sqrt((float)Dh), 0, dtype,
                                 be.stream()),
          "flash_attention");
}

template <class T>
bool same_shape(T& a, T& b) {
    if (a.shape.rank() != b.shape.rank()) return false;
    for (uint32_t i = 0; i < a.shape.rank(); ++i)
        if (a.shape[(int)i] != b.shape[(int)i]) return false;
    return true;
}

// evk_ai.cpp:568-591
template <class T>
void add(const Backend& be, T& a, T& b, T& c, int dtype = EVKCU_F16) {
    if (!same_shape(a, b) || !same_shape(a, c)) return be.fail(EVKCU_BAD_SHAPE, "add: shape mismatch");
    check(be, be.add(dptr(a), dptr(b), dmut(c), a.shape.count(), dtype, be.stream()), "add");
}

// evk_ai.cpp:593-613: rows = count / last dim.
template <class T>
void softmax(const Backend& be, T& in, T& out, float scale, int dtype = EVKCU_F16) {
    if (!same_shape(in, out)) return be.fail(EVKCU_BAD_SHAPE, "softmax: shape mismatch");
    const uint32_t L = in.shape[-1];
    check(be, be.softmax(dptr(in), dmut(out), in.shape.count() / L, L, scale, dtype, be.stream()), "softmax");
}

// evk_ai.cpp:679-699
template <class T>
void gelu(const Backend& be, T& in, T& out, int dtype = EVKCU_F16) {
    if (!same_shape(in, out)) return be.fail(EVKCU_BAD_SHAPE, "gelu: shape mismatch");
    check(be, be.gelu(dptr(in), dmut(out), in.shape.count(), dtype, be.stream()), "gelu");
}

// evk_ai.cpp:782-806: embeddings (V, D); indices any shape of uint16 ids.
template <class T>
void embed(const Backend& be, T& E, T& idx, T& out, uint32_t idx_bytes = 2, int dtype = EVKCU_F16) {
    if (E.shape.rank() != 2) return be.fail(EVKCU_BAD_SHAPE, "embed: embeddings must be rank 2");
    const uint32_t V = E.shape[0], D = E.shape[1];
    const uint32_t n = idx_bytes == 2 ? idx.shape.count() : idx.shape.count() / 2;
    if (out.shape.count() != n * D) return be.fail(EVKCU_BAD_SHAPE, "embed: output size mismatch");
    check(be, be.embed(dptr(E), dptr(idx), dmut(out), V, D, n, idx_bytes, dtype, be.stream()), "embed");
}

// evk_ai.cpp:808-837: logits (B, S, V), out (B) uint16 ids.
template <class T>
void greedy_sample(const Backend& be, T& logits, T& out, uint32_t position, uint32_t token_base, uint32_t token_count,
                   uint32_t out_bytes = 2, int dtype = EVKCU_F16) {
    if (logits.shape.rank() != 3 || out.shape.rank() != 1) return be.fail(EVKCU_BAD_SHAPE, "greedy_sample: ranks");
    const uint32_t B = logits.shape[0], S = logits.shape[1], V = logits.shape[2];
    if (out.shape[0] * 2 / out_bytes < B) return be.fail(EVKCU_BAD_SHAPE, "greedy_sample: output too small");
    check(be, be.greedy_sample(dptr(logits), dmut(out), B, S, V, position, token_base, token_count, out_bytes, dtype,
                               be.stream()),
          "greedy_sample");
}

// evk_ai.cpp:862-882: square last two dims.
template <class T>
void apply_causal_mask(const Backend& be, T& s, int dtype = EVKCU_F16) {
    const uint32_t N = s.shape[-1];
    if (s.shape.rank() < 2 || s.shape[-2] != N) return be.fail(EVKCU_BAD_SHAPE, "apply_causal_mask: not square");
    check(be, be.causal_mask(dmut(s), s.shape.count() / (N * N), N, dtype, be.stream()), "apply_causal_mask");
}

// evk_ai.cpp:945-966 (head_dim = embed_dim, no offset, as the reference).
template <class T>
void rope(const Backend& be, T& in, T& out, uint32_t B, uint32_t S, uint32_t D, float base, uint32_t head_dim = 0,
          uint32_t pos_offset = 0, int dtype = EVKCU_F16) {
    check(be, be.rope(dptr(in), dmut(out), B, S, D, head_dim ? head_dim : D, pos_offset, base, dtype, be.stream()),
          "rope");
}

// evk_ai.cpp:992-1007 / 1010-1024
template <class T>
void scale(const Backend& be, T& t, float s, int dtype = EVKCU_F16) {
    check(be, be.scale(dmut(t), t.shape.count(), s, dtype, be.stream()), "scale");
}
template <class T>
void zero(const Backend& be, T& t, int dtype = EVKCU_F16) {
    check(be, be.zero(dmut(t), t.shape.count(), dtype, be.stream()), "zero");
}

// evk_ai.cpp:1045-1067: rows = count / last dim.
template <class T>
void rms_norm(const Backend& be, T& in, T& out, float eps, const void* gamma = nullptr, int dtype = EVKCU_F16) {
    if (!same_shape(in, out)) return be.fail(EVKCU_BAD_SHAPE, "rms_norm: shape mismatch");
    const uint32_t D = in.shape[-1];
    check(be, be.rms_norm(dptr(in), dmut(out), gamma, in.shape.count() / D, D, eps, dtype, be.stream()), "rms_norm");
}

// ------------------------------------------------------------ training side --
// evk_ai.cpp:635-677, 700-720: elementwise over the input's element count.
template <class T>
void relu(const Backend& be, T& in, T& out, int dtype = EVKCU_F16) {
    if (!same_shape(in, out)) return be.fail(EVKCU_BAD_SHAPE, "relu: shape mismatch");
    check(be, be.relu(dptr(in), dmut(out), in.shape.count(), dtype, be.stream()), "relu");
}
template <class T>
void relu_backward(const Backend& be, T& go, T& in, T& gi, int dtype = EVKCU_F16) {
    if (go.shape.count() != in.shape.count() || gi.shape.count() != in.shape.count())
        return be.fail(EVKCU_BAD_SHAPE, "relu_backward: size mismatch");
    check(be, be.relu_backward(dptr(go), dptr(in), dmut(gi), in.shape.count(), dtype, be.stream()), "relu_backward");
}
template <class T>
void gelu_backward(const Backend& be, T& go, T& in, T& gi, int dtype = EVKCU_F16) {
    if (go.shape.count() != in.shape.count() || gi.shape.count() != in.shape.count())
        return be.fail(EVKCU_BAD_SHAPE, "gelu_backward: size mismatch");
    check(be, be.gelu_backward(dptr(go), dptr(in), dmut(gi), in.shape.count(), dtype, be.stream()), "gelu_backward");
}
// evk_ai.cpp:614-633: rows = count / last dim of probs.
template <class T>
void softmax_backward(const Backend& be, T& probs, T& go, T& gi, float scale, int dtype = EVKCU_F16) {
    const uint32_t L = probs.shape[-1];
    if (go.shape.count() != probs.shape.count() || gi.shape.count() != probs.shape.count())
        return be.fail(EVKCU_BAD_SHAPE, "softmax_backward: size mismatch");
    check(be, be.softmax_backward(dptr(probs), dptr(go), dmut(gi), probs.shape.count() / L, L, scale, dtype,
                                  be.stream()),
          "softmax_backward");
}
// evk_ai.cpp:1068-1092
template <class T>
void rms_norm_backward(const Backend& be, T& in, T& go, T& gi, float eps, int dtype = EVKCU_F16) {
    const uint32_t D = in.shape[-1];
    if (go.shape.count() != in.shape.count() || gi.shape.count() != in.shape.count())
        return be.fail(EVKCU_BAD_SHAPE, "rms_norm_backward: size mismatch");
    check(be, be.rms_norm_backward(dptr(in), dptr(go), dmut(gi), in.shape.count() / D, D, eps, dtype, be.stream()),
          "rms_norm_backward");
}
// evk_ai.cpp:969-990
template <class T>
void rope_backward(const Backend& be, T& go, T& gi, uint32_t B, uint32_t S, uint32_t D, float base,
                   int dtype = EVKCU_F16) {
    if (D % 2 != 0) return be.fail(EVKCU_BAD_SHAPE, "rope_backward: odd embed_dim");
    check(be, be.rope_backward(dptr(go), dmut(gi), B, S, D, base, dtype, be.stream()), "rope_backward");
}
// evk_ai.cpp:839-859: grad_E (V, D); indices any shape of uint16 ids.
template <class T>
void embed_backward(const Backend& be, T& go, T& idx, T& gE, uint32_t idx_bytes = 2, int dtype = EVKCU_F16) {
    if (gE.shape.rank() != 2) return be.fail(EVKCU_BAD_SHAPE, "embed_backward: grad_embeddings must be rank 2");
    const uint32_t V = gE.shape[0], D = gE.shape[1];
    const uint32_t n = idx_bytes == 2 ? idx.shape.count() : idx.shape.count() / 2;
    if (go.shape.count() != n * D) return be.fail(EVKCU_BAD_SHAPE, "embed_backward: grad_out size mismatch");
    check(be, be.embed_backward(dptr(go), dptr(idx), dmut(gE), V, D, n, idx_bytes, dtype, be.stream()),
          "embed_backward");
}
// evk_ai.cpp:883-944
template <class T>
void position_add(const Backend& be, T& in, T& pos, T& out, uint32_t B, uint32_t S, uint32_t D,
                  int dtype = EVKCU_F16) {
    check(be, be.position_add(dptr(in), dptr(pos), dmut(out), B, S, D, dtype, be.stream()), "position_add");
}
template <class T>
void position_add_backward(const Backend& be, T& go, T& gi, T& gp, uint32_t B, uint32_t S, uint32_t D,
                           int dtype = EVKCU_F16) {
    check(be, be.position_add_backward(dptr(go), dmut(gi), dmut(gp), B, S, D, dtype, be.stream()),
          "position_add_backward");
}
// evk_ai.cpp:1024-1043
template <class T>
void sum_batch(const Backend& be, T& in, T& out, uint32_t batch, uint32_t size, int dtype = EVKCU_F16) {
    check(be, be.sum_batch(dptr(in), dmut(out), batch, size, dtype, be.stream()), "sum_batch");
}
// evk_ai.cpp:505-523
template <class T>
void sgd(const Backend& be, T& p, T& g, float lr, int dtype = EVKCU_F16) {
    if (!same_shape(p, g)) return be.fail(EVKCU_BAD_SHAPE, "sgd: shape mismatch");
    check(be, be.sgd(dmut(p), dptr(g), p.shape.count(), lr, dtype, be.stream()), "sgd");
}
// evk_ai.cpp:525-566: the caller owns the state and has incremented its step.
template <class T>
void adam(const Backend& be, T& p, T& g, void* m, void* v, uint32_t step, float lr, float b1, float b2, float eps,
          int dtype = EVKCU_F16) {
    if (!same_shape(p, g)) return be.fail(EVKCU_BAD_SHAPE, "adam: shape mismatch");
    check(be, be.adam(dmut(p), dptr(g), m, v, p.shape.count(), step, lr, b1, b2, eps, dtype, be.stream()), "adam");
}
// evk_ai.cpp:481-503
template <class T>
void mse_loss(const Backend& be, T& pred, T& tgt, T& grad, T& result, int dtype = EVKCU_F16) {
    if (!same_shape(pred, tgt) || result.shape.rank() != 1) return be.fail(EVKCU_BAD_SHAPE, "mse_loss: shapes");
    check(be, be.mse_loss(dptr(pred), dptr(tgt), dmut(grad), dmut(result), pred.shape.count(), dtype, be.stream()),
          "mse_loss");
}
// evk_ai.cpp:722-780: logits (rows, V), targets (rows) uint16 ids.
template <class T>
void cross_entropy_loss(const Backend& be, T& logits, T& tgt, T& grad, T& result, uint32_t target_bytes = 2,
                        int dtype = EVKCU_F16) {
    if (logits.shape.rank() != 2 || tgt.shape.rank() != 1 || result.shape.count() != 1)
        return be.fail(EVKCU_BAD_SHAPE, "cross_entropy_loss: ranks");
    const uint32_t rows = logits.shape[0], V = logits.shape[1];
    if (tgt.shape[0] * 2 / target_bytes != rows || grad.shape.count() != logits.shape.count())
        return be.fail(EVKCU_BAD_SHAPE, "cross_entropy_loss: shapes");
    check(be, be.cross_entropy_loss(dptr(logits), dptr(tgt), dmut(grad), dmut(result), rows, V, target_bytes, dtype,
                                    be.stream()),
          "cross_entropy_loss");
}
// evk_ai.cpp:371-473: Q, O, dO, dQ (B, N, D = H*Dh); K, V, dK, dV (B, N, Dh).
template <class T>
void flash_attention_bwd(const Backend& be, T& q, T& k, T& v, T& o, T& dO, T& dQ, T& dK, T& dV, uint32_t heads,
                         int dtype = EVKCU_F16) {
    if (q.shape.rank() != 3 || k.shape.rank() != 3 || dQ.shape.rank() != 3 || dK.shape.rank() != 3)
        return be.fail(EVKCU_BAD_SHAPE, "flash_attention_bwd: tensors must be rank 3");
    const uint32_t B = q.shape[0], N = q.shape[1], D = q.shape[2], Dh = k.shape[2];
    if (Dh == 0 || D % Dh != 0 || k.shape[0] != B || k.shape[1] != N || !same_shape(k, v) || !same_shape(q, dO) ||
        !same_shape(q, dQ) || !same_shape(k, dK) || !same_shape(k, dV) || (heads != 0 && heads != D / Dh))
        return be.fail(EVKCU_BAD_SHAPE, "flash_attention_bwd: incompatible shapes");
    check(be, be.flash_attention_bwd(dptr(q), dptr(k), dptr(v), dptr(o), dptr(dO), dmut(dQ), dmut(dK), dmut(dV), B, N,
                                     D / Dh, 1, Dh, 1.0f / std::sqrt((float)Dh), 0, dtype, be.stream()),
          "flash_attention_bwd");
}

}  // namespace evk_b200
