// evk_ai_ext.cpp — the extensions of evk_ai_ext.h over the C ABI, through the
// same shape logic (evk_ai_dispatch.h) and backend table as evk_ai.cpp.
#include "evk_ai_ext.h"

#include <cmath>

#include "evk_ai_dispatch.h"
#include "evkcu.h"

namespace evk_b200 {
const Backend& cpp_backend();  // evk_ai.cpp
}

namespace evk::ai {
namespace {
const evk_b200::Backend& be() { return evk_b200::cpp_backend(); }
int dt(DType d) { return static_cast<int>(d); }
}  // namespace

void matmul_ex(Tensor& a, Tensor& b, Tensor& c, bool ta, bool tb, bool acc, DType d) {
    evk_b200::matmul(be(), a, b, c, ta, tb, acc, dt(d));
}
void add_ex(Tensor& a, Tensor& b, Tensor& c, DType d) { evk_b200::add(be(), a, b, c, dt(d)); }
void gelu_ex(Tensor& in, Tensor& out, DType d) { evk_b200::gelu(be(), in, out, dt(d)); }
void softmax_ex(Tensor& in, Tensor& out, float s, DType d) { evk_b200::softmax(be(), in, out, s, dt(d)); }

void flash_attention_ex(Tensor& q, Tensor& k, Tensor& v, Tensor& o, uint32_t heads, bool causal, float scale,
                        DType d) {
    if (q.shape.rank() != 3 || k.shape.rank() != 3 || heads == 0 || q.shape[2] % heads != 0)
        return be().fail(EVKCU_BAD_SHAPE, "flash_attention_ex: shapes");
    const uint32_t B = q.shape[0], N = q.shape[1], Dh = q.shape[2] / heads;
    if (k.shape[2] % Dh != 0 || k.shape[0] != B || k.shape[1] != N || !evk_b200::same_shape(k, v) ||
        !evk_b200::same_shape(q, o))
        return be().fail(EVKCU_BAD_SHAPE, "flash_attention_ex: incompatible shapes");
    evk_b200::check(be(),
                    be().flash_attention(evk_b200::dptr(q), evk_b200::dptr(k), evk_b200::dptr(v), evk_b200::dmut(o), B,
                                         N, heads, k.shape[2] / Dh, Dh, scale, causal ? EVKCU_ATTN_CAUSAL : 0u, dt(d),
                                         be().stream()),
                    "flash_attention_ex");
}

void single_query_attention(Tensor& q, Tensor& kc, Tensor& vc, Tensor& out, uint32_t heads, uint32_t cur_len,
                            float scale, DType d) {
    if (q.shape.rank() < 2 || kc.shape.rank() != 3 || heads == 0 || q.shape[-1] % heads != 0)
        return be().fail(EVKCU_BAD_SHAPE, "single_query_attention: shapes");
    const uint32_t B = kc.shape[0], max_len = kc.shape[1], Dh = q.shape[-1] / heads;
    if (kc.shape[2] % Dh != 0 || !evk_b200::same_shape(kc, vc) || q.shape.count() != B * heads * Dh ||
        out.shape.count() != q.shape.count() || cur_len > max_len)
        return be().fail(EVKCU_BAD_SHAPE, "single_query_attention: incompatible shapes");
    evk_b200::check(be(),
                    be().single_query_attention(evk_b200::dptr(q), evk_b200::dptr(kc), evk_b200::dptr(vc),
                                                evk_b200::dmut(out), B, heads, kc.shape[2] / Dh, Dh, max_len, cur_len,
                                                scale, dt(d), be().stream()),
                    "single_query_attention");
}

void rope_ex(Tensor& in, Tensor& out, uint32_t B, uint32_t S, uint32_t D, float base, uint32_t head_dim,
             uint32_t pos_offset, DType d) {
    evk_b200::rope(be(), in, out, B, S, D, base, head_dim, pos_offset, dt(d));
}

void rms_norm_ex(Tensor& in, Tensor& out, float eps, Tensor* gamma, DType d) {
    if (gamma && gamma->shape.count() != in.shape[-1]) return be().fail(EVKCU_BAD_SHAPE, "rms_norm_ex: gamma size");
    evk_b200::rms_norm(be(), in, out, eps, gamma ? evk_b200::dptr(*gamma) : nullptr, dt(d));
}

void embed_ex(Tensor& E, Tensor& idx, Tensor& out, uint32_t id_bytes, DType d) {
    if (id_bytes != 2 && id_bytes != 4) return be().fail(EVKCU_BAD_ARG, "embed_ex: id_bytes");
    evk_b200::embed(be(), E, idx, out, id_bytes, dt(d));
}

void greedy_sample_ex(Tensor& logits, Tensor& out, uint32_t position, uint32_t base, uint32_t count, uint32_t id_bytes,
                      DType d) {
    if (id_bytes != 2 && id_bytes != 4) return be().fail(EVKCU_BAD_ARG, "greedy_sample_ex: id_bytes");
    evk_b200::greedy_sample(be(), logits, out, position, base, count, id_bytes, dt(d));
}

}  // namespace evk::ai
