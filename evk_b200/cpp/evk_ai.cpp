// evk_ai.cpp — evk::ai operators on the B200 backend: shape logic from
// evk_ai_dispatch.h, kernels from libevkcu (include/evkcu.h).
// Replaces evk_ai.cpp of the reference (pipeline creation :30-246, AdamState
// :193-216 and the per-op bind/push/dispatch/barrier recording :254-1094).
#include "evk_ai.h"

#include <cstdio>
#include <cstdlib>

#include "evk_ai_dispatch.h"
#include "evk_cuda.h"
#include "evkcu.h"

namespace evk::ai {

static evk::Cmd* g_cmd = nullptr;

evk::Cmd& GetCmd() {
    if (!g_cmd) g_cmd = &evk::CmdBegin(evk::Queue::Graphics);
    return *g_cmd;
}

uint64_t SubmitCmd(bool wait) {
    evk::Cmd& cmd = GetCmd();
    const uint64_t idx = cmd.submit();
    g_cmd = nullptr;
    if (wait) evk::CmdWait(idx);
    return idx;
}

static void* current_stream() { return evk::cuda_stream(GetCmd()); }

static void fatal(int status, const char* op) {
    std::fprintf(stderr, "evk::ai::%s failed (status %d): %s\n", op, status, evkcu_last_error());
    std::abort();
}

static const evk_b200::Backend& backend() {
    static const evk_b200::Backend be = {
        current_stream,       fatal,          evkcu_matmul,  evkcu_flash_attention, evkcu_single_query_attention,
        evkcu_rms_norm,       evkcu_rope,     evkcu_gelu,    evkcu_softmax,         evkcu_add,
        evkcu_scale,          evkcu_zero,     evkcu_causal_mask, evkcu_embed,       evkcu_greedy_sample,
        evkcu_relu,           evkcu_relu_backward,     evkcu_gelu_backward,  evkcu_softmax_backward,
        evkcu_rms_norm_backward, evkcu_rope_backward,  evkcu_embed_backward, evkcu_position_add,
        evkcu_position_add_backward, evkcu_sum_batch,  evkcu_sgd,            evkcu_adam,
        evkcu_mse_loss,       evkcu_cross_entropy_loss, evkcu_flash_attention_bwd,
    };
    return be;
}

}  // namespace evk::ai

namespace evk_b200 {
// The backend table, shared with the extensions (evk_ai_ext.cpp).
const Backend& cpp_backend() { return evk::ai::backend(); }
}  // namespace evk_b200

namespace evk::ai {

void initialize() {
    if (evkcu_init(-1) != EVKCU_OK) fatal(EVKCU_CUDA_ERROR, "initialize");
}

void shutdown() { evkcu_shutdown(); }

void matmul(Tensor& a, Tensor& b, Tensor& c, bool ta, bool tb, bool acc, uint8_t, uint8_t) {
    evk_b200::matmul(backend(), a, b, c, ta, tb, acc);
}
void flash_attention(Tensor& q, Tensor& k, Tensor& v, Tensor& o) { evk_b200::flash_attention(backend(), q, k, v, o); }
void add(Tensor& a, Tensor& b, Tensor& c) { evk_b200::add(backend(), a, b, c); }
void softmax(Tensor& in, Tensor& out, float s) { evk_b200::softmax(backend(), in, out, s); }
void gelu(Tensor& in, Tensor& out) { evk_b200::gelu(backend(), in, out); }
void embed(Tensor& E, Tensor& idx, Tensor& out) { evk_b200::embed(backend(), E, idx, out); }
void greedy_sample(Tensor& logits, Tensor& out, uint32_t position, uint16_t base, uint16_t count) {
    evk_b200::greedy_sample(backend(), logits, out, position, base, count);
}
void apply_causal_mask(Tensor& s) { evk_b200::apply_causal_mask(backend(), s); }
void rope(Tensor& in, Tensor& out, uint32_t B, uint32_t S, uint32_t D, float base) {
    evk_b200::rope(backend(), in, out, B, S, D, base);
}
void scale(Tensor& t, float s) { evk_b200::scale(backend(), t, s); }
void zero(Tensor& t) { evk_b200::zero(backend(), t); }
void rms_norm(Tensor& in, Tensor& out, float eps) { evk_b200::rms_norm(backend(), in, out, eps); }

// ------------------------------------------------------------ training side --
void AdamState::init(uint32_t num_elements) {
    const uint64_t bytes = (uint64_t)num_elements * sizeof(float16_t);
    m_buffer = evk::CreateBuffer({.size = bytes, .usage = evk::BufferUsage::Storage | evk::BufferUsage::TransferDst});
    v_buffer = evk::CreateBuffer({.size = bytes, .usage = evk::BufferUsage::Storage | evk::BufferUsage::TransferDst});
    GetCmd().fill(m_buffer, 0u, bytes);
    GetCmd().fill(v_buffer, 0u, bytes);
    SubmitCmd(true);
    t = 0;
}
void AdamState::reset() {
    m_buffer = {};
    v_buffer = {};
    t = 0;
}

void flash_attention_bwd(Tensor& q, Tensor& k, Tensor& v, Tensor& o, Tensor& dO, Tensor& dQ, Tensor& dK, Tensor& dV,
                         uint32_t heads) {
    evk_b200::flash_attention_bwd(backend(), q, k, v, o, dO, dQ, dK, dV, heads);
}
void mse_loss(Tensor& pred, Tensor& target, Tensor& grad, Tensor& result) {
    evk_b200::mse_loss(backend(), pred, target, grad, result);
}
void sgd(Tensor& p, Tensor& g, float lr) { evk_b200::sgd(backend(), p, g, lr); }
// evk_ai.cpp:525-566: lazily creates the state, then steps it.
void adam(Tensor& p, Tensor& g, AdamState& state, float lr, float beta1, float beta2, float eps) {
    if (!state.m_buffer) state.init(p.shape.count());
    state.t += 1;
    evk_b200::adam(backend(), p, g, reinterpret_cast<void*>(state.m_buffer.GetReference()),
                   reinterpret_cast<void*>(state.v_buffer.GetReference()), state.t, lr, beta1, beta2, eps);
}
void softmax_backward(Tensor& probs, Tensor& go, Tensor& gi, float s) {
    evk_b200::softmax_backward(backend(), probs, go, gi, s);
}
void relu(Tensor& in, Tensor& out) { evk_b200::relu(backend(), in, out); }
void relu_backward(Tensor& go, Tensor& in, Tensor& gi) { evk_b200::relu_backward(backend(), go, in, gi); }
void gelu_backward(Tensor& go, Tensor& in, Tensor& gi) { evk_b200::gelu_backward(backend(), go, in, gi); }
void cross_entropy_loss(Tensor& logits, Tensor& targets, Tensor& grad, Tensor& result) {
    evk_b200::cross_entropy_loss(backend(), logits, targets, grad, result);
}
void embed_backward(Tensor& go, Tensor& idx, Tensor& gE) { evk_b200::embed_backward(backend(), go, idx, gE); }
void position_add(Tensor& in, Tensor& pos, Tensor& out, uint32_t B, uint32_t S, uint32_t D) {
    evk_b200::position_add(backend(), in, pos, out, B, S, D);
}
void position_add_backward(Tensor& go, Tensor& gi, Tensor& gp, uint32_t B, uint32_t S, uint32_t D) {
    evk_b200::position_add_backward(backend(), go, gi, gp, B, S, D);
}
void rope_backward(Tensor& go, Tensor& gi, uint32_t B, uint32_t S, uint32_t D, float base) {
    evk_b200::rope_backward(backend(), go, gi, B, S, D, base);
}
void sum_batch(Tensor& in, Tensor& out, uint32_t batch, uint32_t size) {
    evk_b200::sum_batch(backend(), in, out, batch, size);
}
void rms_norm_backward(Tensor& in, Tensor& go, Tensor& gi, float eps) {
    evk_b200::rms_norm_backward(backend(), in, go, gi, eps);
}

}  // namespace evk::ai
