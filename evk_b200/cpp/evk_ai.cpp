// evk_ai.cpp — evk::ai operators on the B200 backend: shape logic from
// evk_ai_dispatch.h, kernels from libevkcu (include/evkcu.h).
// Replaces evk_ai.cpp of the reference (pipeline creation :30-246 and the
// per-op bind/push/dispatch/barrier recording :254-1067).
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
    };
    return be;
}

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

}  // namespace evk::ai
