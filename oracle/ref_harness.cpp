// ref_harness.cpp — TEST INFRASTRUCTURE: runs the reference's own
// known-answer tests (carloshgsilva/evk example/tests.h, compiled from the
// reference checkout, not copied) against the CPU oracle.
//
// It supplies (1) the evk core functions that evk_ai.h / tests.h use, on host
// memory (commands execute at record time; submit/wait are no-ops), and (2)
// the evk::ai operators, inference and training side, through the same shape
// logic as the product (evk_b200/cpp/evk_ai_dispatch.h) with the oracle as
// the backend, so the reference's known-answer tests pin every oracle
// restatement the GPU parity tests compare against.
#include <chrono>
#include <cstring>
#include <type_traits>

#include "evk_ai.h"  // the reference's header (resolved through -I<reference>)
#include "evk_oracle.h"
#include "tests.h"   // the reference's tests (resolved through -I<reference>/example)
#include "../evk_b200/cpp/evk_ai_dispatch.h"  // needs -I../include for evkcu.h

// ------------------------------------------------------------ host evk core --
namespace evk {
namespace {
struct HostBuffer : Resource {
    BufferDesc desc;
    std::vector<uint8_t> mem;
};
HostBuffer* hb(const Buffer& b) { return static_cast<HostBuffer*>(b.res); }
std::vector<TimestampEntry> g_stamps, g_open;
double now_ms() {
    using namespace std::chrono;
    return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}
Cmd g_cmd;
Features g_features;
}  // namespace

void Resource::decRef() {
    if (refCount > 0 && --refCount == 0) delete this;
}
RID ResourceRef::GetRID() const { return res ? res->resourceid : -1; }
Buffer CreateBuffer(const BufferDesc& desc) {
    auto* r = new HostBuffer();
    r->desc = desc;
    r->mem.assign(desc.size ? desc.size : 16, 0);
    return Buffer(r);
}
void* Buffer::GetPtr() { return hb(*this)->mem.data(); }
uint64_t Buffer::GetReference() { return reinterpret_cast<uint64_t>(hb(*this)->mem.data()); }
const BufferDesc& GetDesc(const Buffer& b) { return hb(b)->desc; }
void Cmd::copy(Buffer& src, Buffer& dst, uint64_t size, uint64_t so, uint64_t dO) {
    std::memcpy(hb(dst)->mem.data() + dO, hb(src)->mem.data() + so, size);
}
void Cmd::copy(void* src, Buffer& dst, uint64_t size, uint64_t off) { std::memcpy(hb(dst)->mem.data() + off, src, size); }
void Cmd::barrier() {}
int Cmd::beginTimestamp(const char* name) {
    g_open.push_back(TimestampEntry{now_ms(), 0.0, name});
    return (int)g_open.size() - 1;
}
void Cmd::endTimestamp(int id) { g_open.at(id).end = now_ms(); }
uint64_t Cmd::submit() {
    g_stamps = g_open;
    g_open.clear();
    return 1;
}
Cmd& CmdBegin(Queue) { return g_cmd; }
void CmdWait(uint64_t) {}
bool CmdDone(uint64_t) { return true; }
const std::vector<TimestampEntry>& CmdTimestamps() { return g_stamps; }
const Features& GetFeatures() { return g_features; }
}  // namespace evk

// ------------------------------------------------------- oracle as backend --
namespace {
using u16 = uint16_t;
void* no_stream() { return nullptr; }
void die(int st, const char* op) {
    std::fprintf(stderr, "oracle harness: %s rejected its arguments (status %d)\n", op, st);
    std::exit(2);
}
int o_matmul(const void* A, const void* B, void* C, uint32_t batch, uint32_t M, uint32_t K, uint32_t N, uint64_t sa,
             uint64_t sb, uint64_t sc, uint32_t flags, int dt, void*) {
    oracle_matmul((const u16*)A, (const u16*)B, (u16*)C, batch, M, K, N, sa, sb, sc, flags, dt);
    return 0;
}
int o_flash(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t N, uint32_t H, uint32_t Hkv,
            uint32_t Dh, float scale, uint32_t flags, int dt, void*) {
    oracle_flash_attention((const u16*)q, (const u16*)k, (const u16*)v, (u16*)o, B, N, H, Hkv, Dh, scale, flags, dt);
    return 0;
}
int o_sqa(const void* q, const void* k, const void* v, void* o, uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh,
          uint32_t ml, uint32_t cl, float sc, int dt, void*) {
    oracle_single_query_attention((const u16*)q, (const u16*)k, (const u16*)v, (u16*)o, B, H, Hkv, Dh, ml, cl, sc, dt);
    return 0;
}
int o_rms(const void* in, void* out, const void* g, uint32_t rows, uint32_t D, float eps, int dt, void*) {
    oracle_rms_norm((const u16*)in, (u16*)out, (const u16*)g, rows, D, eps, dt);
    return 0;
}
int o_rope(const void* in, void* out, uint32_t b, uint32_t s, uint32_t d, uint32_t hd, uint32_t off, float base, int dt,
           void*) {
    oracle_rope((const u16*)in, (u16*)out, b, s, d, hd, off, base, dt);
    return 0;
}
int o_gelu(const void* in, void* out, uint64_t n, int dt, void*) {
    oracle_gelu((const u16*)in, (u16*)out, n, dt);
    return 0;
}
int o_softmax(const void* in, void* out, uint32_t rows, uint32_t L, float s, int dt, void*) {
    oracle_softmax((const u16*)in, (u16*)out, rows, L, s, dt);
    return 0;
}
int o_add(const void* a, const void* b, void* c, uint64_t n, int dt, void*) {
    oracle_add((const u16*)a, (const u16*)b, (u16*)c, n, dt);
    return 0;
}
int o_scale(void* x, uint64_t n, float s, int dt, void*) {
    oracle_scale((u16*)x, n, s, dt);
    return 0;
}
int o_zero(void* x, uint64_t n, int, void*) {
    std::memset(x, 0, n * 2);
    return 0;
}
int o_mask(void* s, uint32_t b, uint32_t n, int dt, void*) {
    oracle_causal_mask((u16*)s, b, n, dt);
    return 0;
}
int o_embed(const void* E, const void* idx, void* out, uint32_t V, uint32_t D, uint32_t n, uint32_t ib, int, void*) {
    oracle_embed((const u16*)E, idx, (u16*)out, V, D, n, ib);
    return 0;
}
int o_greedy(const void* l, void* out, uint32_t B, uint32_t S, uint32_t V, uint32_t pos, uint32_t base, uint32_t cnt,
             uint32_t ob, int dt, void*) {
    oracle_greedy_sample((const u16*)l, out, B, S, V, pos, base, cnt, ob, dt);
    return 0;
}
// training side
int o_relu(const void* in, void* out, uint64_t n, int dt, void*) {
    oracle_relu((const u16*)in, (u16*)out, n, dt);
    return 0;
}
int o_relu_bwd(const void* go, const void* in, void* gi, uint64_t n, int dt, void*) {
    oracle_relu_backward((const u16*)go, (const u16*)in, (u16*)gi, n, dt);
    return 0;
}
int o_gelu_bwd(const void* go, const void* in, void* gi, uint64_t n, int dt, void*) {
    oracle_gelu_backward((const u16*)go, (const u16*)in, (u16*)gi, n, dt);
    return 0;
}
int o_softmax_bwd(const void* p, const void* g, void* gi, uint32_t rows, uint32_t L, float s, int dt, void*) {
    oracle_softmax_backward((const u16*)p, (const u16*)g, (u16*)gi, rows, L, s, dt);
    return 0;
}
int o_rms_bwd(const void* x, const void* g, void* gi, uint32_t rows, uint32_t D, float eps, int dt, void*) {
    oracle_rms_norm_backward((const u16*)x, (const u16*)g, (u16*)gi, rows, D, eps, dt);
    return 0;
}
int o_rope_bwd(const void* go, void* gi, uint32_t b, uint32_t s, uint32_t d, float base, int dt, void*) {
    oracle_rope_backward((const u16*)go, (u16*)gi, b, s, d, base, dt);
    return 0;
}
int o_embed_bwd(const void* go, const void* idx, void* gE, uint32_t V, uint32_t D, uint32_t n, uint32_t ib, int dt,
                void*) {
    oracle_embed_backward((const u16*)go, idx, (u16*)gE, V, D, n, ib, dt);
    return 0;
}
int o_pos_add(const void* in, const void* pos, void* out, uint32_t b, uint32_t s, uint32_t d, int dt, void*) {
    oracle_position_add((const u16*)in, (const u16*)pos, (u16*)out, b, s, d, dt);
    return 0;
}
int o_pos_add_bwd(const void* go, void* gi, void* gp, uint32_t b, uint32_t s, uint32_t d, int dt, void*) {
    oracle_position_add_backward((const u16*)go, (u16*)gi, (u16*)gp, b, s, d, dt);
    return 0;
}
int o_sum_batch(const void* in, void* out, uint32_t batch, uint64_t size, int dt, void*) {
    oracle_sum_batch((const u16*)in, (u16*)out, batch, size, dt);
    return 0;
}
int o_sgd(void* p, const void* g, uint64_t n, float lr, int dt, void*) {
    oracle_sgd((u16*)p, (const u16*)g, n, lr, dt);
    return 0;
}
int o_adam(void* p, const void* g, void* m, void* v, uint64_t n, uint32_t step, float lr, float b1, float b2, float eps,
           int dt, void*) {
    oracle_adam((u16*)p, (const u16*)g, (u16*)m, (u16*)v, n, step, lr, b1, b2, eps, dt);
    return 0;
}
int o_mse(const void* p, const void* t, void* g, void* r, uint64_t n, int dt, void*) {
    oracle_mse_loss((const u16*)p, (const u16*)t, (u16*)g, (u16*)r, n, dt);
    return 0;
}
int o_ce(const void* l, const void* t, void* g, void* r, uint32_t rows, uint32_t V, uint32_t tb, int dt, void*) {
    oracle_cross_entropy_loss((const u16*)l, t, (u16*)g, (u16*)r, rows, V, tb, dt);
    return 0;
}
int o_flash_bwd(const void* q, const void* k, const void* v, const void*, const void* dO, void* dQ, void* dK, void* dV,
                uint32_t B, uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dt,
                void*) {
    oracle_flash_attention_bwd((const u16*)q, (const u16*)k, (const u16*)v, (const u16*)dO, (u16*)dQ, (u16*)dK,
                               (u16*)dV, B, N, H, Hkv, Dh, scale, flags, dt);
    return 0;
}
const evk_b200::Backend kOracle = {
    no_stream, die,          o_matmul,   o_flash,   o_sqa,       o_rms,         o_rope,       o_gelu,
    o_softmax, o_add,        o_scale,    o_zero,    o_mask,      o_embed,       o_greedy,     o_relu,
    o_relu_bwd, o_gelu_bwd,  o_softmax_bwd, o_rms_bwd, o_rope_bwd, o_embed_bwd,  o_pos_add,    o_pos_add_bwd,
    o_sum_batch, o_sgd,      o_adam,     o_mse,     o_ce,        o_flash_bwd};
}  // namespace

namespace evk::ai {
evk::Cmd& GetCmd() { return evk::CmdBegin(evk::Queue::Graphics); }
uint64_t SubmitCmd(bool wait) {
    uint64_t i = GetCmd().submit();
    if (wait) evk::CmdWait(i);
    return i;
}
void initialize() {}
void shutdown() {}
void matmul(Tensor& a, Tensor& b, Tensor& c, bool ta, bool tb, bool acc, uint8_t, uint8_t) {
    evk_b200::matmul(kOracle, a, b, c, ta, tb, acc);
}
void flash_attention(Tensor& q, Tensor& k, Tensor& v, Tensor& o) { evk_b200::flash_attention(kOracle, q, k, v, o); }
void add(Tensor& a, Tensor& b, Tensor& c) { evk_b200::add(kOracle, a, b, c); }
void softmax(Tensor& in, Tensor& out, float s) { evk_b200::softmax(kOracle, in, out, s); }
void gelu(Tensor& in, Tensor& out) { evk_b200::gelu(kOracle, in, out); }
void embed(Tensor& E, Tensor& idx, Tensor& out) { evk_b200::embed(kOracle, E, idx, out); }
void greedy_sample(Tensor& l, Tensor& out, uint32_t pos, uint16_t base, uint16_t cnt) {
    evk_b200::greedy_sample(kOracle, l, out, pos, base, cnt);
}
void apply_causal_mask(Tensor& s) { evk_b200::apply_causal_mask(kOracle, s); }
void rope(Tensor& in, Tensor& out, uint32_t B, uint32_t S, uint32_t D, float base) {
    evk_b200::rope(kOracle, in, out, B, S, D, base);
}
void scale(Tensor& t, float s) { evk_b200::scale(kOracle, t, s); }
void zero(Tensor& t) { evk_b200::zero(kOracle, t); }
void rms_norm(Tensor& in, Tensor& out, float eps) { evk_b200::rms_norm(kOracle, in, out, eps); }

// --- training side ---
void AdamState::init(uint32_t n) {
    m_buffer = evk::CreateBuffer({.size = (uint64_t)n * sizeof(float16_t)});
    v_buffer = evk::CreateBuffer({.size = (uint64_t)n * sizeof(float16_t)});  // host memory, zero-filled
    t = 0;
}
void AdamState::reset() {
    m_buffer = {};
    v_buffer = {};
    t = 0;
}
void flash_attention_bwd(Tensor& q, Tensor& k, Tensor& v, Tensor& o, Tensor& dO, Tensor& dQ, Tensor& dK, Tensor& dV,
                         uint32_t heads) {
    evk_b200::flash_attention_bwd(kOracle, q, k, v, o, dO, dQ, dK, dV, heads);
}
void mse_loss(Tensor& p, Tensor& t, Tensor& g, Tensor& r) { evk_b200::mse_loss(kOracle, p, t, g, r); }
void sgd(Tensor& p, Tensor& g, float lr) { evk_b200::sgd(kOracle, p, g, lr); }
void adam(Tensor& p, Tensor& g, AdamState& st, float lr, float b1, float b2, float eps) {
    if (!st.m_buffer) st.init(p.shape.count());
    st.t += 1;
    evk_b200::adam(kOracle, p, g, st.m_buffer.GetPtr(), st.v_buffer.GetPtr(), st.t, lr, b1, b2, eps);
}
void softmax_backward(Tensor& p, Tensor& go, Tensor& gi, float s) { evk_b200::softmax_backward(kOracle, p, go, gi, s); }
void relu(Tensor& in, Tensor& out) { evk_b200::relu(kOracle, in, out); }
void relu_backward(Tensor& go, Tensor& in, Tensor& gi) { evk_b200::relu_backward(kOracle, go, in, gi); }
void gelu_backward(Tensor& go, Tensor& in, Tensor& gi) { evk_b200::gelu_backward(kOracle, go, in, gi); }
void cross_entropy_loss(Tensor& l, Tensor& t, Tensor& g, Tensor& r) { evk_b200::cross_entropy_loss(kOracle, l, t, g, r); }
void embed_backward(Tensor& go, Tensor& idx, Tensor& gE) { evk_b200::embed_backward(kOracle, go, idx, gE); }
void position_add(Tensor& in, Tensor& pos, Tensor& out, uint32_t B, uint32_t S, uint32_t D) {
    evk_b200::position_add(kOracle, in, pos, out, B, S, D);
}
void position_add_backward(Tensor& go, Tensor& gi, Tensor& gp, uint32_t B, uint32_t S, uint32_t D) {
    evk_b200::position_add_backward(kOracle, go, gi, gp, B, S, D);
}
void rope_backward(Tensor& go, Tensor& gi, uint32_t B, uint32_t S, uint32_t D, float base) {
    evk_b200::rope_backward(kOracle, go, gi, B, S, D, base);
}
void sum_batch(Tensor& in, Tensor& out, uint32_t b, uint32_t size) { evk_b200::sum_batch(kOracle, in, out, b, size); }
void rms_norm_backward(Tensor& in, Tensor& go, Tensor& gi, float eps) {
    evk_b200::rms_norm_backward(kOracle, in, go, gi, eps);
}
}  // namespace evk::ai

int main(int argc, char** argv) {
    // Every test of example/tests.h: the reference's default list
    // (run_ai_kernel_tests, tests.h:1565-1585) and the ones it leaves out,
    // except test_adam_batched_matmul: it steps Adam with lr = -0.02
    // (tests.h:1009) on the mse_loss gradient 2 (pred - target) / n, which
    // climbs the loss under the reference's own update rule
    // (shaders/adam.comp: param -= lr * update), so it cannot pass on any
    // faithful backend.  The 32768-token flash-vs-unfused comparison runs only
    // with --flash (it materialises two 2 GB score matrices on the host).
    bool flash = argc > 1 && std::strcmp(argv[1], "--flash") == 0;
    run_ai_kernel_tests();
    test_flash_attention_backward();
    test_graph_backward();
    test_attn_graph();
    test_adam_convergence();
    test_adam_vs_sgd();
    if (flash) test_flash_attention_cmp_softmax();
    std::printf("ALL REFERENCE KATS PASSED (oracle backend)\n");
    return 0;
}
