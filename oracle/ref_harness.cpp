// ref_harness.cpp — TEST INFRASTRUCTURE: runs the reference's own
// known-answer tests (carloshgsilva/evk example/tests.h, compiled from the
// reference checkout, not copied) against the CPU oracle.
//
// It supplies (1) the evk core functions that evk_ai.h / tests.h use, on host
// memory (commands execute at record time; submit/wait are no-ops), and (2)
// the evk::ai operators through the same shape logic as the product
// (evk_b200/cpp/evk_ai_dispatch.h) with the oracle as the backend.  The
// reference's training-side operators are outside this backend's scope; the
// backward passes that the forward tests also exercise (gelu, rope, rms_norm,
// embed) get small host implementations here so those tests run to the end,
// and the remaining ones abort if a selected test ever reaches them.
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
const evk_b200::Backend kOracle = {no_stream, die,     o_matmul, o_flash, o_sqa,  o_rms,   o_rope,  o_gelu,
                                   o_softmax, o_add,   o_scale,  o_zero,  o_mask, o_embed, o_greedy};

[[noreturn]] void out_of_scope(const char* op) {
    std::fprintf(stderr, "oracle harness: %s is a training-side operator outside this backend\n", op);
    std::exit(3);
}
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

// --- backward passes used by the forward tests (host math, test-only) ---
void gelu_backward(Tensor& grad_out, Tensor& in, Tensor& grad_in) {
    auto* go = (float16_t*)grad_out.buffer.GetPtr();
    auto* x = (float16_t*)in.buffer.GetPtr();
    auto* gi = (float16_t*)grad_in.buffer.GetPtr();
    for (uint32_t i = 0; i < in.shape.count(); ++i) gi[i] = float16_t(float(gi[i]) + float(go[i]) * gelu_grad_approx_cpu(float(x[i])));
}
void rope_backward(Tensor& grad_out, Tensor& grad_in, uint32_t B, uint32_t S, uint32_t D, float base) {
    auto* go = (float16_t*)grad_out.buffer.GetPtr();
    auto* gi = (float16_t*)grad_in.buffer.GetPtr();
    for (uint32_t r = 0; r < B * S; ++r)
        for (uint32_t p = 0; p < D / 2; ++p) {
            float ang = float(r % S) * std::pow(base, -2.0f * float(p) / float(D));
            float c = std::cos(ang), s = std::sin(ang);
            float g0 = go[r * D + 2 * p], g1 = go[r * D + 2 * p + 1];
            gi[r * D + 2 * p] = float16_t(float(gi[r * D + 2 * p]) + g0 * c + g1 * s);
            gi[r * D + 2 * p + 1] = float16_t(float(gi[r * D + 2 * p + 1]) - g0 * s + g1 * c);
        }
}
void rms_norm_backward(Tensor& in, Tensor& grad_out, Tensor& grad_in, float eps) {
    auto* x = (float16_t*)in.buffer.GetPtr();
    auto* go = (float16_t*)grad_out.buffer.GetPtr();
    auto* gi = (float16_t*)grad_in.buffer.GetPtr();
    const uint32_t D = in.shape[-1], rows = in.shape.count() / D;
    for (uint32_t r = 0; r < rows; ++r) {
        float ss = 0.0f;
        for (uint32_t d = 0; d < D; ++d) ss += float(x[r * D + d]) * float(x[r * D + d]);
        const float inv = 1.0f / std::sqrt(ss / float(D) + eps);
        float dot = 0.0f;
        for (uint32_t d = 0; d < D; ++d) dot += float(go[r * D + d]) * float(x[r * D + d]) * inv;
        for (uint32_t d = 0; d < D; ++d) {
            const float y = float(x[r * D + d]) * inv;
            gi[r * D + d] = float16_t(float(gi[r * D + d]) + (float(go[r * D + d]) - y * dot / float(D)) * inv);
        }
    }
}
void embed_backward(Tensor& grad_out, Tensor& idx, Tensor& grad_E) {
    auto* go = (float16_t*)grad_out.buffer.GetPtr();
    auto* ids = (uint16_t*)idx.buffer.GetPtr();
    auto* ge = (float16_t*)grad_E.buffer.GetPtr();
    const uint32_t D = grad_E.shape[1];
    for (uint32_t i = 0; i < idx.shape.count(); ++i)
        for (uint32_t d = 0; d < D; ++d) ge[ids[i] * D + d] = float16_t(float(ge[ids[i] * D + d]) + float(go[i * D + d]));
}

// --- training-side operators: outside this backend ---
void AdamState::init(uint32_t) { out_of_scope("AdamState::init"); }
void AdamState::reset() {}
void flash_attention_bwd(Tensor&, Tensor&, Tensor&, Tensor&, Tensor&, Tensor&, Tensor&, Tensor&, uint32_t) { out_of_scope("flash_attention_bwd"); }
void mse_loss(Tensor&, Tensor&, Tensor&, Tensor&) { out_of_scope("mse_loss"); }
void sgd(Tensor&, Tensor&, float) { out_of_scope("sgd"); }
void adam(Tensor&, Tensor&, AdamState&, float, float, float, float) { out_of_scope("adam"); }
void softmax_backward(Tensor&, Tensor&, Tensor&, float) { out_of_scope("softmax_backward"); }
void relu(Tensor&, Tensor&) { out_of_scope("relu"); }
void relu_backward(Tensor&, Tensor&, Tensor&) { out_of_scope("relu_backward"); }
void cross_entropy_loss(Tensor&, Tensor&, Tensor&, Tensor&) { out_of_scope("cross_entropy_loss"); }
void position_add(Tensor&, Tensor&, Tensor&, uint32_t, uint32_t, uint32_t) { out_of_scope("position_add"); }
void position_add_backward(Tensor&, Tensor&, Tensor&, uint32_t, uint32_t, uint32_t) { out_of_scope("position_add_backward"); }
void sum_batch(Tensor&, Tensor&, uint32_t, uint32_t) { out_of_scope("sum_batch"); }
}  // namespace evk::ai

int main(int argc, char** argv) {
    // The inference-path known-answer tests of example/tests.h.  The
    // 32768-token flash-vs-unfused comparison runs only with --flash (it
    // materialises two 2 GB score matrices on the host).
    bool flash = argc > 1 && std::strcmp(argv[1], "--flash") == 0;
    test_add();
    test_matmul();
    test_matmul_broadcast();
    test_softmax();
    test_gelu();
    test_scale_zero();
    test_embed_and_backward();
    test_rope_and_backward();
    test_rms_norm_and_backward();
    test_greedy_sample();
    if (flash) test_flash_attention_cmp_softmax();
    std::printf("ALL REFERENCE KATS PASSED (oracle backend)\n");
    return 0;
}
