// evk_ai.h — the evk::ai inference operator API (carloshgsilva/evk
// evk_ai.h:13-16, 18-472, 474-615, 617-1073) on the B200 backend.
//
// Same names, signatures, argument meaning and tensor layout as the
// reference for the inference path: every Tensor is 2-byte storage of
// shape.count() elements, row-major with the last dimension contiguous; token
// ids are raw unsigned 16-bit integers stored in the element slots.  Ops are
// enqueued on the stream of GetCmd() and run in order; SubmitCmd(wait)
// records a submission and optionally waits for it.  The training-side
// operators of the reference (losses, optimisers, backward passes) are not
// part of this backend.  Additive extensions live in evk_ai_ext.h.
#pragma once

#include <cassert>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <vector>

#include "evk.h"

namespace evk::ai {
evk::Cmd& GetCmd();
uint64_t SubmitCmd(bool wait = true);
}  // namespace evk::ai

// IEEE binary16 value with the reference's host conversions
// (float16_t, evk_ai.h:18-158): fp32 -> fp16 rounds normals to nearest-even
// and subnormals half-up; fp16 -> fp32 is exact.
struct float16_t {
    uint16_t value;

    float16_t() = default;
    float16_t(float f) { value = float_to_float16(f); }
    float16_t(const float16_t&) = default;
    float16_t& operator=(const float16_t&) = default;
    operator float() const { return float16_to_float(value); }
    float16_t& operator+=(const float16_t& o) {
        *this = float16_t(float(*this) + float(o));
        return *this;
    }
    float16_t& operator/=(const float16_t& o) {
        *this = float16_t(float(*this) / float(o));
        return *this;
    }

    static uint16_t float_to_float16(float f) {
        uint32_t x;
        std::memcpy(&x, &f, 4);
        const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
        const uint32_t bexp = (x >> 23) & 0xFFu;
        uint32_t frac = x & 0x7FFFFFu;
        if (bexp == 0xFFu) {
            if (frac == 0) return sign | 0x7C00u;
            uint16_t pl = (uint16_t)((frac >> 13) & 0x3FFu);
            return sign | 0x7C00u | (pl ? pl : 1u);
        }
        const int e = (int)bexp - 127;
        if (e > 15) return sign | 0x7C00u;
        if (e >= -14) {
            uint32_t he = (uint32_t)(e + 15), m = frac >> 13;
            const uint32_t rest = frac & 0x1FFFu;
            if (rest > 0x1000u || (rest == 0x1000u && (m & 1u))) {
                if (++m == 0x400u) {
                    m = 0;
                    if (++he == 0x1Fu) return sign | 0x7C00u;
                }
            }
            return sign | (uint16_t)(he << 10) | (uint16_t)m;
        }
        if (e < -24) return sign;
        frac |= 0x800000u;
        const int sh = -14 - e;
        uint32_t m = frac >> (13 + sh);
        if ((frac >> (12 + sh)) & 1u) ++m;
        return sign | (uint16_t)(m & 0x3FFu);
    }

    static float float16_to_float(uint16_t h) {
        const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
        const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
        float out;
        if (e == 0) {
            out = std::ldexp((float)m, -24);
            return sign ? -out : out;
        }
        uint32_t bits = e == 0x1Fu ? (sign | 0x7F800000u | (m << 13)) : (sign | ((e + 112u) << 23) | (m << 13));
        std::memcpy(&out, &bits, 4);
        return out;
    }
};

// Tensor shape, up to 8 dimensions (evk_ai.h:160-219).
struct Shape {
    static constexpr uint32_t MAX_DIMENSIONS = 8;
    uint32_t values[MAX_DIMENSIONS] = {};
    uint32_t size = 0;

    Shape() {}
    Shape(std::initializer_list<uint32_t> v) {
        assert(v.size() <= MAX_DIMENSIONS);
        size = (uint32_t)v.size();
        uint32_t i = 0;
        for (uint32_t x : v) values[i++] = x;
    }
    // Negative indices count from the end.
    uint32_t operator[](int index) const {
        if (index < 0) index += (int)size;
        assert(index >= 0 && index < (int)size);
        return values[index];
    }
    uint32_t rank() const { return size; }
    uint32_t number_of_elements(uint32_t index = 0) const {
        uint32_t c = 1;
        for (uint32_t i = index; i < size; ++i) c *= values[i];
        return c;
    }
    uint32_t count() const { return number_of_elements(0); }
    // Product of all dimensions except the last `element_count`.
    uint32_t batch_size(uint32_t element_count) const {
        assert(element_count <= size);
        uint32_t b = 1;
        for (uint32_t i = 0; i + element_count < size; ++i) b *= values[i];
        return b;
    }
};

// Device tensor with a lazily created host mirror (evk_ai.h:242-472).
struct Tensor {
    evk::Buffer buffer;
    evk::Buffer cpu_buffer;
    std::unique_ptr<Tensor> grad_tensor;
    Shape shape = {};

    std::function<void()> forward_fn;
    std::function<void()> backward_fn;

    Tensor() = default;
    Tensor(const Shape& s) : shape(s) {
        buffer = evk::CreateBuffer({.size = (uint64_t)s.count() * sizeof(float16_t), .usage = evk::BufferUsage::Storage});
    }
    static Tensor alias(const Shape& s, const evk::Buffer& existing) {
        Tensor t;
        t.shape = s;
        t.buffer = existing;
        return t;
    }
    Tensor& grad() {
        if (!grad_tensor) grad_tensor = std::make_unique<Tensor>(shape);
        return *grad_tensor;
    }
    float16_t* cpu() {
        if (!cpu_buffer)
            cpu_buffer = evk::CreateBuffer({.size = (uint64_t)shape.count() * sizeof(float16_t),
                                            .usage = evk::BufferUsage::TransferDst | evk::BufferUsage::TransferSrc,
                                            .memoryType = evk::MemoryType::CPU});
        return (float16_t*)cpu_buffer.GetPtr();
    }
    void cpu_upload(bool submit = true) {
        cpu();
        evk::ai::GetCmd().copy(cpu_buffer, buffer, (uint64_t)shape.count() * sizeof(float16_t));
        if (submit) evk::ai::SubmitCmd(true);
    }
    void cpu_download(bool submit = true) {
        cpu();
        evk::ai::GetCmd().copy(buffer, cpu_buffer, (uint64_t)shape.count() * sizeof(float16_t));
        if (submit) evk::ai::SubmitCmd(true);
    }
    // Diagonal of `val` in a [rows, cols] view (evk_ai.h:296-303).
    Tensor& identity(float16_t val = float16_t(1.0f)) {
        float16_t* d = cpu();
        for (uint32_t i = 0; i < shape.count(); ++i) d[i] = (i % (shape[0] + 1) == 0) ? val : float16_t(0.0f);
        cpu_upload();
        return *this;
    }
    Tensor& random(float16_t = float16_t(0.0f)) {
        float16_t* d = cpu();
        for (uint32_t i = 0; i < shape.count(); ++i) d[i] = float16_t(float(rand()) / float(RAND_MAX));
        cpu_upload();
        return *this;
    }
    Tensor& fill(float16_t val = float16_t(0.0f)) {
        float16_t* d = cpu();
        for (uint32_t i = 0; i < shape.count(); ++i) d[i] = val;
        cpu_upload();
        return *this;
    }
    // Gaussian init via Box-Muller over libc rand() (evk_ai.h:333-344).
    Tensor& random_init(float stddev = 0.1f) {
        float16_t* d = cpu();
        for (uint32_t i = 0; i < shape.count(); ++i) {
            float u1 = float(rand() + 1) / float(RAND_MAX + 1.0f);
            float u2 = float(rand()) / float(RAND_MAX);
            d[i] = float16_t(sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2) * stddev);
        }
        cpu_upload();
        return *this;
    }
    float16_t item() {
        assert(shape.count() == 1);
        cpu_download();
        return cpu()[0];
    }
    void print(uint32_t max_elements = 8) {
        cpu_download();
        const float16_t* d = cpu();
        std::printf("Tensor (");
        for (uint32_t i = 0; i < shape.rank(); ++i) std::printf(i ? ", %u" : "%u", shape[i]);
        std::printf("): [");
        const uint32_t n = shape.count() < max_elements ? shape.count() : max_elements;
        for (uint32_t i = 0; i < n; ++i) std::printf(i ? ", %g" : "%g", float(d[i]));
        std::printf(n < shape.count() ? ", ...]\n" : "]\n");
    }
};

// fp16 operator set (evk_ai.h:489-615, inference subset).
namespace evk::ai {
void initialize();
void shutdown();

// C = A * B; (...B, M, N) = (...B, M, K) * (...B, K, N).  A batch extent of 1
// broadcasts an operand.  Tile hints are accepted for source compatibility;
// the backend chooses its own tiling and has no divisibility requirement.
void matmul(Tensor& a, Tensor& b, Tensor& c, bool transpose_a = false, bool transpose_b = false, bool acc_c = false,
            uint8_t TILE_M = 80u, uint8_t TILE_N = 80u);

// Multi-query flash attention: Q, O (B, N, H*Dh); K, V (B, N, Dh).
void flash_attention(Tensor& q, Tensor& k, Tensor& v, Tensor& o);

void add(Tensor& a, Tensor& b, Tensor& c);
void softmax(Tensor& in, Tensor& out, float input_scale = 1.0f);
void gelu(Tensor& in, Tensor& out);
void embed(Tensor& embeddings, Tensor& indices, Tensor& out);
void greedy_sample(Tensor& logits, Tensor& out_tokens, uint32_t position, uint16_t token_base, uint16_t token_count);
void apply_causal_mask(Tensor& scores);
void rope(Tensor& input, Tensor& out, uint32_t batch_size, uint32_t seq_len, uint32_t embed_dim,
          float rotary_base = 10000.0f);
void scale(Tensor& tensor, float scale_factor);
void zero(Tensor& tensor);
void rms_norm(Tensor& input, Tensor& output, float eps = 1e-4f);
}  // namespace evk::ai

// Forward-only computation graph (evk_ai.h:617-1073, inference subset): a
// list of nodes whose forward closures call evk::ai ops in insertion order.
struct Graph {
    std::vector<std::unique_ptr<Tensor>> nodes;
    std::vector<Tensor*> params;

    Tensor& tensor(Shape shape, bool param = false) {
        nodes.push_back(std::make_unique<Tensor>(shape));
        if (param) params.push_back(nodes.back().get());
        return *nodes.back();
    }
    Tensor& matmul(Tensor& a, Tensor& b, uint8_t tile_m = 16, uint8_t tile_n = 16) {
        Shape out;
        if (a.shape.rank() == 2 && b.shape.rank() == 2)
            out = Shape({a.shape[0], b.shape[1]});
        else if (a.shape.rank() == 3 && b.shape.rank() == 2)
            out = Shape({a.shape[0], a.shape[1], b.shape[1]});
        else if (a.shape.rank() == 2 && b.shape.rank() == 3)
            out = Shape({b.shape[0], a.shape[0], b.shape[2]});
        else
            out = Shape({a.shape[0], a.shape[1], b.shape[2]});
        Tensor& c = tensor(out);
        c.forward_fn = [&a, &b, &c, tile_m, tile_n]() { evk::ai::matmul(a, b, c, false, false, false, tile_m, tile_n); };
        return c;
    }
    Tensor& add(Tensor& a, Tensor& b) {
        Tensor& c = tensor(a.shape);
        c.forward_fn = [&a, &b, &c]() { evk::ai::add(a, b, c); };
        return c;
    }
    Tensor& residual(Tensor& a, Tensor& b) { return add(a, b); }
    Tensor& gelu(Tensor& in) {
        Tensor& out = tensor(in.shape);
        out.forward_fn = [&in, &out]() { evk::ai::gelu(in, out); };
        return out;
    }
    Tensor& rms_norm(Tensor& in, float eps = 1e-4f) {
        Tensor& out = tensor(in.shape);
        out.forward_fn = [&in, &out, eps]() { evk::ai::rms_norm(in, out, eps); };
        return out;
    }
    Tensor& rope(Tensor& in, float base = 10000.0f) {
        Tensor& out = tensor(in.shape);
        const uint32_t B = in.shape[0], S = in.shape[1], D = in.shape[2];
        out.forward_fn = [&in, &out, B, S, D, base]() { evk::ai::rope(in, out, B, S, D, base); };
        return out;
    }
    Tensor& embed(Tensor& embeddings, Tensor& indices) {
        Tensor& out = tensor(Shape({indices.shape[0], indices.shape[1], embeddings.shape[1]}));
        out.forward_fn = [&embeddings, &indices, &out]() { evk::ai::embed(embeddings, indices, out); };
        return out;
    }
    // Unfused causal attention, one head over the whole model dimension
    // (evk_ai.h:961-1007): scores = q k^T, mask, softmax(scale), probs v.
    Tensor& causal_attention(Tensor& q, Tensor& k, Tensor& v, float scale = 0.0f) {
        const uint32_t B = q.shape[0], N = q.shape[1], D = q.shape[2];
        Tensor& scores = tensor(Shape({B, N, N}));
        Tensor& probs = tensor(Shape({B, N, N}));
        Tensor& out = tensor(Shape({B, N, D}));
        const float s = scale > 0.0f ? scale : 1.0f / std::sqrt(float(D));
        out.forward_fn = [&q, &k, &v, &scores, &probs, &out, s]() {
            evk::ai::matmul(q, k, scores, false, true, false, 16, 16);
            evk::ai::apply_causal_mask(scores);
            evk::ai::softmax(scores, probs, s);
            evk::ai::matmul(probs, v, out, false, false, false, 16, 16);
        };
        return out;
    }
    // Runs every forward closure in insertion order (evk_ai.h:1018-1048);
    // backward passes are not part of this backend.
    void eval(bool backward = false, bool submit = true, bool wait = true) {
        assert(!backward && "backward passes are not part of the inference backend");
        (void)backward;
        evk::ai::GetCmd();
        for (auto& n : nodes)
            if (n->forward_fn) n->forward_fn();
        if (submit) evk::ai::SubmitCmd(wait);
    }
};
