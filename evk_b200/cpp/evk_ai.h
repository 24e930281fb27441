// evk_ai.h — the evk::ai operator API (carloshgsilva/evk evk_ai.h:13-16,
// 18-472, 474-615, 617-1073) on the B200 backend.
//
// Same names, signatures, argument meaning and tensor layout as the
// reference: every Tensor is 2-byte storage of shape.count() elements,
// row-major with the last dimension contiguous; token ids are raw unsigned
// 16-bit integers stored in the element slots.  Ops are enqueued on the
// stream of GetCmd() and run in order; SubmitCmd(wait) records a submission
// and optionally waits for it.  Inference operators, the training side
// (backward passes, losses, SGD / Adam) and the autograd Graph are all
// here.  Additive extensions (bf16, 32-bit ids, causal / grouped-query
// attention, decode attention) live in evk_ai_ext.h.
#pragma once

#include <cassert>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <unordered_map>
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

// fp16 operator set (evk_ai.h:474-615).
namespace evk::ai {
// Adam moments of one parameter tensor in 2-byte storage (evk_ai.h:476-487):
// m_buffer holds m / rms(v), v_buffer holds log2(rms(v)) + 41 (0 = empty).
struct AdamState {
    evk::Buffer m_buffer;
    evk::Buffer v_buffer;
    uint32_t t = 0;  // steps taken

    void init(uint32_t num_elements);
    void reset();
};

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

// Training side.  Backward passes accumulate into their gradient tensor;
// losses and flash_attention_bwd overwrite their outputs.
void flash_attention_bwd(Tensor& q, Tensor& k, Tensor& v, Tensor& o, Tensor& dO, Tensor& dQ, Tensor& dK, Tensor& dV,
                         uint32_t heads = 0);
void mse_loss(Tensor& predicted, Tensor& target, Tensor& predGrad, Tensor& result);
void sgd(Tensor& param, Tensor& gradient, float learning_rate);
void adam(Tensor& param, Tensor& gradient, AdamState& state, float learning_rate = 0.001f, float beta1 = 0.9f,
          float beta2 = 0.999f, float epsilon = 1e-4f);
void softmax_backward(Tensor& probs, Tensor& grad_out, Tensor& grad_in, float scale_factor = 1.0f);
void relu(Tensor& in, Tensor& out);
void relu_backward(Tensor& grad_out, Tensor& in, Tensor& grad_in);
void gelu_backward(Tensor& grad_out, Tensor& in, Tensor& grad_in);
// logits (rows, V), targets (rows) uint16 ids, 0 = ignored position.
void cross_entropy_loss(Tensor& logits, Tensor& targets, Tensor& grad, Tensor& result);
void embed_backward(Tensor& grad_out, Tensor& indices, Tensor& grad_embeddings);
void position_add(Tensor& input, Tensor& pos_emb, Tensor& out, uint32_t batch_size, uint32_t seq_len,
                  uint32_t embed_dim);
void position_add_backward(Tensor& grad_out, Tensor& grad_input, Tensor& grad_pos, uint32_t batch_size,
                           uint32_t seq_len, uint32_t embed_dim);
void rope_backward(Tensor& grad_out, Tensor& grad_input, uint32_t batch_size, uint32_t seq_len, uint32_t embed_dim,
                   float rotary_base = 10000.0f);
void sum_batch(Tensor& input, Tensor& output, uint32_t batch_count, uint32_t size_per_batch);
void rms_norm_backward(Tensor& input, Tensor& grad_out, Tensor& grad_input, float eps = 1e-4f);
}  // namespace evk::ai

// Autograd graph (evk_ai.h:617-1073).  Nodes are created in use order; eval
// runs every forward closure in that order and, with backward, zeroes every
// gradient first and then runs the backward closures in reverse order, so a
// node's gradient is complete before its own backward closure reads it.
// Parameters (tensor(shape, true)) are updated by step (SGD) or step_adam.
struct Graph {
    std::vector<std::unique_ptr<Tensor>> nodes;
    std::vector<Tensor*> params;
    std::unordered_map<Tensor*, evk::ai::AdamState> adam_states;
    std::unique_ptr<Tensor> scratch;  // reused temporary (batched matmul weight gradients)

    Tensor& get_scratch(const Shape& shape) {
        if (scratch && scratch->shape.count() >= shape.count())
            scratch->shape = shape;
        else
            scratch = std::make_unique<Tensor>(shape);
        return *scratch;
    }
    Tensor& tensor(Shape shape, bool param = false) {
        nodes.push_back(std::make_unique<Tensor>(shape));
        if (param) params.push_back(nodes.back().get());
        return *nodes.back();
    }
    // Same elements, new shape: forward copies the buffer, backward copies the gradient back.
    Tensor& view(Tensor& a, Shape new_shape) {
        assert(a.shape.count() == new_shape.count() && "view requires same number of elements");
        Tensor& out = tensor(new_shape);
        const uint64_t bytes = (uint64_t)a.shape.count() * sizeof(float16_t);
        out.forward_fn = [&a, &out, bytes]() { evk::ai::GetCmd().copy(a.buffer, out.buffer, bytes); };
        out.backward_fn = [&a, &out, bytes]() { evk::ai::GetCmd().copy(out.grad().buffer, a.grad().buffer, bytes); };
        return out;
    }
    // (M,K)(K,N), (B,M,K)(K,N), (M,K)(B,K,N), (B,M,K)(B,K,N).
    Tensor& matmul(Tensor& a, Tensor& b, uint8_t tile_m = 16, uint8_t tile_n = 16) {
        Shape out;
        const uint32_t ra = a.shape.rank(), rb = b.shape.rank();
        if (ra == 2 && rb == 2)
            out = Shape({a.shape[0], b.shape[1]});
        else if (ra == 3 && rb == 2)
            out = Shape({a.shape[0], a.shape[1], b.shape[1]});
        else if (ra == 2 && rb == 3)
            out = Shape({b.shape[0], a.shape[0], b.shape[2]});
        else {
            assert(ra == 3 && rb == 3 && "Unsupported matmul shapes");
            out = Shape({a.shape[0], a.shape[1], b.shape[2]});
        }
        Tensor& c = tensor(out);
        c.forward_fn = [&a, &b, &c, tile_m, tile_n]() { evk::ai::matmul(a, b, c, false, false, false, tile_m, tile_n); };
        c.backward_fn = [this, &a, &b, &c, tile_m, tile_n]() {
            // dA += dC B^T
            evk::ai::matmul(c.grad(), b, a.grad(), false, true, true, tile_m, tile_n);
            if (a.shape.rank() == 3 && b.shape.rank() == 2) {
                // dB += sum over the batch of A[i]^T dC[i]
                const uint32_t nb = a.shape[0], K = a.shape[2], N = b.shape[1];
                Tensor& per_batch = get_scratch(Shape({nb, K, N}));
                evk::ai::matmul(a, c.grad(), per_batch, true, false, false, tile_m, tile_n);
                evk::ai::sum_batch(per_batch, b.grad(), nb, K * N);
            } else {
                evk::ai::matmul(a, c.grad(), b.grad(), true, false, true, tile_m, tile_n);
            }
        };
        return c;
    }
    Tensor& add(Tensor& a, Tensor& b) {
        Tensor& c = tensor(a.shape);
        c.forward_fn = [&a, &b, &c]() { evk::ai::add(a, b, c); };
        c.backward_fn = [&a, &b, &c]() {
            evk::ai::add(a.grad(), c.grad(), a.grad());
            evk::ai::add(b.grad(), c.grad(), b.grad());
        };
        return c;
    }
    Tensor& residual(Tensor& a, Tensor& b) { return add(a, b); }
    // The loss kernel writes predicted's gradient itself; there is no backward closure.
    Tensor& mse_loss(Tensor& predicted, Tensor& target) {
        assert(predicted.shape.rank() == target.shape.rank() && "mse_loss: predicted and target must have the same rank");
        Tensor& loss = tensor(Shape({1}));
        loss.forward_fn = [&predicted, &target, &loss]() { evk::ai::mse_loss(predicted, target, predicted.grad(), loss); };
        return loss;
    }
    Tensor& relu(Tensor& a) {
        Tensor& out = tensor(a.shape);
        out.forward_fn = [&a, &out]() { evk::ai::relu(a, out); };
        out.backward_fn = [&a, &out]() { evk::ai::relu_backward(out.grad(), a, a.grad()); };
        return out;
    }
    Tensor& gelu(Tensor& a) {
        Tensor& out = tensor(a.shape);
        out.forward_fn = [&a, &out]() { evk::ai::gelu(a, out); };
        out.backward_fn = [&a, &out]() { evk::ai::gelu_backward(out.grad(), a, a.grad()); };
        return out;
    }
    // out = a * factor; backward scales out's gradient in place (no later
    // reader remains in reverse order) and adds it to a's.
    Tensor& scale(Tensor& a, float factor) {
        Tensor& out = tensor(a.shape);
        const uint64_t bytes = (uint64_t)a.shape.count() * sizeof(float16_t);
        out.forward_fn = [&a, &out, factor, bytes]() {
            evk::ai::GetCmd().copy(a.buffer, out.buffer, bytes);
            evk::ai::scale(out, factor);
        };
        out.backward_fn = [&a, &out, factor]() {
            evk::ai::scale(out.grad(), factor);
            evk::ai::add(a.grad(), out.grad(), a.grad());
        };
        return out;
    }
    Tensor& rms_norm(Tensor& input, float eps = 1e-4f) {
        assert(input.shape.rank() >= 2 && "rms_norm expects at least 2D tensor");
        Tensor& out = tensor(input.shape);
        out.forward_fn = [&input, &out, eps]() { evk::ai::rms_norm(input, out, eps); };
        out.backward_fn = [&input, &out, eps]() { evk::ai::rms_norm_backward(input, out.grad(), input.grad(), eps); };
        return out;
    }
    // input (B, N, D) + pos_emb (N, D) broadcast over the batch.
    Tensor& add_position_embedding(Tensor& input, Tensor& pos_emb, uint32_t batch_size, uint32_t seq_len) {
        const uint32_t D = pos_emb.shape[1];
        assert(input.shape.rank() == 3 && input.shape[0] == batch_size && input.shape[1] == seq_len &&
               input.shape[2] == D && pos_emb.shape[0] == seq_len);
        Tensor& out = tensor(input.shape);
        out.forward_fn = [&input, &pos_emb, &out, batch_size, seq_len, D]() {
            evk::ai::position_add(input, pos_emb, out, batch_size, seq_len, D);
        };
        out.backward_fn = [&input, &pos_emb, &out, batch_size, seq_len, D]() {
            evk::ai::position_add_backward(out.grad(), input.grad(), pos_emb.grad(), batch_size, seq_len, D);
        };
        return out;
    }
    Tensor& rope(Tensor& in, float base = 10000.0f) {
        assert(in.shape.rank() == 3 && "rope expects (B, N, D)");
        assert(in.shape[2] % 2u == 0u && "rope requires an even embedding dimension");
        Tensor& out = tensor(in.shape);
        const uint32_t B = in.shape[0], S = in.shape[1], D = in.shape[2];
        out.forward_fn = [&in, &out, B, S, D, base]() { evk::ai::rope(in, out, B, S, D, base); };
        out.backward_fn = [&in, &out, B, S, D, base]() { evk::ai::rope_backward(out.grad(), in.grad(), B, S, D, base); };
        return out;
    }
    // embeddings (V, D), indices (B, N) of uint16 ids -> (B, N, D).
    Tensor& embed(Tensor& embeddings, Tensor& indices) {
        assert(indices.shape.rank() == 2 && "indices must be (B, N)");
        Tensor& out = tensor(Shape({indices.shape[0], indices.shape[1], embeddings.shape[1]}));
        out.forward_fn = [&embeddings, &indices, &out]() { evk::ai::embed(embeddings, indices, out); };
        out.backward_fn = [&embeddings, &indices, &out]() {
            evk::ai::embed_backward(out.grad(), indices, embeddings.grad());
        };
        return out;
    }
    // logits (B, N, V), targets (B, N) uint16 ids (0 = ignored) -> mean loss.
    // The forward computes the loss and the logits' gradient into a private
    // (B*N, V) tensor; the backward recomputes it (logits may have changed
    // since an earlier eval) and copies it to the logits' gradient.
    Tensor& cross_entropy_loss(Tensor& logits, Tensor& targets) {
        assert(logits.shape.rank() == 3 && "logits must be (B, N, V)");
        assert(targets.shape.rank() == 2 && "targets must be (B, N)");
        const uint32_t B = logits.shape[0], N = logits.shape[1], V = logits.shape[2];
        Tensor& flat_grad = tensor(Shape({B * N, V}));
        Tensor& loss = tensor(Shape({1}));
        auto run = [&logits, &targets, &loss, &flat_grad, B, N, V]() {
            Tensor flat_logits = Tensor::alias(Shape({B * N, V}), logits.buffer);
            Tensor flat_targets = Tensor::alias(Shape({B * N}), targets.buffer);
            evk::ai::cross_entropy_loss(flat_logits, flat_targets, flat_grad, loss);
        };
        loss.forward_fn = run;
        loss.backward_fn = [run, &logits, &flat_grad]() {
            run();
            evk::ai::GetCmd().copy(flat_grad.buffer, logits.grad().buffer,
                                   (uint64_t)logits.shape.count() * sizeof(float16_t));
        };
        return loss;
    }
    Tensor& softmax(Tensor& input, float input_scale = 1.0f) {
        Tensor& out = tensor(input.shape);
        out.forward_fn = [&input, &out, input_scale]() { evk::ai::softmax(input, out, input_scale); };
        out.backward_fn = [&input, &out, input_scale]() {
            evk::ai::softmax_backward(out, out.grad(), input.grad(), input_scale);
        };
        return out;
    }
    // Unfused causal attention, one head over the whole model dimension:
    // scores = q k^T, mask, softmax(scale), probs v; scores and probs
    // (B, N, N) are graph nodes.  scale <= 0 means 1/sqrt(D).
    Tensor& causal_attention(Tensor& q, Tensor& k, Tensor& v, float scale = 0.0f) {
        assert(q.shape.rank() == 3 && k.shape.rank() == 3 && v.shape.rank() == 3);
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
        out.backward_fn = [&q, &k, &v, &scores, &probs, &out, s]() {
            evk::ai::matmul(out.grad(), v, probs.grad(), false, true, false, 16, 16);  // dP = dO v^T
            evk::ai::matmul(probs, out.grad(), v.grad(), true, false, true, 16, 16);   // dv += P^T dO
            evk::ai::softmax_backward(probs, probs.grad(), scores.grad(), s);
            evk::ai::matmul(scores.grad(), k, q.grad(), false, false, true, 16, 16);   // dq += dS k
            evk::ai::matmul(scores.grad(), q, k.grad(), true, false, true, 16, 16);    // dk += dS^T q
        };
        return out;
    }
    void eval(bool backward = false, bool submit = true, bool wait = true) {
        evk::ai::GetCmd();
        if (backward)
            for (auto& n : nodes) evk::ai::zero(n->grad());
        for (auto& n : nodes)
            if (n->forward_fn) n->forward_fn();
        if (backward)
            for (size_t i = nodes.size(); i-- > 0;)
                if (nodes[i]->backward_fn) nodes[i]->backward_fn();
        if (submit) evk::ai::SubmitCmd(wait);
    }
    void step(float lr = 0.001f) {
        for (Tensor* p : params) {
            assert(p->grad_tensor);
            evk::ai::sgd(*p, p->grad(), lr);
        }
    }
    void step_adam(float lr = 0.001f, float beta1 = 0.9f, float beta2 = 0.999f, float epsilon = 1e-4f) {
        for (Tensor* p : params) evk::ai::adam(*p, p->grad(), adam_states[p], lr, beta1, beta2, epsilon);
    }
    void reset_adam() {
        for (auto& kv : adam_states) kv.second.reset();
        adam_states.clear();
    }
};
