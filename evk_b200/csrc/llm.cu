// llm.cu — the decoder that example/main_llm.cpp builds from evk::ai ops
// (CausalAttentionBlock::forward :528-546, MeshTokenModel :588-606,
// sample_autoregressive :622-654), as one device-resident object with a KV
// cache, CUDA-graph decode steps and optional tensor parallelism over NCCL.
//
// Block (pre-norm, as main_llm): x += Wo(attn(rope(Wq n), rope(Wk n), Wv n))
// with n = rms_norm(x); x += W2(gelu(W1 rms_norm(x))); logits =
// rms_norm(x) . LM head; next id = greedy argmax (reference tie rule).
// Attention is multi-head with RoPE per head (head_dim rotation, position
// offset for decode), causal.  Norms have no gain, as evk::ai::rms_norm.
//
// Tensor parallel (Megatron layout): rank r owns q/k/v heads
// [r H/t, (r+1) H/t) (columns of Wqkv), the matching rows of Wo, columns
// [r F/t, ...) of W1 and rows of W2, and vocabulary rows [r V/t, ...) of the
// LM head.  The Wo and W2 products are partial sums, added across ranks with
// one ncclAllReduce each; the greedy ids combine the ranks' 64-bit selection
// keys (greedy_key.cuh) with one ncclAllGather, which yields the same token as
// a single-GPU argmax over the whole vocabulary.
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <cstdlib>
#include <vector>

#include "common.cuh"
#include "decode_mega.cuh"
#include "greedy_key.cuh"

namespace evkcu {
namespace {

constexpr int kT = 256;

inline unsigned grid_for_items(uint64_t n, int threads = kT) {
    DeviceState* s = state();
    uint64_t want = (n + threads - 1) / threads;
    uint64_t cap = (uint64_t)(s ? s->sm_count : 148) * 16;
    return (unsigned)std::max<uint64_t>(1, std::min(want, cap));
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// dst[r, c] (leading dim ld) = N(0, std) drawn from the element's global index
// (row_off + r) * gcols + col_off + c of tensor `tid`: splitmix64 -> Box-Muller.
template <typename T>
__global__ void fill_normal_kernel(T* dst, uint32_t rows, uint32_t cols, uint64_t ld, uint64_t seed, uint32_t tid,
                                   uint64_t row_off, uint64_t col_off, uint64_t gcols, float std) {
    const uint64_t n = (uint64_t)rows * cols;
    const uint64_t base = mix64(seed ^ (0xD1B54A32D192ED03ull * (tid + 1)));
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = i / cols, c = i % cols;
        const uint64_t g = (row_off + r) * gcols + col_off + c;
        const uint64_t z1 = mix64(base ^ (2 * g)), z2 = mix64(base ^ (2 * g + 1));
        const float u1 = ((uint32_t)(z1 >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
        const float u2 = (uint32_t)(z2 >> 40) * (1.0f / 16777216.0f);          // [0, 1)
        const float v = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        dst[r * ld + c] = Elem<T>::from_f(v * std);
    }
}

// After a decode step: one more cached position.
__global__ void advance_kernel(uint32_t* d_pos, uint32_t* d_len) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    const uint32_t p = *d_pos + 1;
    *d_pos = p;
    d_pos[2] += 1;  // decode-step counter (never reset): all-reduce flag values
    *d_len = p + 1;
}
__global__ void set_pos_kernel(uint32_t* d_pos, uint32_t* d_len, uint32_t pos) {
    *d_pos = pos;
    *d_len = pos + 1;
}

// Per sequence b: the maximum selection key over logits[b, 0:Vl] whose tokens
// are voff + j (one CTA per sequence).
template <typename T>
__global__ void argmax_key_kernel(const T* __restrict__ logits, uint32_t Vl, uint32_t voff,
                                  unsigned long long* __restrict__ keys) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    __shared__ unsigned long long sh[32];
    const T* row = logits + (uint64_t)blockIdx.x * Vl;
    unsigned long long best = 0;
    for (uint32_t j = threadIdx.x; j < Vl; j += blockDim.x) {
        const unsigned long long k = elem_key(Elem<T>::to_f(row[j]), voff + j);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
        best = t > best ? t : best;
    }
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x < 32) {
        best = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
            best = t > best ? t : best;
        }
        if (threadIdx.x == 0) keys[blockIdx.x] = best;
    }
}

// ids[b] = token of max_r keys[r * B + b] (token 0 when nothing is selectable).
__global__ void keys_to_ids_kernel(const unsigned long long* __restrict__ keys, uint32_t ranks, uint32_t B,
                                   uint32_t* __restrict__ ids) {
    pdl_trigger();  // the next kernel may launch and run its prologue now
    pdl_wait();     // inputs come from earlier kernels (see launch_pdl)
    const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    unsigned long long best = 0;
    for (uint32_t r = 0; r < ranks; ++r) best = keys[(uint64_t)r * B + b] > best ? keys[(uint64_t)r * B + b] : best;
    ids[b] = best ? key_to_offset(best) : 0u;
}

}  // namespace
}  // namespace evkcu

using namespace evkcu;

struct LlmLayer {
    void *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr, *kc = nullptr, *vc = nullptr;
};

struct evkcu_llm {
    evkcu_llm_config cfg{};
    ncclComm_t comm = nullptr;
    int device = 0;
    uint32_t Dh = 0, Hl = 0, Hkvl = 0, Fl = 0, Vl = 0, C = 0;
    void* emb = nullptr;
    void* lm_head = nullptr;  // [D, Vl] when untied
    std::vector<LlmLayer> layers;
    void *x = nullptr, *xn = nullptr, *q = nullptr, *attn = nullptr,
         *tmp = nullptr, *h1 = nullptr, *xl = nullptr, *logits = nullptr, *logits_all = nullptr;
    unsigned long long *keys = nullptr, *keys_all = nullptr;
    uint32_t *d_pos = nullptr, *d_len = nullptr, *d_epoch = nullptr;
    float2* rope_cs = nullptr;  // (cos, sin) per position and rotation pair
    // Fused all-reduce of the decode Wo / W2 projections (tp > 1): this
    // rank's (value, flag) buffer, and every rank's through IPC.
    uint2* ar_buf = nullptr;
    GemvAllReduce ar{};
    bool ar_ready = false;
    std::vector<void*> ipc_opened;
    uint32_t *gin = nullptr, *gout = nullptr;  // fixed ids in/out words of the decode graph
    // Persistent one-kernel decode step (decode_mega.cu) for small models.
    void* mega_scratch = nullptr;
    void* mega_layers = nullptr;  // device MegaLayer [layers]
    bool mega_ok = false;
    uint32_t cur_len = 0, batch = 0;
    std::vector<void*> allocs;
    std::unordered_map<uint32_t, cudaGraphExec_t> graphs;  // by batch size
    std::unordered_map<uint32_t, std::vector<void*>> graph_ws;
    std::unordered_map<uint32_t, int> eager_steps;
};

namespace {

constexpr size_t kE = 2;  // bytes per element (fp16 / bf16)

int llm_alloc(evkcu_llm* m, void** p, size_t bytes) {
    EVKCU_CUDA_TRY(cudaMalloc(p, bytes ? bytes : 16));
    m->allocs.push_back(*p);
    return EVKCU_OK;
}

int nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) return fail(EVKCU_COMM_ERROR, std::string(what) + ": " + ncclGetErrorString(r));
    return EVKCU_OK;
}

ncclDataType_t nccl_type(int dtype) { return dtype == EVKCU_BF16 ? ncclBfloat16 : ncclFloat16; }

#define LLM_TRY(expr)      \
    do {                   \
        int _r = (expr);   \
        if (_r) return _r; \
    } while (0)

// Largest rows x d_model for the fused decode all-reduce.  Its (value, flag)
// pairs of fp32 partials carry 4x the bytes of NCCL's 16-bit all-reduce;
// measured at tp = 2 (decode ms per step, fused / NCCL): C3 1 x 512 0.235 /
// 0.322, C4 8 x 2048 1.78 / 2.22, C5 16 x 4096 7.19 / 6.91.
constexpr uint64_t kFusedArMaxElems = 32768;
// Above that, up to this size, the partials travel as 16-bit values (the
// numerics of NCCL's all-reduce of 16-bit partials, half the fp32 bytes).
constexpr uint64_t kFusedArHalfMaxElems = 131072;

// Wo / W2 product into the residual.  On one GPU acc_c fuses the add; with
// tensor parallelism the product is a partial sum, summed across ranks first.
int proj_residual(evkcu_llm* m, const void* a, const void* w, uint32_t rows, uint32_t K, bool decode,
                  uint32_t callsite, cudaStream_t st) {
    const uint32_t D = m->cfg.d_model;
    const int dt = m->cfg.dtype;
    if (m->cfg.tp_size == 1) return evkcu_matmul(a, w, m->x, 1, rows, K, D, 0, 0, 0, EVKCU_MM_ACC_C, dt, st);
    static const int force_half = [] {
        const char* e = getenv("EVKCU_FUSED_AR_HALF");
        return e && atoi(e) ? 1 : 0;
    }();
    const uint64_t elems = (uint64_t)rows * D;
    // The 16-bit form is used on its own only at tp = 2, where it was measured
    // against NCCL; the switch forces it at any tp (the TP test).
    const bool half_ok = force_half || m->cfg.tp_size == 2;
    const bool fuse = elems <= kFusedArMaxElems || (half_ok && elems <= kFusedArHalfMaxElems);
    if (decode && rows <= 16 && m->ar_ready && fuse) {
        // GEMV + all-reduce over NVLink peer memory + residual add, one kernel.
        GemvAllReduce ar = m->ar;
        ar.callsite = callsite;
        ar.half = (force_half || elems > kFusedArMaxElems) ? 1u : 0u;
        return gemv_allreduce_residual(a, w, m->x, rows, K, D, ar, dt, st);
    }
    LLM_TRY(evkcu_matmul(a, w, m->tmp, 1, rows, K, D, 0, 0, 0, 0, dt, st));
    const uint64_t n = (uint64_t)rows * D;
    LLM_TRY(nccl_check(ncclAllReduce(m->tmp, m->tmp, n, nccl_type(dt), ncclSum, m->comm, st), "ncclAllReduce"));
    return evkcu_add(m->x, m->tmp, m->x, n, dt, st);
}

// The transformer blocks over B * S rows of m->x (S rows per sequence).
// Prefill: positions 0..S-1, causal flash attention over contiguous K / V.
// Decode (S = 1): position *d_pos, attention over the cache up to *d_len.
int run_blocks(evkcu_llm* m, uint32_t B, uint32_t S, bool decode, cudaStream_t st) {
    const evkcu_llm_config& c = m->cfg;
    const uint32_t R = B * S, D = c.d_model;
    const int dt = c.dtype;
    for (uint32_t l = 0; l < c.layers; ++l) {
        LlmLayer& L = m->layers[l];
        LLM_TRY(evkcu_rms_norm(m->x, m->xn, nullptr, R, D, c.eps, dt, st));
        // QKV projection whose epilogue applies RoPE to q and k and writes q
        // and the cache rows directly (the [R, C] product is never stored).
        QkvRope qr;
        qr.q = m->q;
        qr.kc = L.kc;
        qr.vc = L.vc;
        qr.Hq = m->Hl;
        qr.Hk = m->Hkvl;
        qr.Dh = m->Dh;
        qr.S = S;
        qr.max_len = c.max_seq;
        qr.pos0 = 0;
        qr.d_pos = decode ? m->d_pos : nullptr;
        qr.base = c.rope_base;
        qr.cs = m->rope_cs;
        qr.cs_len = c.max_seq;
        LLM_TRY(matmul_ex(m->xn, L.wqkv, m->q /* not written */, 1, R, D, m->C, 0, 0, 0, 0, dt, 0, st, &qr));
        if (decode)
            LLM_TRY(evkcu_single_query_attention_devlen(m->q, L.kc, L.vc, m->attn, B, m->Hl, m->Hkvl, m->Dh,
                                                         c.max_seq, m->d_len, 0.0f, dt, st));
        else
            // Prefill attention reads K and V straight from the cache rows
            // the append kernel just wrote (batch stride max_seq rows).
            LLM_TRY(flash_attention_kv_strided(m->q, L.kc, L.vc, m->attn, B, S, m->Hl, m->Hkvl, m->Dh, 0.0f,
                                               EVKCU_ATTN_CAUSAL, dt, (uint64_t)c.max_seq * m->Hkvl * m->Dh, st));
        LLM_TRY(proj_residual(m, m->attn, L.wo, R, m->Hl * m->Dh, decode, 2 * l, st));
        LLM_TRY(evkcu_rms_norm(m->x, m->xn, nullptr, R, D, c.eps, dt, st));
        // W1 with the GELU applied in the GEMM / GEMV epilogue.
        LLM_TRY(matmul_ex(m->xn, L.w1, m->h1, 1, R, D, m->Fl, 0, 0, 0, 0, dt, 1, st));
        LLM_TRY(proj_residual(m, m->h1, L.w2, R, m->Fl, decode, 2 * l + 1, st));
    }
    return EVKCU_OK;
}

// Final norm, LM head and greedy ids for the B rows of `xrows` ([B, D]).
int head_and_sample(evkcu_llm* m, const void* xrows, uint32_t B, uint32_t* next_ids, void* logits_out,
                    cudaStream_t st) {
    const evkcu_llm_config& c = m->cfg;
    const int dt = c.dtype;
    const uint32_t D = c.d_model;
    const bool tied = c.tied_embeddings;
    const void* w_head = tied ? (const void*)((const char*)m->emb + (uint64_t)c.tp_rank * m->Vl * D * kE) : m->lm_head;
    if (B <= 16 && !logits_out) {
        // Fused LM head + greedy argmax: the GEMV reduces its own outputs to
        // selection keys, so the [B, V] logits never reach HBM.
        LLM_TRY(evkcu_rms_norm(xrows, m->xn, nullptr, B, D, c.eps, dt, st));
        if (c.tp_size == 1)
            return gemv_argmax(m->xn, w_head, B, D, m->Vl, tied, 0, nullptr, next_ids, nullptr, dt, st);
        LLM_TRY(gemv_argmax(m->xn, w_head, B, D, m->Vl, tied, c.tp_rank * m->Vl, (unsigned long long*)m->keys,
                            nullptr, nullptr, dt, st));
        LLM_TRY(nccl_check(ncclAllGather(m->keys, m->keys_all, B, ncclUint64, m->comm, st), "ncclAllGather(keys)"));
        return launch_pdl("llm keys_to_ids", keys_to_ids_kernel, (B + 127) / 128, 128, 0, st,
                          (const unsigned long long*)m->keys_all, c.tp_size, B, next_ids);
    }
    if (tied) {
        LLM_TRY(evkcu_rms_norm(xrows, m->xn, nullptr, B, D, c.eps, dt, st));
        const void* eshard = (const char*)m->emb + (uint64_t)c.tp_rank * m->Vl * D * kE;
        LLM_TRY(evkcu_matmul(m->xn, eshard, m->logits, 1, B, D, m->Vl, 0, 0, 0, EVKCU_MM_TRANSPOSE_B, dt, st));
    } else {
        LLM_TRY(evkcu_rms_norm(xrows, m->xn, nullptr, B, D, c.eps, dt, st));
        LLM_TRY(evkcu_matmul(m->xn, m->lm_head, m->logits, 1, B, D, m->Vl, 0, 0, 0, 0, dt, st));
    }
    if (c.tp_size == 1) {
        LLM_TRY(evkcu_greedy_sample(m->logits, next_ids, B, 1, m->Vl, 0, 0, m->Vl, 4, dt, st));
        if (logits_out)
            EVKCU_CUDA_TRY(cudaMemcpyAsync(logits_out, m->logits, (size_t)B * m->Vl * kE, cudaMemcpyDeviceToDevice, st));
        return EVKCU_OK;
    }
    LLM_TRY(EVKCU_DISPATCH_DTYPE(dt, T, [&] {
        return launch_pdl("llm argmax_key", argmax_key_kernel<T>, B, 1024, 0, st, (const T*)m->logits, m->Vl,
                          c.tp_rank * m->Vl, m->keys);
    }));
    LLM_TRY(nccl_check(ncclAllGather(m->keys, m->keys_all, B, ncclUint64, m->comm, st), "ncclAllGather(keys)"));
    LLM_TRY(launch_pdl("llm keys_to_ids", keys_to_ids_kernel, (B + 127) / 128, 128, 0, st,
                       (const unsigned long long*)m->keys_all, c.tp_size, B, next_ids));
    if (logits_out) {
        // [t][B][Vl] -> [B][t * Vl]
        LLM_TRY(nccl_check(ncclAllGather(m->logits, m->logits_all, (size_t)B * m->Vl, nccl_type(dt), m->comm, st),
                           "ncclAllGather(logits)"));
        for (uint32_t r = 0; r < c.tp_size; ++r)
            EVKCU_CUDA_TRY(cudaMemcpy2DAsync((char*)logits_out + (size_t)r * m->Vl * kE, (size_t)c.vocab * kE,
                                             (const char*)m->logits_all + (size_t)r * B * m->Vl * kE,
                                             (size_t)m->Vl * kE, (size_t)m->Vl * kE, B, cudaMemcpyDeviceToDevice, st));
    }
    return EVKCU_OK;
}

bool use_decode_mega(const evkcu_llm* m) { return m->mega_ok; }

int decode_body(evkcu_llm* m, const uint32_t* ids, uint32_t* next_ids, void* logits_out, cudaStream_t st) {
    const evkcu_llm_config& c = m->cfg;
    const uint32_t B = m->batch;
    if (use_decode_mega(m)) {
        MegaHost h{};
        h.B = B;
        h.D = c.d_model;
        h.H = c.heads;
        h.Hkv = c.kv_heads;
        h.Dh = m->Dh;
        h.F = c.hidden;
        h.V = c.vocab;
        h.layers = c.layers;
        h.max_seq = c.max_seq;
        h.tied = c.tied_embeddings ? 1u : 0u;
        h.eps = c.eps;
        h.rope_base = c.rope_base;
        h.emb = m->emb;
        h.lm_head = m->lm_head;
        h.layer_table = m->mega_layers;
        h.x = m->x;
        h.q = m->q;
        h.attn = m->attn;
        h.h1 = m->h1;
        h.logits = logits_out;
        h.rope_cs = m->rope_cs;
        h.d_pos = m->d_pos;
        h.d_len = m->d_len;
        h.ids_in = ids;
        h.ids_out = next_ids;
        h.scratch = m->mega_scratch;
        return decode_mega_step(h, c.dtype, st);
    }
    LLM_TRY(evkcu_embed(m->emb, ids, m->x, c.vocab, c.d_model, B, 4, c.dtype, st));
    LLM_TRY(run_blocks(m, B, 1, true, st));
    LLM_TRY(head_and_sample(m, m->x, B, next_ids, logits_out, st));
    return launch_pdl("llm advance", advance_kernel, 1, 1, 0, st, m->d_pos, m->d_len);
}

std::vector<void*> ws_signature() {
    DeviceState* s = state();
    std::vector<void*> v;
    for (int i = 0; i < WS_COUNT; ++i) v.push_back(s->ws[i]);
    return v;
}

}  // namespace

// ------------------------------------------------------------------ C ABI ----
extern "C" int evkcu_comm_unique_id(void* id128) {
    EVKCU_CHECK_ARG(id128, EVKCU_BAD_ARG, "evkcu_comm_unique_id: null pointer");
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    ncclUniqueId id;
    LLM_TRY(nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId"));
    std::memcpy(id128, &id, sizeof(id));
    return EVKCU_OK;
}

extern "C" int evkcu_comm_init(const void* id128, int rank, int world, void** comm) {
    EVKCU_CHECK_ARG(id128 && comm && world >= 1 && rank >= 0 && rank < world, EVKCU_BAD_ARG, "evkcu_comm_init: bad args");
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    ncclComm_t c = nullptr;
    LLM_TRY(nccl_check(ncclCommInitRank(&c, world, id, rank), "ncclCommInitRank"));
    *comm = c;
    return EVKCU_OK;
}

extern "C" int evkcu_comm_destroy(void* comm) {
    if (comm) LLM_TRY(nccl_check(ncclCommDestroy((ncclComm_t)comm), "ncclCommDestroy"));
    return EVKCU_OK;
}

// Exchanges CUDA IPC handles of every rank's all-reduce buffer
// (ncclAllGather of the 64-byte handles), maps the peers' into this
// process, then agrees across ranks (ncclAllReduce, min) on whether every rank
// succeeded and has the fused path switched on.  Every rank issues the same
// two collectives whatever happens locally, so a failure on one rank (or
// EVKCU_DISABLE_FUSED_ALLREDUCE set on some ranks only) makes all of them keep
// the NCCL all-reduce instead of one rank waiting for peers that never arrive.
// `xch` is a device buffer of 128 * (t + 1) + 4 bytes allocated by the caller.
static void setup_allreduce(evkcu_llm* m, char* xch) {
    const uint32_t t = m->cfg.tp_size, rank = m->cfg.tp_rank;
    if (t > 8) return;  // same decision on every rank: t is shared
    // Flags are step * 256 + callsite + 1 with callsite < 2 * layers.
    bool ok = m->ar_buf && 2 * m->cfg.layers < 255 && getenv("EVKCU_DISABLE_FUSED_ALLREDUCE") == nullptr;
    const size_t bbytes = (size_t)2 * t * 16 * m->cfg.d_model * sizeof(uint2);
    ok = ok && cudaMemset(m->ar_buf, 0, bbytes) == cudaSuccess;
    cudaIpcMemHandle_t h[1];
    std::memset(h, 0, sizeof(h));
    ok = ok && cudaIpcGetMemHandle(&h[0], m->ar_buf) == cudaSuccess;
    cudaGetLastError();
    std::vector<cudaIpcMemHandle_t> all(t);
    bool comm_ok = cudaMemcpy(xch, h, sizeof(h), cudaMemcpyHostToDevice) == cudaSuccess &&
                   ncclAllGather(xch, xch + sizeof(h), sizeof(h), ncclUint8, m->comm, 0) == ncclSuccess &&
                   cudaStreamSynchronize(0) == cudaSuccess &&
                   cudaMemcpy(all.data(), xch + sizeof(h), sizeof(h) * t, cudaMemcpyDeviceToHost) == cudaSuccess;
    ok = ok && comm_ok;
    GemvAllReduce ar;
    ar.tp = t;
    ar.rank = rank;
    ar.epoch = m->d_epoch;
    for (uint32_t q = 0; q < t && ok; ++q) {
        if (q == rank) {
            ar.buf[q] = m->ar_buf;
            continue;
        }
        void* pb = nullptr;
        ok = cudaIpcOpenMemHandle(&pb, all[q], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
        if (ok) m->ipc_opened.push_back(pb);
        ar.buf[q] = (uint2*)pb;
    }
    cudaGetLastError();
    // Agreement: the fused path is used only if it is ready on every rank.
    int32_t* flag = (int32_t*)(xch + sizeof(h) * (t + 1));
    const int32_t mine = ok ? 1 : 0;
    int32_t agreed = 0;
    if (!(cudaMemcpy(flag, &mine, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
          ncclAllReduce(flag, flag, 1, ncclInt32, ncclMin, m->comm, 0) == ncclSuccess &&
          cudaStreamSynchronize(0) == cudaSuccess &&
          cudaMemcpy(&agreed, flag, 4, cudaMemcpyDeviceToHost) == cudaSuccess)) {
        cudaGetLastError();
        agreed = 0;
    }
    m->ar = ar;
    m->ar_ready = agreed == 1;
}

extern "C" int evkcu_llm_create(const evkcu_llm_config* cfg, void* comm, evkcu_llm** out) {
    EVKCU_CHECK_ARG(cfg && out, EVKCU_BAD_ARG, "evkcu_llm_create: null pointer");
    const evkcu_llm_config& c = *cfg;
    const uint32_t t = c.tp_size ? c.tp_size : 1;
    EVKCU_CHECK_ARG(c.dtype == EVKCU_F16 || c.dtype == EVKCU_BF16, EVKCU_BAD_ARG, "evkcu_llm_create: dtype");
    EVKCU_CHECK_ARG(c.layers && c.d_model && c.heads && c.kv_heads && c.hidden && c.vocab && c.max_batch && c.max_seq,
                    EVKCU_BAD_SHAPE, "evkcu_llm_create: zero dimension");
    EVKCU_CHECK_ARG(c.d_model % c.heads == 0 && c.heads % c.kv_heads == 0, EVKCU_BAD_SHAPE,
                    "evkcu_llm_create: heads must divide d_model and kv_heads must divide heads");
    const uint32_t Dh = c.d_model / c.heads;
    EVKCU_CHECK_ARG(Dh % 16 == 0 && Dh <= 256, EVKCU_BAD_SHAPE, "evkcu_llm_create: head_dim must be a multiple of 16");
    EVKCU_CHECK_ARG(c.heads % t == 0 && c.kv_heads % t == 0 && c.hidden % t == 0 && c.vocab % t == 0 && c.tp_rank < t,
                    EVKCU_BAD_SHAPE, "evkcu_llm_create: heads, kv_heads, hidden and vocab must divide by tp_size");
    EVKCU_CHECK_ARG(t == 1 || comm, EVKCU_BAD_ARG, "evkcu_llm_create: tp_size > 1 needs a communicator");
    EVKCU_CHECK_ARG(c.d_model % 8 == 0 && (c.hidden / t) % 8 == 0 && (c.vocab / t) % 8 == 0, EVKCU_BAD_SHAPE,
                    "evkcu_llm_create: d_model, hidden/tp and vocab/tp must be multiples of 8");
    DeviceState* ds = state();
    EVKCU_CHECK_ARG(ds, EVKCU_CUDA_ERROR, "evkcu_llm_create: no device state");
    auto* m = new evkcu_llm();
    m->cfg = c;
    m->cfg.tp_size = t;
    m->comm = (ncclComm_t)comm;
    m->device = ds->device;
    m->Dh = Dh;
    m->Hl = c.heads / t;
    m->Hkvl = c.kv_heads / t;
    m->Fl = c.hidden / t;
    m->Vl = c.vocab / t;
    m->C = (m->Hl + 2 * m->Hkvl) * Dh;
    const uint64_t D = c.d_model, R = (uint64_t)c.max_batch * c.max_seq;
    int r = EVKCU_OK;
    auto A = [&](void** p, size_t bytes) {
        if (r == EVKCU_OK) r = llm_alloc(m, p, bytes);
    };
    A(&m->emb, (size_t)c.vocab * D * kE);
    if (!c.tied_embeddings) A(&m->lm_head, (size_t)D * m->Vl * kE);
    m->layers.resize(c.layers);
    for (auto& L : m->layers) {
        A(&L.wqkv, (size_t)D * m->C * kE);
        A(&L.wo, (size_t)m->Hl * Dh * D * kE);
        A(&L.w1, (size_t)D * m->Fl * kE);
        A(&L.w2, (size_t)m->Fl * D * kE);
        A(&L.kc, (size_t)c.max_batch * c.max_seq * m->Hkvl * Dh * kE);
        A(&L.vc, (size_t)c.max_batch * c.max_seq * m->Hkvl * Dh * kE);
    }
    A(&m->x, R * D * kE);
    A(&m->xn, R * D * kE);
    A(&m->q, R * m->Hl * Dh * kE);
    A(&m->attn, R * m->Hl * Dh * kE);
    if (t > 1) A(&m->tmp, R * D * kE);
    A(&m->h1, R * m->Fl * kE);
    A(&m->xl, (size_t)c.max_batch * D * kE);
    A(&m->logits, (size_t)c.max_batch * m->Vl * kE);
    if (t > 1) {
        A(&m->logits_all, (size_t)c.max_batch * c.vocab * kE);
        A((void**)&m->keys, (size_t)c.max_batch * 8);
        A((void**)&m->keys_all, (size_t)c.max_batch * t * 8);
    }
    A((void**)&m->d_pos, 4 * sizeof(uint32_t));  // position, length, decode-step counter
    A((void**)&m->rope_cs, (size_t)c.max_seq * (Dh / 2) * sizeof(float2));
    char* xch = nullptr;  // handle exchange / agreement word of setup_allreduce
    if (t > 1) {
        A((void**)&xch, (size_t)128 * (t + 1) + 4);
        A((void**)&m->ar_buf, (size_t)2 * t * 16 * D * sizeof(uint2));
    }
    A((void**)&m->gin, (size_t)c.max_batch * 4);
    A((void**)&m->gout, (size_t)c.max_batch * 4);
    if (r != EVKCU_OK) {
        evkcu_llm_destroy(m);
        return r;
    }
    m->d_len = m->d_pos + 1;
    m->d_epoch = m->d_pos + 2;
    {
        const uint32_t init[4] = {0u, 0u, 1u, 0u};
        EVKCU_CUDA_TRY(cudaMemcpy(m->d_pos, init, sizeof(init), cudaMemcpyHostToDevice));
    }
    if ((r = rope_table(m->rope_cs, c.max_seq, Dh, c.rope_base, 0)) != EVKCU_OK) {
        evkcu_llm_destroy(m);
        return r;
    }
    // Opt-in (EVKCU_DECODE_MEGA=1 when the model is created): measured slower
    // than the per-op chain at C3 (0.28 vs 0.20 ms per step: a grid barrier
    // costs 2.3 us and each phase adds L2 round trips).
    const char* mega_env = getenv("EVKCU_DECODE_MEGA");
    if (t == 1 && mega_env && atoi(mega_env) == 1 &&
        decode_mega_supported(c.max_batch, c.d_model, c.heads, c.kv_heads, Dh, c.hidden, c.vocab,
                              c.tied_embeddings != 0)) {
        // The persistent decode step: its scratch (zero-filled) and the
        // per-layer pointer table it reads.
        const size_t sb = decode_mega_scratch_bytes(c.max_batch, c.d_model, c.heads, c.kv_heads, Dh, c.hidden,
                                                    c.max_seq, ds->sm_count);
        std::vector<MegaLayer> tab(c.layers);
        for (uint32_t l = 0; l < c.layers; ++l)
            tab[l] = {m->layers[l].wqkv, m->layers[l].wo, m->layers[l].w1, m->layers[l].w2, m->layers[l].kc,
                      m->layers[l].vc};
        if ((r = llm_alloc(m, &m->mega_scratch, sb)) != EVKCU_OK ||
            (r = llm_alloc(m, &m->mega_layers, sizeof(MegaLayer) * c.layers)) != EVKCU_OK) {
            evkcu_llm_destroy(m);
            return r;
        }
        EVKCU_CUDA_TRY(cudaMemset(m->mega_scratch, 0, sb));
        EVKCU_CUDA_TRY(cudaMemcpy(m->mega_layers, tab.data(), sizeof(MegaLayer) * c.layers, cudaMemcpyHostToDevice));
        m->mega_ok = true;
    }
    EVKCU_CUDA_TRY(cudaDeviceSynchronize());
    if (t > 1) setup_allreduce(m, xch);  // all ranks fall back to NCCL unless every rank mapped its peers
    *out = m;
    return EVKCU_OK;
}

extern "C" int evkcu_llm_destroy(evkcu_llm* m) {
    if (!m) return EVKCU_OK;
    cudaDeviceSynchronize();
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    for (void* p : m->ipc_opened) cudaIpcCloseMemHandle(p);
    for (void* p : m->allocs) cudaFree(p);
    delete m;
    return EVKCU_OK;
}

extern "C" uint32_t evkcu_llm_length(const evkcu_llm* m) { return m ? m->cur_len : 0; }

extern "C" uint32_t evkcu_llm_fused_allreduce(const evkcu_llm* m) { return m && m->ar_ready ? 1u : 0u; }

extern "C" int evkcu_llm_init_random(evkcu_llm* m, uint64_t seed, float std, void* stream) {
    EVKCU_CHECK_ARG(m, EVKCU_BAD_ARG, "evkcu_llm_init_random: null model");
    const evkcu_llm_config& c = m->cfg;
    cudaStream_t st = as_stream(stream);
    const uint32_t D = c.d_model, Dh = m->Dh, rk = c.tp_rank;
    const uint64_t gq = (uint64_t)(c.heads + 2 * c.kv_heads) * Dh;  // global Wqkv columns
    return EVKCU_DISPATCH_DTYPE(c.dtype, T, [&]() -> int {
        // (dst, rows, cols, ld, tensor id, row_off, col_off, global cols)
        auto fill = [&](void* dst, uint32_t rows, uint32_t cols, uint64_t ld, uint32_t tid, uint64_t ro, uint64_t co,
                        uint64_t gc) -> int {
            fill_normal_kernel<T><<<grid_for_items((uint64_t)rows * cols), kT, 0, st>>>((T*)dst, rows, cols, ld, seed,
                                                                                       tid, ro, co, gc, std);
            return after_launch("llm init_random");
        };
        LLM_TRY(fill(m->emb, c.vocab, D, D, 1, 0, 0, D));
        if (!c.tied_embeddings) LLM_TRY(fill(m->lm_head, D, m->Vl, m->Vl, 2, 0, (uint64_t)rk * m->Vl, c.vocab));
        for (uint32_t l = 0; l < c.layers; ++l) {
            LlmLayer& L = m->layers[l];
            const uint32_t b = 16 + 8 * l;
            const uint32_t hq = m->Hl * Dh, hk = m->Hkvl * Dh;
            LLM_TRY(fill(L.wqkv, D, hq, m->C, b + 0, 0, (uint64_t)rk * hq, gq));
            LLM_TRY(fill((T*)L.wqkv + hq, D, hk, m->C, b + 0, 0, (uint64_t)c.heads * Dh + (uint64_t)rk * hk, gq));
            LLM_TRY(fill((T*)L.wqkv + hq + hk, D, hk, m->C, b + 0, 0,
                         (uint64_t)(c.heads + c.kv_heads) * Dh + (uint64_t)rk * hk, gq));
            LLM_TRY(fill(L.wo, hq, D, D, b + 1, (uint64_t)rk * hq, 0, D));
            LLM_TRY(fill(L.w1, D, m->Fl, m->Fl, b + 2, 0, (uint64_t)rk * m->Fl, c.hidden));
            LLM_TRY(fill(L.w2, m->Fl, D, D, b + 3, (uint64_t)rk * m->Fl, 0, D));
        }
        return EVKCU_OK;
    });
}

extern "C" int evkcu_llm_set_weight(evkcu_llm* m, const char* name, uint32_t layer, const void* src, void* stream) {
    EVKCU_CHECK_ARG(m && name && src, EVKCU_BAD_ARG, "evkcu_llm_set_weight: null pointer");
    const evkcu_llm_config& c = m->cfg;
    cudaStream_t st = as_stream(stream);
    const uint32_t D = c.d_model, Dh = m->Dh, rk = c.tp_rank;
    const std::string n(name);
    // `rows` rows of `width` elements from src (row pitch spitch, column
    // offset scol) to dst (row pitch dpitch, column offset dcol)
    auto copy2d = [&](void* dst, size_t dpitch, size_t dcol, const void* s, size_t spitch, size_t scol, size_t width,
                      size_t rows) -> int {
        EVKCU_CUDA_TRY(cudaMemcpy2DAsync((char*)dst + dcol * kE, dpitch * kE, (const char*)s + scol * kE, spitch * kE,
                                         width * kE, rows, cudaMemcpyDefault, st));
        return EVKCU_OK;
    };
    if (n == "embedding") return copy2d(m->emb, D, 0, src, D, 0, D, c.vocab);
    if (n == "lm_head") {
        EVKCU_CHECK_ARG(!c.tied_embeddings, EVKCU_BAD_ARG, "evkcu_llm_set_weight: model ties the LM head");
        return copy2d(m->lm_head, m->Vl, 0, src, c.vocab, (size_t)rk * m->Vl, m->Vl, D);
    }
    EVKCU_CHECK_ARG(layer < c.layers, EVKCU_BAD_ARG, "evkcu_llm_set_weight: layer out of range");
    LlmLayer& L = m->layers[layer];
    const size_t hq = (size_t)m->Hl * Dh, hk = (size_t)m->Hkvl * Dh;
    const size_t gq = (size_t)(c.heads + 2 * c.kv_heads) * Dh;
    if (n == "wqkv") {
        LLM_TRY(copy2d(L.wqkv, m->C, 0, src, gq, rk * hq, hq, D));
        LLM_TRY(copy2d(L.wqkv, m->C, hq, src, gq, (size_t)c.heads * Dh + rk * hk, hk, D));
        return copy2d(L.wqkv, m->C, hq + hk, src, gq, (size_t)(c.heads + c.kv_heads) * Dh + rk * hk, hk, D);
    }
    if (n == "wo") return copy2d(L.wo, D, 0, (const char*)src + rk * hq * D * kE, D, 0, D, hq);
    if (n == "w1") return copy2d(L.w1, m->Fl, 0, src, c.hidden, (size_t)rk * m->Fl, m->Fl, D);
    if (n == "w2") return copy2d(L.w2, D, 0, (const char*)src + (size_t)rk * m->Fl * D * kE, D, 0, D, m->Fl);
    return fail(EVKCU_BAD_ARG, "evkcu_llm_set_weight: unknown weight " + n);
}

// ---- weight blob ------------------------------------------------------------
// One file holding every weight of a model in its storage type, unsharded:
// a 64-byte header (magic "EVKWBLOB", then uint32 version 1, dtype, layers,
// d_model, heads, kv_heads, hidden, vocab, tied_embeddings, zero padding),
// then the tensors row-major in this order: embedding [V, D], lm_head [D, V]
// (untied models only), and per layer wqkv [D, (H + 2 Hkv) Dh], wo [H Dh, D],
// w1 [D, F], w2 [F, D] (the layouts of evkcu_llm_set_weight).
namespace {
constexpr char kBlobMagic[8] = {'E', 'V', 'K', 'W', 'B', 'L', 'O', 'B'};
struct BlobHeader {
    char magic[8];
    uint32_t version, dtype, layers, d_model, heads, kv_heads, hidden, vocab, tied;
    uint32_t pad[5];
};
static_assert(sizeof(BlobHeader) == 64, "blob header is 64 bytes");

struct BlobTensor {
    const char* name;
    uint32_t layer;
    uint64_t elems;
};
std::vector<BlobTensor> blob_layout(const evkcu_llm_config& c) {
    const uint64_t D = c.d_model, Dh = D / c.heads, V = c.vocab, F = c.hidden;
    std::vector<BlobTensor> t;
    t.push_back({"embedding", 0, V * D});
    if (!c.tied_embeddings) t.push_back({"lm_head", 0, D * V});
    for (uint32_t l = 0; l < c.layers; ++l) {
        t.push_back({"wqkv", l, D * (c.heads + 2ull * c.kv_heads) * Dh});
        t.push_back({"wo", l, (uint64_t)c.heads * Dh * D});
        t.push_back({"w1", l, D * F});
        t.push_back({"w2", l, F * D});
    }
    return t;
}
}  // namespace

extern "C" int evkcu_llm_load(evkcu_llm* m, const char* path, void* stream) {
    EVKCU_CHECK_ARG(m && path, EVKCU_BAD_ARG, "evkcu_llm_load: null pointer");
    const evkcu_llm_config& c = m->cfg;
    FILE* f = std::fopen(path, "rb");
    EVKCU_CHECK_ARG(f, EVKCU_BAD_ARG, std::string("evkcu_llm_load: cannot open ") + path);
    BlobHeader h{};
    const bool hdr_ok = std::fread(&h, sizeof(h), 1, f) == 1 && std::memcmp(h.magic, kBlobMagic, 8) == 0 &&
                        h.version == 1;
    const bool cfg_ok = hdr_ok && h.dtype == (uint32_t)c.dtype && h.layers == c.layers && h.d_model == c.d_model &&
                        h.heads == c.heads && h.kv_heads == c.kv_heads && h.hidden == c.hidden &&
                        h.vocab == c.vocab && h.tied == (c.tied_embeddings ? 1u : 0u);
    if (!cfg_ok) {
        std::fclose(f);
        return fail(hdr_ok ? EVKCU_BAD_SHAPE : EVKCU_BAD_ARG,
                    hdr_ok ? "evkcu_llm_load: blob does not match the model configuration"
                           : "evkcu_llm_load: not a version-1 weight blob");
    }
    cudaStream_t st = as_stream(stream);
    std::vector<uint16_t> host;
    for (const BlobTensor& t : blob_layout(c)) {
        host.resize(t.elems);
        if (std::fread(host.data(), kE, t.elems, f) != t.elems) {
            std::fclose(f);
            return fail(EVKCU_BAD_SHAPE, std::string("evkcu_llm_load: file ends inside ") + t.name);
        }
        // set_weight copies this rank's shard straight from host memory.
        int r = evkcu_llm_set_weight(m, t.name, t.layer, host.data(), stream);
        if (r == EVKCU_OK && cudaStreamSynchronize(st) != cudaSuccess) r = cuda_fail(cudaGetLastError(), "load sync");
        if (r != EVKCU_OK) {
            std::fclose(f);
            return r;
        }
    }
    std::fclose(f);
    return EVKCU_OK;
}

extern "C" int evkcu_llm_save(evkcu_llm* m, const char* path, void* stream) {
    EVKCU_CHECK_ARG(m && path, EVKCU_BAD_ARG, "evkcu_llm_save: null pointer");
    const evkcu_llm_config& c = m->cfg;
    EVKCU_CHECK_ARG(c.tp_size == 1, EVKCU_UNSUPPORTED, "evkcu_llm_save: a tensor-parallel rank holds only shards");
    cudaStream_t st = as_stream(stream);
    EVKCU_CUDA_TRY(cudaStreamSynchronize(st));
    FILE* f = std::fopen(path, "wb");
    EVKCU_CHECK_ARG(f, EVKCU_BAD_ARG, std::string("evkcu_llm_save: cannot create ") + path);
    BlobHeader h{};
    std::memcpy(h.magic, kBlobMagic, 8);
    h.version = 1;
    h.dtype = (uint32_t)c.dtype;
    h.layers = c.layers;
    h.d_model = c.d_model;
    h.heads = c.heads;
    h.kv_heads = c.kv_heads;
    h.hidden = c.hidden;
    h.vocab = c.vocab;
    h.tied = c.tied_embeddings ? 1u : 0u;
    bool ok = std::fwrite(&h, sizeof(h), 1, f) == 1;
    std::vector<uint16_t> host;
    for (const BlobTensor& t : blob_layout(c)) {
        if (!ok) break;
        const void* src = nullptr;
        if (!std::strcmp(t.name, "embedding")) src = m->emb;
        else if (!std::strcmp(t.name, "lm_head")) src = m->lm_head;
        else if (!std::strcmp(t.name, "wqkv")) src = m->layers[t.layer].wqkv;
        else if (!std::strcmp(t.name, "wo")) src = m->layers[t.layer].wo;
        else if (!std::strcmp(t.name, "w1")) src = m->layers[t.layer].w1;
        else src = m->layers[t.layer].w2;
        host.resize(t.elems);
        if (cudaMemcpy(host.data(), src, t.elems * kE, cudaMemcpyDeviceToHost) != cudaSuccess) {
            std::fclose(f);
            return cuda_fail(cudaGetLastError(), "evkcu_llm_save: device read");
        }
        ok = std::fwrite(host.data(), kE, t.elems, f) == t.elems;
    }
    ok = (std::fclose(f) == 0) && ok;
    EVKCU_CHECK_ARG(ok, EVKCU_BAD_ARG, std::string("evkcu_llm_save: write failed: ") + path);
    return EVKCU_OK;
}

extern "C" int evkcu_llm_prefill(evkcu_llm* m, const uint32_t* tokens, uint32_t B, uint32_t S, uint32_t* next_ids,
                                 void* logits_out, void* stream) {
    EVKCU_CHECK_ARG(m && tokens && next_ids, EVKCU_BAD_ARG, "evkcu_llm_prefill: null pointer");
    const evkcu_llm_config& c = m->cfg;
    EVKCU_CHECK_ARG(B >= 1 && B <= c.max_batch && S >= 1 && S < c.max_seq, EVKCU_BAD_SHAPE,
                    "evkcu_llm_prefill: need 1 <= B <= max_batch and 1 <= S < max_seq");
    cudaStream_t st = as_stream(stream);
    const uint32_t D = c.d_model;
    LLM_TRY(evkcu_embed(m->emb, tokens, m->x, c.vocab, D, B * S, 4, c.dtype, st));
    LLM_TRY(run_blocks(m, B, S, false, st));
    // the last position of every sequence
    EVKCU_CUDA_TRY(cudaMemcpy2DAsync(m->xl, (size_t)D * kE, (const char*)m->x + (size_t)(S - 1) * D * kE,
                                     (size_t)S * D * kE, (size_t)D * kE, B, cudaMemcpyDeviceToDevice, st));
    LLM_TRY(head_and_sample(m, m->xl, B, next_ids, logits_out, st));
    set_pos_kernel<<<1, 1, 0, st>>>(m->d_pos, m->d_len, S);
    LLM_TRY(after_launch("llm set_pos"));
    m->cur_len = S;
    m->batch = B;
    return EVKCU_OK;
}

extern "C" int evkcu_llm_decode(evkcu_llm* m, const uint32_t* ids, uint32_t* next_ids, void* logits_out,
                                void* stream) {
    EVKCU_CHECK_ARG(m && ids && next_ids, EVKCU_BAD_ARG, "evkcu_llm_decode: null pointer");
    EVKCU_CHECK_ARG(m->batch > 0, EVKCU_BAD_ARG, "evkcu_llm_decode: call evkcu_llm_prefill first");
    EVKCU_CHECK_ARG(m->cur_len + 1 <= m->cfg.max_seq, EVKCU_BAD_SHAPE, "evkcu_llm_decode: KV cache is full");
    cudaStream_t st = as_stream(stream);
    const uint32_t B = m->batch;
    const bool graphable = st != nullptr && logits_out == nullptr;
    if (!graphable || m->eager_steps[B] < 1) {
        // The first step of a batch size runs eagerly so every lazily
        // allocated scratch buffer exists before a graph is captured.
        m->eager_steps[B] += 1;
        LLM_TRY(decode_body(m, ids, next_ids, logits_out, st));
        m->cur_len += 1;
        return EVKCU_OK;
    }
    // A replayed graph reads and writes fixed buffers: ids / next_ids are
    // staged through m->gin / m->gout.
    auto g = m->graphs.find(B);
    if (g != m->graphs.end() && m->graph_ws[B] != ws_signature()) {
        cudaGraphExecDestroy(g->second);
        m->graphs.erase(g);
        g = m->graphs.end();
    }
    if (g == m->graphs.end()) {
        cudaGraph_t graph;
        EVKCU_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        const int r = decode_body(m, m->gin, m->gout, nullptr, st);
        const cudaError_t ce = cudaStreamEndCapture(st, &graph);
        if (r) return r;
        if (ce != cudaSuccess) return cuda_fail(ce, "cudaStreamEndCapture(llm decode)");
        cudaGraphExec_t exec;
        const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) return cuda_fail(ie, "cudaGraphInstantiate(llm decode)");
        g = m->graphs.emplace(B, exec).first;
        m->graph_ws[B] = ws_signature();
    }
    EVKCU_CUDA_TRY(cudaMemcpyAsync(m->gin, ids, (size_t)B * 4, cudaMemcpyDeviceToDevice, st));
    EVKCU_CUDA_TRY(cudaGraphLaunch(g->second, st));
    EVKCU_CUDA_TRY(cudaMemcpyAsync(next_ids, m->gout, (size_t)B * 4, cudaMemcpyDeviceToDevice, st));
    m->cur_len += 1;
    return EVKCU_OK;
}
