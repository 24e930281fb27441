/*
 * evkcu.h — C ABI of the B200 (sm_100a) backend for the evk::ai operator set.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream (`void*`, NULL = legacy default stream), enqueues its kernels on that
 * stream and returns immediately with an evkcu_status.  Nothing here
 * allocates or frees caller memory.  Tensors use the reference's layout:
 * row-major, last dimension contiguous, 2-byte elements (fp16, or bf16 as an
 * extension).  Token ids are raw unsigned integers stored in the element slots
 * (uint16 as in the reference, or uint32 as an extension for vocabularies
 * above 65535).
 *
 * Each function cites the reference interface it replaces (carloshgsilva/evk,
 * path:line).  In the reference an op records bind+push+dispatch+barrier into
 * a global Vulkan command buffer; here stream order replaces the barrier.
 *
 * Errors never exit the process: a failing call returns a non-zero status and
 * evkcu_last_error() returns a message for the calling thread.
 */
#ifndef EVKCU_H
#define EVKCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum evkcu_status {
    EVKCU_OK = 0,
    EVKCU_BAD_SHAPE = 1,   /* shape / size precondition violated               */
    EVKCU_BAD_ALIGN = 2,   /* pointer or row pitch not aligned as required      */
    EVKCU_CUDA_ERROR = 3,  /* a CUDA runtime / driver call failed               */
    EVKCU_COMM_ERROR = 4,  /* a collective failed (tensor-parallel helpers)      */
    EVKCU_TIMEOUT = 5,     /* a bounded device-side wait gave up                 */
    EVKCU_UNSUPPORTED = 6, /* valid request this build does not implement        */
    EVKCU_BAD_ARG = 7      /* null pointer / invalid enum                        */
} evkcu_status;

typedef enum evkcu_dtype {
    EVKCU_F16 = 0,  /* the reference's only storage type (evk_ai.h:252-260) */
    EVKCU_BF16 = 1  /* extension for the bf16 LLM configurations            */
} evkcu_dtype;

/* matmul flags, evk_ai.h:495 (transpose_a, transpose_b, acc_c) */
#define EVKCU_MM_TRANSPOSE_A 1u
#define EVKCU_MM_TRANSPOSE_B 2u
#define EVKCU_MM_ACC_C 4u

/* flash attention flags (extension: the reference is non-causal only) */
#define EVKCU_ATTN_CAUSAL 1u
/* flash_attention_bwd only: use the exact softmax gradient term
 * sum_j p_ij dp_ij (= t_i / l_i) instead of the reference shader's t_i.     */
#define EVKCU_ATTN_BWD_NORMALIZED 2u

/* ---- context -------------------------------------------------------------
 * Replaces evk::ai::initialize / shutdown (evk_ai.h:489-490, evk_ai.cpp:211-252):
 * selects the device and creates the per-device state (SM count, device error
 * word, small workspace).  Every op calls it lazily for the current device.   */
int evkcu_init(int device);
int evkcu_shutdown(void);
const char* evkcu_last_error(void);
const char* evkcu_version(void);
/* Reads and clears the device error word written by bounded device-side waits
 * (EVKCU_TIMEOUT when a kernel gave up waiting).  Synchronises the device.   */
int evkcu_check_device_error(void);
/* Number of kernels this library launched on the calling thread since the
 * last reset (evidence for the benchmark's gpu_launches field).              */
uint64_t evkcu_launch_count(void);
void evkcu_reset_launch_count(void);

/* ---- matmul ----------------------------------------------------------------
 * evk::ai::matmul  evk_ai.h:495, evk_ai.cpp:254-330, shaders/matmul.comp:44-140
 * C[b] = op(A[b]) . op(B[b])  (+ C[b] when EVKCU_MM_ACC_C)
 *   op(A) is M x K: A is stored [M,K] row-major, or [K,M] with TRANSPOSE_A.
 *   op(B) is K x N: B is stored [K,N] row-major, or [N,K] with TRANSPOSE_B.
 *   C is [M,N] row-major.  stride_a/b/c are per-batch element strides; 0 means
 *   the operand is broadcast over the batch (evk_ai.cpp:299-304).
 * fp32 accumulation on tcgen05 tensor cores, one rounding to the storage type.
 * Requires the contiguous dimension of each operand to be a multiple of 8
 * elements and 16-byte aligned base pointers.  Unlike the reference, M, N and K
 * need not be tile multiples: tails are computed, not left unwritten.        */
int evkcu_matmul(const void* A, const void* B, void* C,
                 uint32_t batch, uint32_t M, uint32_t K, uint32_t N,
                 uint64_t stride_a, uint64_t stride_b, uint64_t stride_c,
                 uint32_t flags, int dtype, void* stream);

/* ---- flash attention -------------------------------------------------------
 * evk::ai::flash_attention  evk_ai.h:497-501, evk_ai.cpp:332-369,
 * shaders/flash_attention.comp:53-185.
 * O = softmax(Q_h K_g^T * scale) V_g per batch b, query head h, with KV head
 * g = h / (H / Hkv).  Q, O: [B, N, H*Dh];  K, V: [B, N, Hkv*Dh].
 * The reference call is Hkv = 1 (multi-query), non-causal, scale = 1/sqrt(Dh);
 * Hkv = H (per-head K/V) and EVKCU_ATTN_CAUSAL are extensions.
 * Rows whose softmax denominator is 0 produce 0 (flash_attention.comp:166).
 * Dh must be a multiple of 16 and at most 256.                              */
int evkcu_flash_attention(const void* q, const void* k, const void* v, void* o,
                          uint32_t B, uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh,
                          float scale, uint32_t flags, int dtype, void* stream);

/* ---- single-query (decode) attention --------------------------------------
 * shaders/single_query_attention.comp:27-71 (the reference ships the shader
 * without a host wrapper; this is that wrapper, generalised to B sequences,
 * H query heads over Hkv cached heads, and any cache length).
 * q, out: [B, H*Dh];  kcache, vcache: [B, max_len, Hkv*Dh];  attends over the
 * first cur_len positions of each sequence.  scale <= 0 selects 1/sqrt(Dh)
 * (the shader's inversesqrt(dim)).                                           */
int evkcu_single_query_attention(const void* q, const void* kcache, const void* vcache, void* out,
                                 uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh,
                                 uint32_t max_len, uint32_t cur_len, float scale,
                                 int dtype, void* stream);

/* ---- row / elementwise ops ------------------------------------------------ */

/* evk::ai::rms_norm  evk_ai.h:607-610, evk_ai.cpp:1045-1067, shaders/rms_norm.comp:21-48
 * y = clamp(x, +-65504) * rsqrt(mean(clamp(x)^2) + eps) per row of D.
 * gamma (optional, [D], extension) multiplies the result when non-NULL.      */
int evkcu_rms_norm(const void* in, void* out, const void* gamma,
                   uint32_t rows, uint32_t D, float eps, int dtype, void* stream);

/* evk::ai::rope  evk_ai.h:587-591, evk_ai.cpp:945-966, shaders/rope.comp:18-40
 * Interleaved pairs (x[2i], x[2i+1]) rotated by angle t*base^(-2i/rot_dim).
 * in/out: [batch, seq_len, dim].  The reference is head_dim = dim and
 * pos_offset = 0; head_dim < dim rotates each head_dim slice independently and
 * pos_offset shifts t (decode), both extensions.                             */
int evkcu_rope(const void* in, void* out, uint32_t batch, uint32_t seq_len, uint32_t dim,
               uint32_t head_dim, uint32_t pos_offset, float base, int dtype, void* stream);

/* evk::ai::gelu  evk_ai.h:538-540, evk_ai.cpp:679-699, shaders/gelu.comp:15-29 (tanh form) */
int evkcu_gelu(const void* in, void* out, uint64_t n, int dtype, void* stream);

/* evk::ai::softmax  evk_ai.h:523-525, evk_ai.cpp:593-613, shaders/softmax.comp:23-66
 * Row softmax of raw*scale over L; raw <= -65504 is masked (output 0).       */
int evkcu_softmax(const void* in, void* out, uint32_t rows, uint32_t L, float scale,
                  int dtype, void* stream);

/* evk::ai::add  evk_ai.h:520-521, evk_ai.cpp:568-591, shaders/add.comp:18-26 */
int evkcu_add(const void* a, const void* b, void* c, uint64_t n, int dtype, void* stream);

/* evk::ai::scale  evk_ai.cpp:992-1007, shaders/scale.comp (in place)        */
int evkcu_scale(void* x, uint64_t n, float s, int dtype, void* stream);

/* evk::ai::zero  evk_ai.cpp:1010-1024, shaders/zero.comp                    */
int evkcu_zero(void* x, uint64_t n, int dtype, void* stream);

/* evk::ai::apply_causal_mask  evk_ai.h:574-577, evk_ai.cpp:862-882,
 * shaders/causal_mask.comp:16-33: scores[b,i,j] = -65504 for j > i.          */
int evkcu_causal_mask(void* scores, uint32_t batch, uint32_t N, int dtype, void* stream);

/* evk::ai::embed  evk_ai.h:554-558, evk_ai.cpp:782-806, shaders/embed.comp:18-28
 * out[i,:] = E[idx[i],:].  idx_bytes = 2 (reference uint16) or 4 (extension).
 * Indices >= vocab are clamped to vocab-1 instead of reading out of bounds.  */
int evkcu_embed(const void* E, const void* idx, void* out, uint32_t vocab, uint32_t dim,
                uint32_t n_idx, uint32_t idx_bytes, int dtype, void* stream);

/* evk::ai::greedy_sample  evk_ai.h:560-566, evk_ai.cpp:808-837,
 * shaders/greedy_sample.comp:24-64.
 * out[b] = argmax_j logits[b, position, token_base + j], j < token_count, with
 * the reference's exact tie rule (256-lane strided scan keeping the first
 * strict maximum, then a strict-greater tree: ties go to the lower lane).
 * out_bytes = 2 (uint16, reference) or 4 (uint32 extension).                 */
int evkcu_greedy_sample(const void* logits, void* out, uint32_t B, uint32_t S, uint32_t V,
                        uint32_t position, uint32_t token_base, uint32_t token_count,
                        uint32_t out_bytes, int dtype, void* stream);

/* No counterpart in the reference.  Same arguments, result and tie rule as
 * evkcu_greedy_sample, for callers that cannot allocate GPU memory when they
 * call it: code that runs while a CUDA stream is being captured (cudaMalloc
 * is not allowed there), serving loops that reserve all HBM up front for
 * weights and KV cache, and host programs that forbid allocation on their hot
 * path.  This entry point never allocates or frees memory: its scratch is one
 * fixed 128 KiB device array inside the library, which every GPU that loads
 * the library keeps until the process exits.
 *   - Limit: B <= 1024 and B * ceil(token_count / 4096) <= 15872; larger
 *     requests return EVKCU_BAD_SHAPE (use evkcu_greedy_sample for those).
 *   - The first call on a device looks up the array's device address with
 *     that device current; make that first call before any stream capture.
 *   - All calls on a device share that device's array, which keeps the last
 *     call's contents: calls that overlap on the GPU (for example on two
 *     streams of one device) race and must be ordered by the caller.        */
int evkcu_greedy_sample_noalloc(const void* logits, void* out, uint32_t B, uint32_t S, uint32_t V,
                                uint32_t position, uint32_t token_base, uint32_t token_count,
                                uint32_t out_bytes, int dtype, void* stream);


/* Decode attention whose cache length is read from device memory (*d_cur_len)
 * when the kernel runs, so one captured CUDA graph can replay every decode
 * step of a growing cache.  Otherwise as evkcu_single_query_attention; the
 * grid is sized for max_len.  Extension (no reference counterpart).         */
int evkcu_single_query_attention_devlen(const void* q, const void* kcache, const void* vcache, void* out,
                                        uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh,
                                        uint32_t max_len, const uint32_t* d_cur_len, float scale,
                                        int dtype, void* stream);

/* Fused RMSNorm + RoPE (extension: the two bandwidth ops of evk_ai.h:607-610
 * and 587-591 in one pass).  rows = batch * seq_len rows of `dim`:
 * out = rope(rms_norm(in, eps) [* gamma]) with RoPE over each head_dim slice
 * (0 = the whole row, as the reference) at positions row % seq_len +
 * pos_offset; no rounding between the two.  dim, head_dim multiples of 8;
 * 16-byte-aligned buffers.                                                  */
int evkcu_rms_norm_rope(const void* in, void* out, const void* gamma, uint32_t rows, uint32_t seq_len, uint32_t dim,
                        uint32_t head_dim, uint32_t pos_offset, float eps, float base, int dtype, void* stream);

/* ---- training side ---------------------------------------------------------
 * The reference's training operators (evk_ai.h:474-615).  Backward passes
 * accumulate into their gradient tensor (grad_in += ...) as the shaders do;
 * losses and flash_attention_bwd overwrite their outputs.                    */

/* evk::ai::relu / relu_backward, evk_ai.cpp:635-677, shaders/relu.comp,
 * relu_bwd.comp: out = max(0, in); grad_in += in > 0 ? grad_out : 0.        */
int evkcu_relu(const void* in, void* out, uint64_t n, int dtype, void* stream);
int evkcu_relu_backward(const void* grad_out, const void* in, void* grad_in, uint64_t n, int dtype, void* stream);

/* evk::ai::gelu_backward, evk_ai.cpp:702-720, shaders/gelu_bwd.comp:
 * grad_in += grad_out * d gelu(in) / d in (tanh form).                      */
int evkcu_gelu_backward(const void* grad_out, const void* in, void* grad_in, uint64_t n, int dtype, void* stream);

/* evk::ai::softmax_backward, evk_ai.cpp:614-633, shaders/softmax_bwd.comp:
 * per row grad_in += probs * (grad_out - dot(grad_out, probs)) * scale.    */
int evkcu_softmax_backward(const void* probs, const void* grad_out, void* grad_in, uint32_t rows, uint32_t L,
                           float scale, int dtype, void* stream);

/* evk::ai::rms_norm_backward, evk_ai.cpp:1068-1092, shaders/rms_norm_bwd.comp:
 * grad_in += (g - y dot(g, y) / D) / rms over rows of D.                    */
int evkcu_rms_norm_backward(const void* in, const void* grad_out, void* grad_in, uint32_t rows, uint32_t D,
                            float eps, int dtype, void* stream);

/* evk::ai::rope_backward, evk_ai.cpp:969-990, shaders/rope_bwd.comp: the
 * inverse rotation of rope over the whole last dimension, accumulated.      */
int evkcu_rope_backward(const void* grad_out, void* grad_in, uint32_t batch, uint32_t seq_len, uint32_t dim,
                        float base, int dtype, void* stream);

/* evk::ai::embed_backward, evk_ai.cpp:839-859, shaders/embed_bwd.comp:
 * grad_E[idx[i], :] += grad_out[i, :], indices in order, rounded per add.
 * idx_bytes: 2 (reference) or 4 (extension).                                */
int evkcu_embed_backward(const void* grad_out, const void* idx, void* grad_E, uint32_t vocab, uint32_t dim,
                         uint32_t n_idx, uint32_t idx_bytes, int dtype, void* stream);

/* evk::ai::position_add / position_add_backward, evk_ai.cpp:883-944,
 * shaders/position_add.comp, position_add_bwd.comp: out = in + pos
 * (broadcast over batch); grad_in += grad_out, grad_pos += sum_b grad_out.  */
int evkcu_position_add(const void* in, const void* pos, void* out, uint32_t batch, uint32_t seq_len, uint32_t dim,
                       int dtype, void* stream);
int evkcu_position_add_backward(const void* grad_out, void* grad_in, void* grad_pos, uint32_t batch,
                                uint32_t seq_len, uint32_t dim, int dtype, void* stream);

/* evk::ai::sum_batch, evk_ai.cpp:1024-1043, shaders/sum_batch.comp:
 * out[i] += sum_b in[b * size + i].                                          */
int evkcu_sum_batch(const void* in, void* out, uint32_t batch, uint64_t size, int dtype, void* stream);

/* evk::ai::sgd, evk_ai.cpp:505-523, shaders/sgd.comp: param -= lr * grad.   */
int evkcu_sgd(void* param, const void* grad, uint64_t n, float lr, int dtype, void* stream);

/* evk::ai::adam, evk_ai.cpp:525-566, shaders/adam.comp.  m and v are the
 * AdamState buffers (2-byte storage: m normalised by rms, v as biased log2
 * rms; zero-initialised); step is the state's timestep after increment
 * (1 on the first call).                                                    */
int evkcu_adam(void* param, const void* grad, void* m, void* v, uint64_t n, uint32_t step, float lr, float beta1,
               float beta2, float eps, int dtype, void* stream);

/* evk::ai::mse_loss, evk_ai.cpp:481-503, shaders/mse_loss.comp:
 * grad = 2 (pred - target) / n, result[0] = mean((pred - target)^2).        */
int evkcu_mse_loss(const void* pred, const void* target, void* grad, void* result, uint64_t n, int dtype,
                   void* stream);

/* evk::ai::cross_entropy_loss, evk_ai.cpp:722-780, shaders/cross_entropy*.comp:
 * logits [rows, V], targets [rows] (target 0 = ignore); grad = (softmax -
 * onehot) / valid_count on valid rows, 0 elsewhere; result[0] = mean loss
 * over valid rows.  target_bytes: 2 (reference) or 4 (extension).           */
int evkcu_cross_entropy_loss(const void* logits, const void* targets, void* grad, void* result, uint32_t rows,
                             uint32_t V, uint32_t target_bytes, int dtype, void* stream);

/* evk::ai::flash_attention_bwd, evk_ai.cpp:371-473,
 * shaders/flash_attention_bwd.comp: gradients of O = softmax(Q K^T scale) V
 * for Q, dO, dQ [B, N, H*Dh] and K, V, dK, dV [B, N, Hkv*Dh] (the reference
 * is Hkv = 1, non-causal; flags may add EVKCU_ATTN_CAUSAL and
 * EVKCU_ATTN_BWD_NORMALIZED).  scale <= 0 means 1/sqrt(Dh).  O is accepted
 * for the reference's signature but not read (the forward is recomputed).  */
int evkcu_flash_attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dO, void* dQ,
                              void* dK, void* dV, uint32_t B, uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh,
                              float scale, uint32_t flags, int dtype, void* stream);

/* ---- LLM driver (extension) ------------------------------------------------
 * The decoder that example/main_llm.cpp builds from these operators
 * (CausalAttentionBlock::forward :528-546, MeshTokenModel::build_graph
 * :588-606, sample_autoregressive :622-654), as one device-resident object:
 * pre-RMSNorm (no gain, as evk::ai::rms_norm), multi-head attention with
 * per-head interleaved RoPE, GELU MLP, residual adds, final RMSNorm, LM head
 * (tied to the embedding or separate), greedy sampling.  Unlike the
 * reference's full-sequence recompute per token, decode keeps a KV cache and
 * runs one CUDA graph per step with no host round trip.
 * Tensor parallel (tp_size > 1, one process per GPU): attention heads and MLP
 * columns are split across ranks, Wo / W2 outputs are summed with an NCCL
 * all-reduce, the vocabulary is split for the LM head and greedy sampling
 * combines the ranks' 64-bit selection keys with an all-gather.            */
typedef struct evkcu_llm_config {
    uint32_t layers, d_model, heads, kv_heads, hidden, vocab;
    uint32_t max_batch, max_seq;
    float rope_base, eps;
    int dtype;                /* EVKCU_F16 or EVKCU_BF16 */
    uint32_t tied_embeddings; /* 1: logits = x . embedding^T */
    uint32_t tp_rank, tp_size;
} evkcu_llm_config;

typedef struct evkcu_llm evkcu_llm;

/* NCCL communicator set-up for tensor parallelism: rank 0 creates the id, the
 * caller distributes its 128 bytes, every rank calls evkcu_comm_init.       */
int evkcu_comm_unique_id(void* id128);
int evkcu_comm_init(const void* id128, int rank, int world, void** comm);
int evkcu_comm_destroy(void* comm);

/* Allocates weights, KV cache and activations on the current device.  comm is
 * an evkcu_comm_init communicator when tp_size > 1, else NULL.              */
int evkcu_llm_create(const evkcu_llm_config* cfg, void* comm, evkcu_llm** out);
int evkcu_llm_destroy(evkcu_llm* m);
/* Seeded N(0, std) weights generated on the device from each element's global
 * index, so every tensor-parallel size builds the same model.              */
int evkcu_llm_init_random(evkcu_llm* m, uint64_t seed, float std, void* stream);
/* Copies one full (unsharded) weight from device memory; this rank keeps its
 * shard.  name: "embedding" [V, D], "lm_head" [D, V], and per layer "wqkv"
 * [D, (H + 2 Hkv) Dh] (columns: q heads, k heads, v heads), "wo" [H Dh, D],
 * "w1" [D, F], "w2" [F, D].                                                  */
int evkcu_llm_set_weight(evkcu_llm* m, const char* name, uint32_t layer, const void* src, void* stream);
/* Weight blob (extension; the reference keeps only an in-memory parameter
 * snapshot, example/main_llm.cpp:306-354): one file with every weight of the
 * model in its storage type, unsharded.  Layout: a 64-byte header (magic
 * "EVKWBLOB", uint32 version = 1, dtype, layers, d_model, heads, kv_heads,
 * hidden, vocab, tied_embeddings, zero padding), then row-major tensors in
 * the order embedding, lm_head (untied only), and per layer wqkv, wo, w1,
 * w2, each in the layout of evkcu_llm_set_weight.  load checks the header
 * against the model's configuration and keeps this rank's shards; save
 * needs tp_size == 1.  Both synchronise the stream.                        */
int evkcu_llm_load(evkcu_llm* m, const char* path, void* stream);
int evkcu_llm_save(evkcu_llm* m, const char* path, void* stream);
/* Prefill: tokens [B, S] (uint32, device) -> KV cache positions 0..S-1 and
 * the next token per sequence (next_ids [B], uint32, device).  Resets the
 * cache.  Optionally logits_out [B, vocab] (device, storage dtype) receives
 * the last position's logits (gathered across ranks).                      */
int evkcu_llm_prefill(evkcu_llm* m, const uint32_t* tokens, uint32_t B, uint32_t S, uint32_t* next_ids,
                      void* logits_out, void* stream);
/* One decode step for the B sequences of the last prefill: consumes ids [B]
 * (the tokens at the current position) and writes next_ids [B].  From the
 * second step of a batch size on, replays a captured CUDA graph (needs a
 * non-default stream and logits_out == NULL; otherwise runs eagerly).      */
int evkcu_llm_decode(evkcu_llm* m, const uint32_t* ids, uint32_t* next_ids, void* logits_out, void* stream);
/* Number of cached positions (prefill length + decode steps).  Host value. */
uint32_t evkcu_llm_length(const evkcu_llm* m);
/* 1 when the decode Wo / W2 all-reduce of this tensor-parallel model can run
 * fused over peer memory (every rank mapped its peers and none set
 * EVKCU_DISABLE_FUSED_ALLREDUCE; the ranks agree at creation), 0 when it
 * uses NCCL.  Even when 1, calls of more than 32,768 elements (batch rows x
 * d_model) use NCCL, except at tp = 2 up to 131,072, where the fused path
 * sends 16-bit partials.  Host value.                                        */
uint32_t evkcu_llm_fused_allreduce(const evkcu_llm* m);

#ifdef __cplusplus
}
#endif
#endif /* EVKCU_H */
