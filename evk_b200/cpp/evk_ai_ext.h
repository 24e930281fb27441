// evk_ai_ext.h — additive extensions of the evk::ai operator API for the
// B200 backend.  Nothing here changes a reference signature; each function
// is a new entry point beside its reference counterpart (evk_ai.h:489-615)
// and calls the same C ABI (include/evkcu.h).
//
//   DType            tensors are 2-byte storage; fp16 as in the reference, or
//                    bf16 for the LLM configurations.
//   *_ex             the reference operator plus the parameters it lacks:
//                    grouped-query / causal attention, RoPE per head with a
//                    position offset (decode), RMSNorm with a gain, 32-bit
//                    token ids and counts (vocabularies above 65,535).
//   single_query_attention  host wrapper of the decode-attention shader,
//                    which the reference ships without one
//                    (shaders/single_query_attention.comp:27-71), generalised
//                    to batches, heads and long KV caches.
#pragma once

#include "evk_ai.h"

namespace evk::ai {

enum class DType : int { F16 = 0, BF16 = 1 };

// c = op(a) op(b) (+ c), as matmul (evk_ai.h:495), in the given storage type.
void matmul_ex(Tensor& a, Tensor& b, Tensor& c, bool transpose_a, bool transpose_b, bool acc_c, DType dtype);
void add_ex(Tensor& a, Tensor& b, Tensor& c, DType dtype);
void gelu_ex(Tensor& in, Tensor& out, DType dtype);
void softmax_ex(Tensor& in, Tensor& out, float input_scale, DType dtype);

// Attention O = softmax(Q K^T scale) V with Q, O (B, N, heads * Dh) and K, V
// (B, N, Hkv * Dh), Dh = Q.shape[2] / heads, Hkv = K.shape[2] / Dh (1 is the
// reference's multi-query call; heads is multi-head); causal masks keys
// after the query; scale <= 0 means 1 / sqrt(Dh).
void flash_attention_ex(Tensor& q, Tensor& k, Tensor& v, Tensor& o, uint32_t heads, bool causal, float scale = 0.0f,
                        DType dtype = DType::F16);

// Decode attention for one new query per sequence over a KV cache:
// q, out (B, heads * Dh); kcache, vcache (B, max_len, Hkv * Dh) of which the
// first cur_len positions are used.
void single_query_attention(Tensor& q, Tensor& kcache, Tensor& vcache, Tensor& out, uint32_t heads, uint32_t cur_len,
                            float scale = 0.0f, DType dtype = DType::F16);

// rope (evk_ai.h:587-591) rotating each head_dim slice of the last dimension
// (0 = the whole dimension, as the reference) at positions pos_offset + t.
void rope_ex(Tensor& input, Tensor& out, uint32_t batch_size, uint32_t seq_len, uint32_t embed_dim, float rotary_base,
             uint32_t head_dim, uint32_t pos_offset, DType dtype = DType::F16);

// rms_norm (evk_ai.h:607-610) followed by a per-column gain (gamma: (D), or
// nullptr for none).
void rms_norm_ex(Tensor& input, Tensor& output, float eps, Tensor* gamma, DType dtype = DType::F16);

// embed / greedy_sample with 2- or 4-byte token ids (id_bytes) and 32-bit
// token_base / token_count.  With 4-byte ids, `indices` / `out_tokens` hold
// two 2-byte slots per id.
void embed_ex(Tensor& embeddings, Tensor& indices, Tensor& out, uint32_t id_bytes, DType dtype = DType::F16);
void greedy_sample_ex(Tensor& logits, Tensor& out_tokens, uint32_t position, uint32_t token_base,
                      uint32_t token_count, uint32_t id_bytes, DType dtype = DType::F16);

}  // namespace evk::ai
