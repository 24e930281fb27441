/*
 * evk_oracle.h — CPU restatement of the reference's evk::ai shader math.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * backend (libevkcu) and the CPU baseline timed by bench.py; the product path
 * never links, loads or calls it.
 *
 * Each function restates one shader of carloshgsilva/evk (cited per function
 * in evk_oracle.cpp) on host memory: 2-byte storage (fp16 = dtype 0, bf16 =
 * dtype 1), fp32 arithmetic, one rounding at the shader's storage points.
 * fp16 rounding follows the reference's host quantiser
 * float16_t::float_to_float16 (evk_ai.h:52-121): round-to-nearest-even for
 * normals, round-half-up for subnormals.  Matmul and attention accumulate in
 * fp64 (the reference's fp16 cooperative-matrix accumulation is driver-defined
 * and not reproduced; the target semantics are fp32 accumulation).
 *
 * Pinning: oracle/ref_harness.cpp compiles the reference's own
 * example/tests.h against this library (make -C oracle ref) and its
 * known-answer tests must pass; tests/golden/ holds vectors generated from it.
 */
#ifndef EVK_ORACLE_H
#define EVK_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t oracle_f32_to_f16(float f);
float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_bf16(float f);
float oracle_bf16_to_f32(uint16_t h);
void oracle_quantize(const float* in, uint16_t* out, uint64_t n, int dtype);
void oracle_dequantize(const uint16_t* in, float* out, uint64_t n, int dtype);

void oracle_matmul(const uint16_t* A, const uint16_t* B, uint16_t* C, uint32_t batch, uint32_t M, uint32_t K,
                   uint32_t N, uint64_t stride_a, uint64_t stride_b, uint64_t stride_c, uint32_t flags, int dtype);
void oracle_flash_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* o, uint32_t B,
                            uint32_t N, uint32_t H, uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype);
void oracle_single_query_attention(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, uint16_t* out,
                                   uint32_t B, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t max_len,
                                   uint32_t cur_len, float scale, int dtype);
void oracle_rms_norm(const uint16_t* in, uint16_t* out, const uint16_t* gamma, uint32_t rows, uint32_t D, float eps,
                     int dtype);
void oracle_rope(const uint16_t* in, uint16_t* out, uint32_t batch, uint32_t seq_len, uint32_t dim, uint32_t head_dim,
                 uint32_t pos_offset, float base, int dtype);
void oracle_gelu(const uint16_t* in, uint16_t* out, uint64_t n, int dtype);
void oracle_softmax(const uint16_t* in, uint16_t* out, uint32_t rows, uint32_t L, float scale, int dtype);
void oracle_add(const uint16_t* a, const uint16_t* b, uint16_t* c, uint64_t n, int dtype);
void oracle_scale(uint16_t* x, uint64_t n, float s, int dtype);
void oracle_causal_mask(uint16_t* scores, uint32_t batch, uint32_t N, int dtype);
void oracle_embed(const uint16_t* E, const void* idx, uint16_t* out, uint32_t vocab, uint32_t dim, uint32_t n_idx,
                  uint32_t idx_bytes);
void oracle_greedy_sample(const uint16_t* logits, void* out, uint32_t B, uint32_t S, uint32_t V, uint32_t position,
                          uint32_t token_base, uint32_t token_count, uint32_t out_bytes, int dtype);

/* training side (shaders cited in evk_oracle.cpp) */
void oracle_relu(const uint16_t* in, uint16_t* out, uint64_t n, int dtype);
void oracle_relu_backward(const uint16_t* go, const uint16_t* in, uint16_t* gi, uint64_t n, int dtype);
void oracle_gelu_backward(const uint16_t* go, const uint16_t* in, uint16_t* gi, uint64_t n, int dtype);
void oracle_softmax_backward(const uint16_t* p, const uint16_t* g, uint16_t* gi, uint32_t rows, uint32_t L,
                             float scale, int dtype);
void oracle_rms_norm_backward(const uint16_t* x, const uint16_t* g, uint16_t* gi, uint32_t rows, uint32_t D,
                              float eps, int dtype);
void oracle_rope_backward(const uint16_t* go, uint16_t* gi, uint32_t batch, uint32_t seq_len, uint32_t dim,
                          float base, int dtype);
void oracle_embed_backward(const uint16_t* go, const void* idx, uint16_t* gE, uint32_t vocab, uint32_t dim,
                           uint32_t n_idx, uint32_t idx_bytes, int dtype);
void oracle_position_add(const uint16_t* in, const uint16_t* pos, uint16_t* out, uint32_t batch, uint32_t seq_len,
                         uint32_t dim, int dtype);
void oracle_position_add_backward(const uint16_t* go, uint16_t* gi, uint16_t* gp, uint32_t batch, uint32_t seq_len,
                                  uint32_t dim, int dtype);
void oracle_sum_batch(const uint16_t* in, uint16_t* out, uint32_t batch, uint64_t size, int dtype);
void oracle_sgd(uint16_t* p, const uint16_t* g, uint64_t n, float lr, int dtype);
void oracle_adam(uint16_t* p, const uint16_t* g, uint16_t* m, uint16_t* v, uint64_t n, uint32_t step, float lr,
                 float beta1, float beta2, float eps, int dtype);
void oracle_mse_loss(const uint16_t* pred, const uint16_t* tgt, uint16_t* grad, uint16_t* result, uint64_t n,
                     int dtype);
void oracle_cross_entropy_loss(const uint16_t* logits, const void* tgt, uint16_t* grad, uint16_t* result,
                               uint32_t rows, uint32_t V, uint32_t target_bytes, int dtype);
void oracle_flash_attention_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* dO,
                                uint16_t* dQ, uint16_t* dK, uint16_t* dV, uint32_t B, uint32_t N, uint32_t H,
                                uint32_t Hkv, uint32_t Dh, float scale, uint32_t flags, int dtype);

/* Seeded generator shared by tests, bench and fixtures (portable, unlike the
 * reference's libc rand()): splitmix64 stream -> Box-Muller normals. */
void oracle_fill_normal(uint16_t* out, uint64_t n, uint64_t seed, float mean, float stddev, int dtype);
void oracle_fill_uniform_ids(void* out, uint64_t n, uint64_t seed, uint32_t lo, uint32_t hi, uint32_t id_bytes);

int oracle_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
