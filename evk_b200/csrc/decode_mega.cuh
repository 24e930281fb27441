// decode_mega.cuh — host interface of the persistent decode step
// (decode_mega.cu), used by the LLM driver (llm.cu).
#pragma once

#include "common.cuh"

namespace evkcu {

// One layer's weights and KV cache, as the kernel reads them (device array).
struct MegaLayer {
    const void *wqkv, *wo, *w1, *w2;
    void *kc, *vc;
};

struct MegaHost {
    uint32_t B, D, H, Hkv, Dh, F, V, layers, max_seq, tied;
    float eps, rope_base;
    const void* emb;
    const void* lm_head;
    const void* layer_table;  // device array of MegaLayer [layers]
    void *x, *q, *attn, *h1, *logits;  // logits optional ([B, V])
    const float2* rope_cs;
    uint32_t *d_pos, *d_len;
    const uint32_t* ids_in;
    uint32_t* ids_out;
    void* scratch;  // decode_mega_scratch_bytes, zero-filled once at allocation
};

// Whether the persistent step handles this shape (tensor parallelism off).
bool decode_mega_supported(uint32_t B, uint32_t D, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t F, uint32_t V,
                           bool tied);
size_t decode_mega_scratch_bytes(uint32_t B, uint32_t D, uint32_t H, uint32_t Hkv, uint32_t Dh, uint32_t F,
                                 uint32_t max_seq, int grid);
// One decode step (embed ... greedy ids, position advanced) as one
// cooperative launch on `st`.
int decode_mega_step(const MegaHost& h, int dtype, cudaStream_t st);

}  // namespace evkcu
