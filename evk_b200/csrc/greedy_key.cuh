// greedy_key.cuh — the 64-bit selection key of greedy_sample.
//
// The reference's argmax (shaders/greedy_sample.comp:24-64) scans with 256
// lanes (j = lane, lane + 256, ...; first strict maximum per lane) and merges
// lanes in a strict-greater shared-memory tree at strides 128..1.  Unrolled,
// its winner among lanes holding the global maximum is the lane with the
// smallest bit-reversed index, and within a lane the smallest j.  The key
//     hi32 = order-preserving bits of the value (0 for NaN and -inf, which the
//            reference never selects since `v > -FLT_MAX` is false; -0.0
//            keys as +0.0, since `>` treats the two zeros as equal)
//     lo32 = ~(bitrev8(j & 255) << 24 | (j >> 8))
// makes that winner the maximum key, so any reduction order (split CTAs,
// tensor-parallel vocabulary shards) selects the reference's token.
#pragma once
#include <float.h>
#include <stdint.h>

namespace evkcu {

__device__ __forceinline__ uint64_t elem_key(float v, uint32_t j) {
    if (!(v > -FLT_MAX)) return 0ull;  // NaN, -inf: never selected
    if (v == 0.0f) v = 0.0f;           // -0.0 ties with +0.0
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    uint32_t rank = (__brev(j & 255u) >> 24) << 24 | (j >> 8);
    return ((uint64_t)u << 32) | (uint64_t)(0xFFFFFFFFu - rank);
}

__device__ __forceinline__ uint32_t key_to_offset(uint64_t key) {
    uint32_t rank = 0xFFFFFFFFu - (uint32_t)key;
    uint32_t lane = __brev(rank >> 24) >> 24;
    return (rank & 0xFFFFFFu) * 256u + lane;
}

}  // namespace evkcu
