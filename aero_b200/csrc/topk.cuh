// Top-k routing of one token by one warp, shared by the standalone top-k
// kernel and the fused decode kernel. Semantics of src/moe.cpp:26-66: experts
// ranked by descending logit, equal logits by the lower index; with norm the k
// weights are the softmax over the selected logits (max-subtracted, f32 exp,
// summed in selection order), otherwise the full-softmax probability with an f64
// denominator over all E experts.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace aero {

// Order-preserving unsigned image of a logit: larger value -> larger key, -0
// as +0, NaN below every number (key 0; std::partial_sort in the reference
// leaves NaN order unspecified, this is one deterministic choice). key_value
// inverts it (NaN for 0).
__device__ __forceinline__ uint32_t order_key(float v) {
    if (v != v) return 0u;
    uint32_t u = __float_as_uint(v);
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    if (k == 0u) return __uint_as_float(0x7FC00000u);
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// The whole warp calls it for the logits lg[0..E) (E <= 32 * PER, k <= 32):
// lane 0 writes idx_out[0..k), lanes < k write w_out[lane]; *sel_i_out receives,
// in lane r < k, the r-th selected expert.
template <int PER>
__device__ __forceinline__ void topk_warp(const float* lg, int E, int k, int norm, int32_t* idx_out, float* w_out,
                                          int* sel_i_out) {
    const int lane = threadIdx.x & 31;
    float v[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? lg[e] : 0.f;
    }
    // Selection on 64-bit keys: the order-preserving bits of the logit above the
    // complemented index, so the largest key is the larger logit and, on equal
    // logits, the lower index (NaNs rank below every number, lower index first
    // among them). Each lane keeps its best remaining key; a round is one warp
    // max, and only the winning lane rescans its slots.
    uint64_t key[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        key[i] = e < E ? ((uint64_t)order_key(v[i]) << 32) | (0xFFFFFFFFu - (uint32_t)e) : 0ull;
    }
    uint64_t lb = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) lb = key[i] > lb ? key[i] : lb;

    float sel_v = 0.f;  // lane j keeps the j-th selected logit
    int sel_i = 0;      // and its expert
    float mx = 0.f;
    for (int r = 0; r < k; ++r) {
        uint64_t best = lb;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t ot = __shfl_xor_sync(0xffffffffu, best, o);
            best = ot > best ? ot : best;
        }
        const int bi = (int)(0xFFFFFFFFu - (uint32_t)best);
        const float bv = key_value((uint32_t)(best >> 32));
        if ((bi & 31) == lane) {
            const int slot = bi >> 5;
            lb = 0;
#pragma unroll
            for (int i = 0; i < PER; ++i) {
                if (i == slot) key[i] = 0ull;
                lb = key[i] > lb ? key[i] : lb;
            }
        }
        if (lane == 0) idx_out[r] = bi;
        if (r == 0) mx = bv;
        if ((r & 31) == lane) {
            sel_v = bv;
            sel_i = bi;
        }
    }
    if (norm) {
        // softmax over the selected logits; max is the first pick, summed in
        // selection order (src/moe.cpp:47-53)
        float e_mine = 0.f, wsum = 0.f;
        if (lane < k) e_mine = expf(sel_v - mx);
        for (int r = 0; r < k; ++r) wsum += __shfl_sync(0xffffffffu, e_mine, r);
        if (lane < k) w_out[lane] = e_mine / wsum;
    } else {
        double den = 0.0;
#pragma unroll
        for (int i = 0; i < PER; ++i) {
            const int e = lane + 32 * i;
            if (e < E) den += (double)expf(v[i] - mx);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
        if (lane < k) w_out[lane] = (float)((double)expf(sel_v - mx) / den);
    }
    *sel_i_out = sel_i;
}

}  // namespace aero
