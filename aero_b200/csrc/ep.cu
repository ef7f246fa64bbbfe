// Expert-parallel exchange kernels: what one rank runs before and after the
// all-to-all that moves token rows to the ranks owning their experts.
//
// Rank r owns experts [begin[r], begin[r+1]). A token goes to a remote rank
// once, however many of its k experts that rank owns (the per-destination
// de-duplication of the exchange), carrying a metadata row of
//   [k expert ids (global id, or -1 where the slot's expert is elsewhere),
//    k weights (f32 bits), shared-expert gate (f32 bits), 0]
// so the receiver computes sum_s w_s * expert_s(x) over its own slots and sends
// back one row per received token. The reference is single-process
// (src/moe.cpp:122-161 loops over all experts of a token in one place); the
// exchange is this library's addition and keeps its sum per token: the local
// rank's partial (with the shared expert) first, then the remote partials in
// rank order, so results do not depend on message timing.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cub/block/block_scan.cuh>

#include "internal.h"

namespace aero {
namespace {

constexpr int kPlanThreads = 1024;

__device__ __forceinline__ bool slot_in(const int32_t* idx_t, int k, int lo, int hi) {
    for (int s = 0; s < k; ++s) {
        const int e = idx_t[s];
        if (e >= lo && e < hi) return true;
    }
    return false;
}

// One CTA. For each remote rank in rank order, the tokens with at least one
// slot in that rank's range, in token order: send_tok / send_rank for the S
// sent rows in that compact order, counts[r] rows per rank (0 for this rank),
// counts[n] = S, and pos[t*n + r] = the row of token t in rank r's slab of the
// send buffer, r * slab + (its index among r's rows) (-1: not sent; for r = me
// the token's own row t).
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int32_t* __restrict__ idx, int T, int k,
                                                               EpRankTable rt, int me, int slab,
                                                               int32_t* __restrict__ send_tok,
                                                               int32_t* __restrict__ send_rank,
                                                               int32_t* __restrict__ counts,
                                                               int32_t* __restrict__ pos) {
    using Scan = cub::BlockScan<int, kPlanThreads>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ int carry;
    const int n = rt.n;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int r = 0; r < n; ++r) {
        const int lo = rt.begin[r], hi = rt.begin[r + 1];
        const int start = carry;
        for (int t0 = 0; t0 < T; t0 += kPlanThreads) {
            const int t = t0 + threadIdx.x;
            const bool hit = r != me && t < T && slot_in(idx + (int64_t)t * k, k, lo, hi);
            int ex, tot;
            Scan(tmp).ExclusiveSum(hit ? 1 : 0, ex, tot);
            const int base = carry;
            if (t < T) {
                if (r == me) {
                    pos[(int64_t)t * n + r] = t;
                } else if (hit) {
                    send_tok[base + ex] = t;
                    send_rank[base + ex] = r;
                    pos[(int64_t)t * n + r] = r * slab + (base + ex - start);
                } else {
                    pos[(int64_t)t * n + r] = -1;
                }
            }
            __syncthreads();
            if (threadIdx.x == 0) carry = base + tot;
            __syncthreads();
        }
        if (threadIdx.x == 0) counts[r] = carry - start;
        __syncthreads();
    }
    if (threadIdx.x == 0) counts[n] = carry;
}

__device__ __forceinline__ uint32_t pack_h2f(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Rows [0, T) are this rank's tokens (self rows); rows [T, T + n * slab) the send
// slabs, slab r carrying counts[r] rows for rank r and padding after them whose
// metadata names no expert. Each thread moves 8 values of a real row; the
// thread of a row's first chunk also writes the row's metadata.
template <typename RT>
__global__ void ep_pack_kernel(const float* __restrict__ x, int T, int dp, int k, const int32_t* __restrict__ idx,
                               const float* __restrict__ w, const float* __restrict__ sgate, int has_shared,
                               EpRankTable rt, int me, int slab, const int32_t* __restrict__ send_tok,
                               const int32_t* __restrict__ counts, RT* __restrict__ self_rows,
                               int32_t* __restrict__ self_meta, RT* __restrict__ send_rows,
                               int32_t* __restrict__ send_meta, int meta_ld) {
    const int per_row = dp / 8;
    const int n = rt.n;
    const int64_t total = (int64_t)(T + n * slab) * per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / per_row), c = (int)(i % per_row) * 8;
        const bool self = row < T;
        int t = row, dst = me;
        int64_t orow = row;
        if (!self) {
            orow = row - T;
            dst = (int)(orow / slab);
            const int kk = (int)(orow % slab);
            if (kk >= counts[dst]) {
                // padding: no expert for this row at the receiver
                if (c == 0) {
                    int32_t* m = send_meta + orow * meta_ld;
                    for (int s = 0; s < k; ++s) m[s] = -1;
                    for (int j = k; j < meta_ld; ++j) m[j] = 0;
                }
                continue;
            }
            int pre = 0;
            for (int r = 0; r < dst; ++r) pre += counts[r];
            t = send_tok[pre + kk];
        }
        RT* rows = self ? self_rows : send_rows;
        const float* src = x + (int64_t)t * dp + c;
        const float4 a = ld_f4(src), b = ld_f4(src + 4);
        if constexpr (sizeof(RT) == 2) {
            *reinterpret_cast<uint4*>(rows + orow * dp + c) =
                make_uint4(pack_h2f(a.x, a.y), pack_h2f(a.z, a.w), pack_h2f(b.x, b.y), pack_h2f(b.z, b.w));
        } else {
            float* o = reinterpret_cast<float*>(rows) + orow * dp + c;
            *reinterpret_cast<float4*>(o) = a;
            *reinterpret_cast<float4*>(o + 4) = b;
        }
        if (c == 0) {
            int32_t* m = (self ? self_meta : send_meta) + orow * meta_ld;
            const int lo = rt.begin[dst], hi = rt.begin[dst + 1];
            for (int s = 0; s < k; ++s) {
                const int e = idx[(int64_t)t * k + s];
                m[s] = (e >= lo && e < hi) ? e : -1;
                m[k + s] = __float_as_int(w[(int64_t)t * k + s]);
            }
            m[2 * k] = __float_as_int(self && has_shared ? sgate[t] : 0.f);
            for (int j = 2 * k + 1; j < meta_ld; ++j) m[j] = 0;
        }
    }
}

// Receiver: metadata rows -> pair buckets (sentinel E for slots held
// elsewhere), weights and shared gates. Ids that are neither -1 nor owned here
// are treated as held elsewhere and counted in *bad.
__global__ void ep_prep_kernel(const int32_t* __restrict__ meta, int meta_ld, int R, int k, int Tsh, int e_begin,
                               int e_end, int E, int32_t* __restrict__ idx, float* __restrict__ w,
                               float* __restrict__ sgate, int32_t* __restrict__ bad) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)R * k) return;
    const int r = (int)(i / k), s = (int)(i % k);
    const int32_t* m = meta + (int64_t)r * meta_ld;
    const int e = m[s];
    const bool own = e >= e_begin && e < e_end;
    if (!own && e != -1) atomicAdd(bad, 1);
    idx[i] = own ? e : E;
    w[i] = __int_as_float(m[k + s]);
    if (s == 0) sgate[r] = r < Tsh ? __int_as_float(m[2 * k]) : 0.f;
}

// out[t] = self_out[t] + sum over remote ranks r (ascending) of back[pos[t][r]];
// the partial rows are f32, or f16 (PT = __half).
template <typename PT>
__device__ __forceinline__ float4 part4(const PT* p) {
    if constexpr (sizeof(PT) == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        return make_float4(a.x, a.y, b.x, b.y);
    } else {
        return ld_f4(reinterpret_cast<const float*>(p));
    }
}

template <typename PT>
__global__ void ep_combine_kernel(const PT* __restrict__ self_out, const PT* __restrict__ back,
                                  const int32_t* __restrict__ pos, int T, int n, int me, int dp,
                                  float* __restrict__ out) {
    const int d4 = dp >> 2;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * d4) return;
    const int t = (int)(i / d4), c = (int)(i % d4) * 4;
    float4 acc = part4(self_out + (int64_t)t * dp + c);
    for (int r = 0; r < n; ++r) {
        if (r == me) continue;
        const int p = pos[(int64_t)t * n + r];
        if (p < 0) continue;
        const float4 v = part4(back + (int64_t)p * dp + c);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    *reinterpret_cast<float4*>(out + (int64_t)t * dp + c) = acc;
}

}  // namespace

cudaError_t launch_ep_plan(const int32_t* idx, int T, int k, const EpRankTable& rt, int me, int slab,
                           int32_t* send_tok, int32_t* send_rank, int32_t* counts, int32_t* pos, cudaStream_t s) {
    ep_plan_kernel<<<1, kPlanThreads, 0, s>>>(idx, T, k, rt, me, slab, send_tok, send_rank, counts, pos);
    return cudaGetLastError();
}

cudaError_t launch_ep_pack(const float* x, int T, int dp, int k, const int32_t* idx, const float* w,
                           const float* sgate, int has_shared, const EpRankTable& rt, int me, int slab,
                           const int32_t* send_tok, const int32_t* counts, int rows_f16, void* self_rows,
                           int32_t* self_meta, void* send_rows, int32_t* send_meta, int meta_ld, int n_sm,
                           cudaStream_t s) {
    const int64_t n = (int64_t)(T + rt.n * slab) * (dp / 8);
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)n_sm * 16));
    if (rows_f16)
        ep_pack_kernel<__half><<<grid, 256, 0, s>>>(x, T, dp, k, idx, w, sgate, has_shared, rt, me, slab, send_tok,
                                                    counts, static_cast<__half*>(self_rows), self_meta,
                                                    static_cast<__half*>(send_rows), send_meta, meta_ld);
    else
        ep_pack_kernel<float><<<grid, 256, 0, s>>>(x, T, dp, k, idx, w, sgate, has_shared, rt, me, slab, send_tok,
                                                   counts, static_cast<float*>(self_rows), self_meta,
                                                   static_cast<float*>(send_rows), send_meta, meta_ld);
    return cudaGetLastError();
}

cudaError_t launch_ep_prep(const int32_t* meta, int meta_ld, int R, int k, int Tsh, int e_begin, int e_end, int E,
                           int32_t* idx, float* w, float* sgate, int32_t* bad, cudaStream_t s) {
    const int64_t n = (int64_t)R * k;
    if (n == 0) return cudaSuccess;
    ep_prep_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(meta, meta_ld, R, k, Tsh, e_begin, e_end, E, idx, w,
                                                               sgate, bad);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const void* self_out, const void* back, int parts_f16, const int32_t* pos, int T, int n,
                              int me, int dp, float* out, cudaStream_t s) {
    const int64_t total = (int64_t)T * (dp / 4);
    if (total == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((total + 255) / 256);
    if (parts_f16)
        ep_combine_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(self_out),
                                                       static_cast<const __half*>(back), pos, T, n, me, dp, out);
    else
        ep_combine_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(self_out),
                                                      static_cast<const float*>(back), pos, T, n, me, dp, out);
    return cudaGetLastError();
}

}  // namespace aero
