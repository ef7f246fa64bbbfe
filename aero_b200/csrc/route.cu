// Router projection, top-k routing and expert dispatch.
//
// Routing follows src/moe.cpp:26-66: experts ranked by descending logit, equal
// logits ranked by the lower expert index; with norm_topk_prob the k weights are
// the softmax over the selected logits (max-subtracted, f32 exp), otherwise the
// full-softmax probability with an f64 denominator over all experts.
//
// Dispatch (no reference counterpart — the reference loops token by token):
// the T*k (token, slot) pairs, pair id p = t*k + s, are counting-sorted by
// expert; inside an expert they keep pair order, i.e. (token, slot) order.
#include <algorithm>

#include <cub/block/block_scan.cuh>

#include "internal.h"
#include "topk.cuh"

namespace aero {
namespace {

// ----------------------------------------------------------- router, small T
// One warp per W row; the row is streamed once per group of 8 tokens.
constexpr int kRouterTG = 8;

__global__ void __launch_bounds__(256) router_gemv_kernel(const float* __restrict__ x, int T, int d,
                                                          const float* __restrict__ W, int row_begin,
                                                          int row_end, const float* __restrict__ bias,
                                                          int n_bias, float* __restrict__ logits, int ld) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = row_begin + blockIdx.x * 8 + warp;
    if (r >= row_end) return;
    const float* wr = W + (int64_t)r * d;
    const int n4 = d >> 2;
    for (int t0 = 0; t0 < T; t0 += kRouterTG) {
        float acc[kRouterTG];
#pragma unroll
        for (int i = 0; i < kRouterTG; ++i) acc[i] = 0.f;
        for (int c = lane; c < n4; c += 32) {
            const float4 wv = ld_f4(wr + 4 * c);
#pragma unroll
            for (int i = 0; i < kRouterTG; ++i) {
                if (t0 + i < T) {
                    const float4 xv = ld_f4(x + (int64_t)(t0 + i) * d + 4 * c);
                    acc[i] = fmaf(wv.x, xv.x, acc[i]);
                    acc[i] = fmaf(wv.y, xv.y, acc[i]);
                    acc[i] = fmaf(wv.z, xv.z, acc[i]);
                    acc[i] = fmaf(wv.w, xv.w, acc[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kRouterTG; ++i) {
            const float v = warp_sum(acc[i]);
            if (lane == 0 && t0 + i < T) logits[(int64_t)(t0 + i) * ld + r] = v + (r < n_bias && bias ? bias[r] : 0.f);
        }
    }
}

// ----------------------------------------------------------- router, T <= 4
// One CTA per W row: its 256 threads split the row (one float4 of W per step,
// all of the row's loads in flight at once) and a block reduction adds them.
constexpr int kRouterTinyT = 4;

__global__ void __launch_bounds__(256) router_tiny_kernel(const float* __restrict__ x, int T, int d,
                                                          const float* __restrict__ W, int row_begin,
                                                          const float* __restrict__ bias, int n_bias,
                                                          float* __restrict__ logits, int ld) {
    __shared__ float part[kRouterTinyT][8];
    const int r = row_begin + blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* wr = W + (int64_t)r * d;
    float acc[kRouterTinyT] = {0.f, 0.f, 0.f, 0.f};
    for (int c = threadIdx.x * 4; c < d; c += 256 * 4) {
        const float4 wv = ld_f4(wr + c);
#pragma unroll
        for (int i = 0; i < kRouterTinyT; ++i)
            if (i < T) {
                const float4 xv = ld_f4(x + (int64_t)i * d + c);
                acc[i] = fmaf(wv.x, xv.x, acc[i]);
                acc[i] = fmaf(wv.y, xv.y, acc[i]);
                acc[i] = fmaf(wv.z, xv.z, acc[i]);
                acc[i] = fmaf(wv.w, xv.w, acc[i]);
            }
    }
#pragma unroll
    for (int i = 0; i < kRouterTinyT; ++i) {
        const float v = warp_sum(acc[i]);
        if (lane == 0) part[i][warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < T) {
        float v = 0.f;
#pragma unroll
        for (int w8 = 0; w8 < 8; ++w8) v += part[threadIdx.x][w8];
        logits[(int64_t)threadIdx.x * ld + r] = v + (r < n_bias && bias ? bias[r] : 0.f);
    }
}

// ----------------------------------------------------------- router, large T
// 64x64 output tile per CTA, 256 threads with a 4x4 micro-tile each, K in steps
// of 16 through shared memory (both operands are K-major in global memory).
constexpr int kSgBM = 64, kSgBN = 64, kSgBK = 16;

__global__ void __launch_bounds__(256) router_sgemm_kernel(const float* __restrict__ x, int T, int d,
                                                           const float* __restrict__ W, int row_begin,
                                                           int row_end, const float* __restrict__ bias,
                                                           int n_bias, float* __restrict__ logits, int ld) {
    __shared__ float As[kSgBK][kSgBM + 4];
    __shared__ float Bs[kSgBK][kSgBN + 4];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * kSgBM, n0 = row_begin + blockIdx.x * kSgBN;
    const int tm = (tid / 16) * 4, tn = (tid % 16) * 4;
    float acc[4][4] = {};
    // each thread loads one float4 of A and one of B per K step: 64 rows x 4 float4
    const int lr = tid >> 2, lk = (tid & 3) * 4;
    for (int k0 = 0; k0 < d; k0 += kSgBK) {
        {
            const int gm = m0 + lr;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gm < T) v = ld_f4(x + (int64_t)gm * d + k0 + lk);
            As[lk + 0][lr] = v.x;
            As[lk + 1][lr] = v.y;
            As[lk + 2][lr] = v.z;
            As[lk + 3][lr] = v.w;
            const int gn = n0 + lr;
            float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gn < row_end) u = ld_f4(W + (int64_t)gn * d + k0 + lk);
            Bs[lk + 0][lr] = u.x;
            Bs[lk + 1][lr] = u.y;
            Bs[lk + 2][lr] = u.z;
            Bs[lk + 3][lr] = u.w;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kSgBK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][tm + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tn + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + tm + i;
        if (gm >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tn + j;
            if (gn < row_end) logits[(int64_t)gm * ld + gn] = acc[i][j] + (gn < n_bias && bias ? bias[gn] : 0.f);
        }
    }
}

// ---------------------------------------------------------------- top-k
// One warp per token (topk_warp in topk.cuh).
constexpr int kTopkMaxPerLane = 32;  // E <= 1024

template <int PER>  // values per lane: E <= 32 * PER
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ logits, int ld, int T, int E,
                                                   int k, int norm, int has_shared, int32_t* __restrict__ idx,
                                                   float* __restrict__ w, float* __restrict__ sgate,
                                                   const float* __restrict__ x, QInput xq, SingleDispatch one) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    const float* lg = logits + (int64_t)t * ld;
    int sel_i = 0;
    topk_warp<PER>(lg, E, k, norm, idx + (int64_t)t * k, w + (int64_t)t * k, &sel_i);
    if (one.perm && T == 1) {
        if (lane < k) {
            one.perm[lane] = lane;
            one.inv[lane] = lane;
            one.act_e[lane] = sel_i;
            one.act_off[lane] = lane;
        }
        if (lane == 0) {
            one.act_off[k] = k;
            *one.n_active = k;
            *one.p_real = k;
        }
    }
    if (has_shared && lane == 0) sgate[t] = sigmoid_f(lg[E]);
    if (xq.q1) {
        // this token's x row as integer input for the decode GEMVs
        const int K = xq.K;
        const float* xr = x + (int64_t)t * K;
        for (int b = lane; b < K / 32; b += 32)
            qinput_block(xr + 32 * b, xq.q1 + (int64_t)t * K + 32 * b, xq.q0 + (int64_t)t * K + 32 * b,
                         xq.sx + (int64_t)t * (K / 32) + b, xq.s16 + (int64_t)t * (K / 16) + 2 * b);
    }
}

// ---------------------------------------------------------------- dispatch
// Chunks of kDispChunk pairs. count: per-chunk per-expert histogram; scan:
// per-expert running offsets over chunks plus the expert prefix; scatter: each
// chunk is walked in pair order by one warp, 32 pairs at a time, ranking equal
// experts with __match_any_sync, so the result is stable.
constexpr int kDispChunk = 256;  // minimum chunk; large calls use ~148 chunks (one per SM)

int dispatch_chunk(int P) {
    const int per = (P + 147) / 148;
    return std::max(kDispChunk, (per + 31) / 32 * 32);
}

__global__ void dispatch_count_kernel(const int32_t* __restrict__ idx, int P, int E, int chunk,
                                      int32_t* __restrict__ counts) {
    extern __shared__ int32_t hist[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * chunk;
    for (int p = p0 + threadIdx.x; p < min(P, p0 + chunk); p += blockDim.x) atomicAdd(&hist[idx[p]], 1);
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[(int64_t)blockIdx.x * E + e] = hist[e];
}

constexpr int kScanThreads = 1024;

// Per expert (a lane of each warp), the chunk histogram becomes the
// within-expert exclusive prefix over chunks: warp w of the CTA sums a
// contiguous run of chunks, the runs are prefixed across warps, and each run
// is rewritten from its prefix. totals[e] = the expert's pair count.
__global__ void __launch_bounds__(kScanThreads) dispatch_colscan_kernel(int32_t* __restrict__ counts, int n_chunks,
                                                                        int E, int32_t* __restrict__ totals) {
    __shared__ int part[32][33];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.x * 32 + lane;
    const int per = (n_chunks + 31) / 32;
    const int c0 = warp * per, c1 = min(n_chunks, c0 + per);
    int sum = 0;
    if (e < E)
        for (int c = c0; c < c1; ++c) sum += counts[(int64_t)c * E + e];
    part[warp][lane] = sum;
    __syncthreads();
    int run = 0;
    for (int w = 0; w < warp; ++w) run += part[w][lane];
    if (e < E) {
        for (int c = c0; c < c1; ++c) {
            const int v = counts[(int64_t)c * E + e];
            counts[(int64_t)c * E + e] = run;
            run += v;
        }
        if (warp == 31) totals[e] = run;
    }
}

// Expert offsets (exclusive prefix of totals), offsets[E] = P, and the active
// experts below n_real in order with their offsets.
__global__ void __launch_bounds__(kScanThreads) dispatch_scan_kernel(const int32_t* __restrict__ totals, int E,
                                                                     int n_real, int P,
                                                                     int32_t* __restrict__ offsets,
                                                                     int32_t* __restrict__ act_e,
                                                                     int32_t* __restrict__ act_off,
                                                                     int32_t* __restrict__ n_active) {
    using Scan = cub::BlockScan<int, kScanThreads>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ int carry_tot, carry_act;
    if (threadIdx.x == 0) {
        carry_tot = 0;
        carry_act = 0;
    }
    __syncthreads();
    for (int e0 = 0; e0 < E; e0 += kScanThreads) {
        const int e = e0 + threadIdx.x;
        const int tot = e < E ? totals[e] : 0;
        int excl, excl_act;
        Scan(tmp).ExclusiveSum(tot, excl);
        __syncthreads();
        const bool active = tot > 0 && e < n_real;  // buckets >= n_real hold skipped slots
        Scan(tmp).ExclusiveSum(active ? 1 : 0, excl_act);
        const int base = carry_tot, abase = carry_act;
        if (e < E) {
            offsets[e] = base + excl;
            if (active) {
                act_e[abase + excl_act] = e;
                act_off[abase + excl_act] = base + excl;
            }
        }
        __syncthreads();
        if (threadIdx.x == kScanThreads - 1) {
            carry_tot = base + excl + tot;
            carry_act = abase + excl_act + (active ? 1 : 0);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        offsets[E] = P;
        act_off[carry_act] = n_real < E ? offsets[n_real] : P;
        *n_active = carry_act;
    }
}

__global__ void dispatch_scatter_kernel(const int32_t* __restrict__ idx, int P, int E, int chunk_len,
                                        const int32_t* __restrict__ offsets,
                                        const int32_t* __restrict__ counts, int32_t* __restrict__ perm,
                                        int32_t* __restrict__ inv) {
    extern __shared__ int32_t cursor[];  // per expert, for this chunk
    const int chunk = blockIdx.x;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = offsets[e] + counts[(int64_t)chunk * E + e];
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    const int p_end = min(P, (chunk + 1) * chunk_len);
    for (int base = chunk * chunk_len; base < p_end; base += 32) {
        const int p = base + lane;
        const bool valid = p < p_end;
        const int e = valid ? idx[p] : -1 - lane;  // invalid lanes never match a real expert
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int pos = 0;
        if (valid) pos = cursor[e] + rank;
        __syncwarp();
        if (valid) {
            perm[pos] = p;
            inv[p] = pos;
            // the highest peer advances the cursor past the whole group
            if ((peers >> lane) == 1u) cursor[e] = pos + 1;
        }
        __syncwarp();
    }
}

// One thread per 32-value block.
__global__ void qinput_kernel(const float* __restrict__ x, int R, int ld, QInput q) {
    const int nb = q.K / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)R * nb) return;
    const int r = (int)(i / nb), b = (int)(i % nb);
    qinput_block(x + (int64_t)r * ld + 32 * b, q.q1 + (int64_t)r * q.K + 32 * b, q.q0 + (int64_t)r * q.K + 32 * b,
                 q.sx + (int64_t)r * nb + b, q.s16 + (int64_t)r * (q.K / 16) + 2 * b);
}

// Routed global expert ids -> resident slots. An id without a slot records
// kErrNotResident and takes slot 0, so the rest of the call stays in bounds
// (its output is then reported invalid).
__global__ void resident_remap_kernel(int32_t* __restrict__ idx, int n, const int32_t* __restrict__ slot,
                                      int32_t* __restrict__ err, int32_t* err_host) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t r = slot[idx[i]];
    if (r < 0 && atomicCAS(err, 0, kErrNotResident) == 0 && err_host)
        *reinterpret_cast<volatile int32_t*>(err_host) = kErrNotResident;
    idx[i] = r < 0 ? 0 : r;
}

}  // namespace

cudaError_t launch_resident_remap(int32_t* idx, int n, const int32_t* slot, int32_t* err, int32_t* err_host,
                                  cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    resident_remap_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(idx, n, slot, err, err_host);
    return cudaGetLastError();
}

cudaError_t launch_qinput(const float* x, int R, int ld, QInput q, cudaStream_t s) {
    const int64_t n = (int64_t)R * (q.K / 32);
    if (n == 0) return cudaSuccess;
    qinput_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(x, R, ld, q);
    return cudaGetLastError();
}

cudaError_t launch_router(const float* x, int T, int d, const float* W, int row_begin, int row_end,
                          const float* bias, int n_bias, float* logits, int ld, cudaStream_t s) {
    const int rows = row_end - row_begin;
    if (rows <= 0 || T <= 0) return cudaSuccess;
    if (T <= kRouterTinyT && d % 4 == 0) {
        router_tiny_kernel<<<rows, 256, 0, s>>>(x, T, d, W, row_begin, bias, n_bias, logits, ld);
    } else if (T <= 32) {
        router_gemv_kernel<<<(rows + 7) / 8, 256, 0, s>>>(x, T, d, W, row_begin, row_end, bias, n_bias, logits, ld);
    } else {
        dim3 grid((rows + kSgBN - 1) / kSgBN, (T + kSgBM - 1) / kSgBM);
        router_sgemm_kernel<<<grid, 256, 0, s>>>(x, T, d, W, row_begin, row_end, bias, n_bias, logits, ld);
    }
    return cudaGetLastError();
}

cudaError_t launch_topk(const float* logits, int ld, int T, int E, int k, int norm, int has_shared, int32_t* idx,
                        float* w, float* sgate, const float* x, QInput xq, cudaStream_t s, SingleDispatch one) {
    if (T <= 0) return cudaSuccess;
    const unsigned grid = (unsigned)((T + 7) / 8);
    if (E <= 32)
        topk_kernel<1><<<grid, 256, 0, s>>>(logits, ld, T, E, k, norm, has_shared, idx, w, sgate, x, xq, one);
    else if (E <= 64)
        topk_kernel<2><<<grid, 256, 0, s>>>(logits, ld, T, E, k, norm, has_shared, idx, w, sgate, x, xq, one);
    else if (E <= 128)
        topk_kernel<4><<<grid, 256, 0, s>>>(logits, ld, T, E, k, norm, has_shared, idx, w, sgate, x, xq, one);
    else if (E <= 256)
        topk_kernel<8><<<grid, 256, 0, s>>>(logits, ld, T, E, k, norm, has_shared, idx, w, sgate, x, xq, one);
    else if (E <= 512)
        topk_kernel<16><<<grid, 256, 0, s>>>(logits, ld, T, E, k, norm, has_shared, idx, w, sgate, x, xq, one);
    else
        topk_kernel<32><<<grid, 256, 0, s>>>(logits, ld, T, E, k, norm, has_shared, idx, w, sgate, x, xq, one);
    return cudaGetLastError();
}

size_t dispatch_work_bytes(int P, int E) {
    const int chunk = dispatch_chunk(P);
    const size_t n_chunks = (size_t)(P + chunk - 1) / chunk;
    return (std::max<size_t>(1, n_chunks) + 1) * (size_t)E * sizeof(int32_t);  // histograms, then totals
}

cudaError_t launch_dispatch(const int32_t* idx, int P, int E, int32_t* offsets, int32_t* perm, int32_t* inv,
                            int32_t* act_e, int32_t* act_off, int32_t* n_active, void* work, cudaStream_t s,
                            int n_real) {
    if (n_real < 0) n_real = E;
    const int chunk = dispatch_chunk(P);
    const int n_chunks = std::max(1, (P + chunk - 1) / chunk);
    int32_t* counts = static_cast<int32_t*>(work);
    int32_t* totals = counts + (size_t)n_chunks * E;
    const size_t hist_smem = (size_t)E * sizeof(int32_t);
    dispatch_count_kernel<<<n_chunks, 256, hist_smem, s>>>(idx, P, E, chunk, counts);
    dispatch_colscan_kernel<<<(E + 31) / 32, kScanThreads, 0, s>>>(counts, n_chunks, E, totals);
    dispatch_scan_kernel<<<1, kScanThreads, 0, s>>>(totals, E, n_real, P, offsets, act_e, act_off, n_active);
    dispatch_scatter_kernel<<<n_chunks, 128, hist_smem, s>>>(idx, P, E, chunk, offsets, counts, perm, inv);
    return cudaGetLastError();
}

}  // namespace aero
