// Decode-path expert products: bandwidth-bound grouped GEMVs on CUDA cores.
//
// Only the selected experts' quant blocks are streamed, dequantised in
// registers and accumulated in fp32; no tensor cores. Semantics per (token,
// expert) are those of aero_moe_expert_accum (src/moe.cpp:68-88): act =
// silu(gate.h) * (up.h), y = down.act, with the routing weight applied later by
// the combine kernel in slot order.
//
// A warp computes one row dot at a time: its lanes split the row into 16-byte
// code chunks (coalesced streaming loads, the next row's chunks prefetched into
// registers), and each lane keeps the input values matching its chunks in
// registers for the whole CTA, so the only per-row traffic is the weights. A
// CTA owns one unit (an active expert, or the shared expert) x a block of rows
// x one token; tokens of a unit take successive passes (decode units hold 1-2).
// Per 32-value sub-block the products follow the reference factorisation of the
// quantised dot (src/kernels.cpp:78-84, 123-156):
//   Q8_0: d * sum(q x)            Q4_K: d sc * sum(q x) - dmin m * sum(x)
// For the quantised families the input rows come in integer form (QInput: a
// 15-bit code per value split into two int8 planes, one f32 scale per 32
// values, exact f32 sums per 16), so sum(q x) is two chains of dp4a over the
// raw code bytes: no per-value conversion. Its relative error is bounded by
// 2^-15 of the block's largest input; accumulation is f32. F32 experts take a
// plain f32 dot.
#include <algorithm>

#include "gemv_rows.cuh"
#include "internal.h"

namespace aero {
namespace {

constexpr int kWarps = 8;
constexpr int kMaxChunks = 4;    // code chunks per lane

struct UnitSrc {
    int e;        // expert index within the QMat
    int pos0;     // first sorted position of its pairs
    int npairs;
    bool shared;
};

__device__ __forceinline__ bool unit_of(const GemvArgs& a, int ui, bool shared_launch, UnitSrc& u) {
    const int P = a.T * a.k;
    if (!shared_launch) {
        if (ui >= *a.n_active) return false;
        u.e = a.act_e[ui];
        u.pos0 = a.act_off[ui];
        u.npairs = a.act_off[ui + 1] - u.pos0;
        u.shared = false;
    } else {
        u.e = 0;
        u.pos0 = P;
        u.npairs = a.Tsh;
        u.shared = true;
    }
    return true;
}

__device__ __forceinline__ int token_of(const GemvArgs& a, const UnitSrc& u, int pos) {
    return u.shared ? pos - a.T * a.k : a.perm[pos] / a.k;
}


// gate/up: CTA = (unit, 32-row block, token of the unit). The warp's row slots
// (32 / LPR rows at once) walk the block's rows; each slot streams the items
// gate row j, up row j, gate row j', ... with the next item prefetched.
template <int DT, int LPR, int CPL, bool SHARED>
__global__ void __launch_bounds__(kWarps * 32, 2) gateup_kernel(GemvArgs a, int rows_per_cta) {
    constexpr int kSlots = 32 / LPR;
    const int F = SHARED ? a.Fs : a.F;
    const int row_blocks = (F + rows_per_cta - 1) / rows_per_cta;
    UnitSrc u;
    const int ui = SHARED ? 0 : (int)blockIdx.x / row_blocks;
    if (!unit_of(a, ui, SHARED, u)) return;
    const int rb = (int)blockIdx.x % row_blocks;
    const QMat& G = SHARED ? a.sg : a.gate;
    const QMat& U = SHARED ? a.su : a.up;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = lane / LPR, gl = lane % LPR;
    const int nch = Layout<DT>::chunks(a.d);
    __shared__ __align__(16) float act_s[256];  // this block's act values of the current token
    // tokens of the unit: blockIdx.y, blockIdx.y + gridDim.y, ...
    for (int t = (int)blockIdx.y; t < u.npairs; t += (int)gridDim.y) {
    const int64_t pos = u.pos0 + t;
    LaneInput<DT, CPL> in;
    input_load<DT, LPR, CPL>(a.x, a.xq, token_of(a, u, (int)pos), gl, nch, in);
    const int j0 = rb * rows_per_cta + warp * kSlots + slot;
    const int jstep = kWarps * kSlots;
    const int jend = min(F, (rb + 1) * rows_per_cta);
    const int n_items = 2 * ((rb * rows_per_cta + rows_per_cta - j0 + jstep - 1) / jstep);  // same count for every lane
    auto item_row = [&](int it) { return j0 + (it >> 1) * jstep; };
    RowRaw<DT, CPL> cur;
    if (item_row(0) < jend) row_load<DT, LPR, CPL>(G, u.e, item_row(0), gl, nch, cur);
    float g = 0.f;
    for (int it = 0; it < n_items; ++it) {
        const int j = item_row(it);
        RowRaw<DT, CPL> nxt;
        if (it + 1 < n_items && item_row(it + 1) < jend)
            row_load<DT, LPR, CPL>((it + 1) & 1 ? U : G, u.e, item_row(it + 1), gl, nch, nxt);
        float v = j < jend ? row_dot<DT, LPR, CPL>(cur, in, gl, nch) : 0.f;
        v = lanes_sum<LPR>(v);
        if (it & 1) {
            if (j < jend && gl == 0) {
                const float h = silu_f(g) * v;
                a.act[pos * a.act_ld + j] = h;
                if (DT != AERO_DT_F32) act_s[j - rb * rows_per_cta] = h;
            }
        } else {
            g = v;
        }
        cur = nxt;
    }
    if (DT != AERO_DT_F32) {
        // the block's act values (whole 32-row blocks: rows_per_cta and F are
        // multiples of 32) as integer input of the down product
        __syncthreads();
        for (int b = threadIdx.x; b * 32 < jend - rb * rows_per_cta; b += blockDim.x) {
            const int j = rb * rows_per_cta + 32 * b;
            qinput_block(act_s + 32 * b, a.aq.q1 + pos * a.aq.K + j, a.aq.q0 + pos * a.aq.K + j,
                         a.aq.sx + pos * (a.aq.K / 32) + (j >> 5), a.aq.s16 + pos * (a.aq.K / 16) + (j >> 4));
        }
        __syncthreads();
    }
    }
}

// down: CTA = (unit, 32 output rows, token); y[pos][n] = down_n . act[pos].
template <int DT, int LPR, int CPL, bool SHARED>
__global__ void __launch_bounds__(kWarps * 32, 2) down_kernel(GemvArgs a, int rows_per_cta) {
    constexpr int kSlots = 32 / LPR;
    const int K = SHARED ? a.Fs : a.F;
    const int row_blocks = (a.d + rows_per_cta - 1) / rows_per_cta;
    UnitSrc u;
    const int ui = SHARED ? 0 : (int)blockIdx.x / row_blocks;
    if (!unit_of(a, ui, SHARED, u)) return;
    const int rb = (int)blockIdx.x % row_blocks;
    const QMat& D = SHARED ? a.sd : a.down;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int slot = lane / LPR, gl = lane % LPR;
    const int nch = Layout<DT>::chunks(K);
    for (int t = (int)blockIdx.y; t < u.npairs; t += (int)gridDim.y) {
    const int64_t pos = u.pos0 + t;
    LaneInput<DT, CPL> in;
    input_load<DT, LPR, CPL>(a.act, a.aq, pos, gl, nch, in);
    const int n0 = rb * rows_per_cta + warp * kSlots + slot;
    const int nstep = kWarps * kSlots;
    const int nend = min(a.d, (rb + 1) * rows_per_cta);
    RowRaw<DT, CPL> w;
    if (n0 < nend) row_load<DT, LPR, CPL>(D, u.e, n0, gl, nch, w);
    for (int n = n0; n < rb * rows_per_cta + rows_per_cta; n += nstep) {
        const bool ok = n < nend;
        RowRaw<DT, CPL> nx;
        if (n + nstep < nend) row_load<DT, LPR, CPL>(D, u.e, n + nstep, gl, nch, nx);
        float v = ok ? row_dot<DT, LPR, CPL>(w, in, gl, nch) : 0.f;
        v = lanes_sum<LPR>(v);
        if (ok && gl == 0) a.y[pos * a.d + n] = v;
        w = nx;
    }
    }
}

// Lanes per row and chunks per lane for rows of K values: a full warp with up to
// kMaxChunks chunks per lane, or fewer lanes with one chunk each for short rows.
template <int DT>
bool row_split(int K, int* lpr, int* cpl) {
    const int nch = Layout<DT>::chunks(K);
    if (nch <= 0) return false;
    for (int l : {4, 8, 16}) {
        if (nch <= l) {
            *lpr = l;
            *cpl = 1;
            return true;
        }
    }
    *lpr = 32;
    *cpl = (nch + 31) / 32;
    return *cpl <= kMaxChunks;
}

template <int DT, int LPR, int CPL>
cudaError_t gemv_launch(const GemvArgs& a, bool shared, bool gateup, cudaStream_t s) {
    const int rows = gateup ? (shared ? a.Fs : a.F) : a.d;
    // rows per CTA: about 2048 CTAs over the launch's units (32 rows at least, so
    // a few decode experts still spread over every SM; 256 at most)
    const int units = shared ? 1 : std::max(1, a.max_active);
    int rows_per_cta = 32;
    while (rows_per_cta < 256 && (int64_t)units * ((rows + rows_per_cta - 1) / rows_per_cta) > 2048) rows_per_cta *= 2;
    const int row_blocks = (rows + rows_per_cta - 1) / rows_per_cta;
    // token slots in y: every shared-expert token; up to 4 for a routed expert (decode
    // experts hold one or two), each CTA looping over the rest
    const dim3 grid = shared ? dim3(row_blocks, a.Tsh) : dim3(a.max_active * row_blocks, std::min(a.max_pairs, 4));
    if (grid.x == 0 || grid.y == 0) return cudaSuccess;
    if (gateup) {
        if (shared)
            gateup_kernel<DT, LPR, CPL, true><<<grid, kWarps * 32, 0, s>>>(a, rows_per_cta);
        else
            gateup_kernel<DT, LPR, CPL, false><<<grid, kWarps * 32, 0, s>>>(a, rows_per_cta);
    } else {
        if (shared)
            down_kernel<DT, LPR, CPL, true><<<grid, kWarps * 32, 0, s>>>(a, rows_per_cta);
        else
            down_kernel<DT, LPR, CPL, false><<<grid, kWarps * 32, 0, s>>>(a, rows_per_cta);
    }
    return cudaGetLastError();
}

template <int DT>
cudaError_t gemv_dt(const GemvArgs& a, bool shared, bool gateup, cudaStream_t s) {
    const int K = gateup ? a.d : (shared ? a.Fs : a.F);
    int lpr = 0, cpl = 0;
    if (!row_split<DT>(K, &lpr, &cpl)) return cudaErrorInvalidValue;
    if (lpr == 4) return gemv_launch<DT, 4, 1>(a, shared, gateup, s);
    if (lpr == 8) return gemv_launch<DT, 8, 1>(a, shared, gateup, s);
    if (lpr == 16) return gemv_launch<DT, 16, 1>(a, shared, gateup, s);
    switch (cpl) {
        case 1: return gemv_launch<DT, 32, 1>(a, shared, gateup, s);
        case 2: return gemv_launch<DT, 32, 2>(a, shared, gateup, s);
        case 3: return gemv_launch<DT, 32, 3>(a, shared, gateup, s);
        case 4: return gemv_launch<DT, 32, 4>(a, shared, gateup, s);
    }
    return cudaErrorInvalidValue;
}

template <int DT>
cudaError_t gateup_dt(const GemvArgs& a, bool shared, cudaStream_t s) {
    return gemv_dt<DT>(a, shared, true, s);
}
template <int DT>
cudaError_t down_dt(const GemvArgs& a, bool shared, cudaStream_t s) {
    return gemv_dt<DT>(a, shared, false, s);
}

cudaError_t gateup_any(int dtype, const GemvArgs& a, bool shared, cudaStream_t s) {
    switch (dtype) {
        case AERO_DT_Q8_0: return gateup_dt<AERO_DT_Q8_0>(a, shared, s);
        case AERO_DT_Q4_K: return gateup_dt<AERO_DT_Q4_K>(a, shared, s);
        case AERO_DT_F32: return gateup_dt<AERO_DT_F32>(a, shared, s);
    }
    return cudaErrorInvalidValue;
}
cudaError_t down_any(int dtype, const GemvArgs& a, bool shared, cudaStream_t s) {
    switch (dtype) {
        case AERO_DT_Q8_0: return down_dt<AERO_DT_Q8_0>(a, shared, s);
        case AERO_DT_Q4_K: return down_dt<AERO_DT_Q4_K>(a, shared, s);
        case AERO_DT_F32: return down_dt<AERO_DT_F32>(a, shared, s);
    }
    return cudaErrorInvalidValue;
}

__global__ void combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ inv,
                               const float* __restrict__ w, const float* __restrict__ sgate,
                               const int32_t* __restrict__ idx, int E_real, int T, int Tsh, int k, int d,
                               int has_shared, float* __restrict__ out) {
    const int d4 = d >> 2;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * d4) return;
    const int t = (int)(i / d4), c = (int)(i % d4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < k; ++s) {
        if (idx && idx[(int64_t)t * k + s] >= E_real) continue;
        const float wt = w[(int64_t)t * k + s];
        const float4 v = ld_f4(y + (int64_t)inv[(int64_t)t * k + s] * d + c);
        acc.x += wt * v.x;
        acc.y += wt * v.y;
        acc.z += wt * v.z;
        acc.w += wt * v.w;
    }
    if (has_shared && t < Tsh) {
        const float g = sgate[t];
        const float4 v = ld_f4(y + ((int64_t)T * k + t) * d + c);
        acc.x += g * v.x;
        acc.y += g * v.y;
        acc.z += g * v.z;
        acc.w += g * v.w;
    }
    *reinterpret_cast<float4*>(out + (int64_t)t * d + c) = acc;
}

}  // namespace

cudaError_t launch_gemv_gateup(const GemvArgs& a, cudaStream_t s) {
    cudaError_t e = gateup_any(a.gate.dtype, a, false, s);
    if (e == cudaSuccess && a.has_shared && a.Tsh > 0) e = gateup_any(a.sg.dtype, a, true, s);
    return e;
}

cudaError_t launch_gemv_down(const GemvArgs& a, cudaStream_t s) {
    cudaError_t e = down_any(a.down.dtype, a, false, s);
    if (e == cudaSuccess && a.has_shared && a.Tsh > 0) e = down_any(a.sd.dtype, a, true, s);
    return e;
}

cudaError_t launch_combine(const float* y, const int32_t* inv, const float* w, const float* sgate,
                           const int32_t* idx, int E_real, int T, int Tsh, int k, int d, int has_shared, float* out,
                           cudaStream_t s) {
    const int64_t n = (int64_t)T * (d / 4);
    if (n == 0) return cudaSuccess;
    combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, inv, w, sgate, idx, E_real, T, Tsh, k, d,
                                                               has_shared, out);
    return cudaGetLastError();
}

}  // namespace aero
