// Decode-path expert products: bandwidth-bound grouped GEMVs on CUDA cores.
//
// Only the selected experts' quant blocks are streamed (16-byte non-allocating
// loads), dequantised in registers and accumulated in fp32; no tensor cores.
// Each active expert's weights are read once and applied to every token routed
// to it. Semantics per (token, expert) are those of aero_moe_expert_accum
// (src/moe.cpp:68-88): act = silu(gate.h) * (up.h), y = down.act, with the
// routing weight applied later by the combine kernel in slot order.
//
// gate/up: one CTA (4 warps) per (active expert, group of 16 rows); each warp
//          owns 4 rows and writes act[pos][row] for every routed pair; the CTA
//          then writes asum16[pos][group] = sum of its 16 act values, which the
//          Q4_K down product needs for its min term.
// down:    one CTA per (active expert, group of output rows); lanes split a row
//          into 16-byte chunks; y[pos][n] per routed pair.
#include "internal.h"

namespace aero {
namespace {

constexpr int kPairGroup = 4;  // tokens accumulated per pass over a row
constexpr int kMaxSlots = 4;   // 16-byte chunks per lane held in flight per matrix

struct UnitSrc {
    int e;        // expert index within the QMat
    int pos0;     // first sorted position of its pairs
    int npairs;
    bool shared;
};

__device__ __forceinline__ bool unit_of(const GemvArgs& a, int b, int groups_routed, int groups_shared,
                                        bool shared_launch, UnitSrc& u, int& grp) {
    const int P = a.T * a.k;
    if (!shared_launch) {
        const int n_act = *a.n_active;
        if (b >= n_act * groups_routed) return false;
        const int ui = b / groups_routed;
        grp = b % groups_routed;
        u.e = a.act_e[ui];
        u.pos0 = a.act_off[ui];
        u.npairs = a.act_off[ui + 1] - u.pos0;
        u.shared = false;
    } else {
        if (b >= groups_shared) return false;
        grp = b;
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

template <int DT, bool SHARED>
__global__ void __launch_bounds__(128) gateup_kernel(GemvArgs a) {
    const int F = SHARED ? a.Fs : a.F;
    UnitSrc u;
    int grp;
    if (!unit_of(a, blockIdx.x, a.F / 16, a.Fs / 16, SHARED, u, grp)) return;
    const QMat& G = SHARED ? a.sg : a.gate;
    const QMat& U = SHARED ? a.su : a.up;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = qm_chunks_per_row(DT, a.d);
    const int xs_ld = a.d / 16;

    for (int rr = 0; rr < 4; ++rr) {
        const int j = grp * 16 + warp * 4 + rr;
        if (j >= F) break;
        const uint8_t* gq = qm_row_qs(G, u.e, j);
        const uint8_t* gm = qm_row_meta(G, u.e, j);
        const uint8_t* uq = qm_row_qs(U, u.e, j);
        const uint8_t* um = qm_row_meta(U, u.e, j);
        for (int p0 = 0; p0 < u.npairs; p0 += kPairGroup) {
            float ga[kPairGroup], ua[kPairGroup];
            int tok[kPairGroup];
#pragma unroll
            for (int i = 0; i < kPairGroup; ++i) {
                ga[i] = ua[i] = 0.f;
                tok[i] = (p0 + i < u.npairs) ? token_of(a, u, u.pos0 + p0 + i) : -1;
            }
            for (int cb = 0; cb < nch; cb += 32 * kMaxSlots) {
                uint4 rg[kMaxSlots], ru[kMaxSlots], mg[kMaxSlots], mu[kMaxSlots];
#pragma unroll
                for (int s = 0; s < kMaxSlots; ++s) {
                    const int c = cb + s * 32 + lane;
                    if (c < nch) {
                        chunk_load<DT>(G, gq, gm, c, rg[s], mg[s]);
                        chunk_load<DT>(U, uq, um, c, ru[s], mu[s]);
                    }
                }
#pragma unroll
                for (int s = 0; s < kMaxSlots; ++s) {
                    const int c = cb + s * 32 + lane;
                    if (c >= nch) continue;
                    Chunk kc;
                    chunk_decode<DT>(c, rg[s], mg[s], kc);
#pragma unroll
                    for (int i = 0; i < kPairGroup; ++i)
                        if (tok[i] >= 0)
                            ga[i] += chunk_dot<DT>(kc, a.x + (int64_t)tok[i] * a.d, a.xsum16 + (int64_t)tok[i] * xs_ld);
                    chunk_decode<DT>(c, ru[s], mu[s], kc);
#pragma unroll
                    for (int i = 0; i < kPairGroup; ++i)
                        if (tok[i] >= 0)
                            ua[i] += chunk_dot<DT>(kc, a.x + (int64_t)tok[i] * a.d, a.xsum16 + (int64_t)tok[i] * xs_ld);
                }
            }
#pragma unroll
            for (int i = 0; i < kPairGroup; ++i) {
                const float g = warp_sum(ga[i]);
                const float uu = warp_sum(ua[i]);
                if (lane == 0 && tok[i] >= 0) a.act[(int64_t)(u.pos0 + p0 + i) * a.act_ld + j] = silu_f(g) * uu;
            }
        }
    }
    __syncthreads();
    // 16-row sums of act for this group (fixed summation order)
    const int as_ld = a.act_ld / 16;
    for (int p = threadIdx.x; p < u.npairs; p += blockDim.x) {
        const float* ar = a.act + (int64_t)(u.pos0 + p) * a.act_ld + grp * 16;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) s += (grp * 16 + i < F) ? ar[i] : 0.f;
        a.asum16[(int64_t)(u.pos0 + p) * as_ld + grp] = s;
    }
}

template <int DT, int LPR, bool SHARED>
__global__ void __launch_bounds__(128) down_kernel(GemvArgs a, int rows_per_cta) {
    const int Fin = SHARED ? a.Fs : a.F;
    const int groups = (a.d + rows_per_cta - 1) / rows_per_cta;
    UnitSrc u;
    int grp;
    if (!unit_of(a, blockIdx.x, groups, groups, SHARED, u, grp)) return;
    const QMat& D = SHARED ? a.sd : a.down;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane / LPR, gl = lane % LPR;
    constexpr int RPW = 32 / LPR;  // rows per warp pass
    const int nch = qm_chunks_per_row(DT, Fin);
    const int as_ld = a.act_ld / 16;

    for (int r0 = grp * rows_per_cta + warp * RPW; r0 < min(a.d, (grp + 1) * rows_per_cta); r0 += 4 * RPW) {
        const int n = r0 + sub;
        const bool row_ok = n < a.d && n < (grp + 1) * rows_per_cta;
        const uint8_t* dq = row_ok ? qm_row_qs(D, u.e, n) : nullptr;
        const uint8_t* dm = row_ok ? qm_row_meta(D, u.e, n) : nullptr;
        for (int p0 = 0; p0 < u.npairs; p0 += kPairGroup) {
            float acc[kPairGroup];
#pragma unroll
            for (int i = 0; i < kPairGroup; ++i) acc[i] = 0.f;
            for (int cb = 0; cb < nch; cb += LPR * kMaxSlots) {
                uint4 rw[kMaxSlots], mw[kMaxSlots];
#pragma unroll
                for (int s = 0; s < kMaxSlots; ++s) {
                    const int c = cb + s * LPR + gl;
                    if (row_ok && c < nch) chunk_load<DT>(D, dq, dm, c, rw[s], mw[s]);
                }
#pragma unroll
                for (int s = 0; s < kMaxSlots; ++s) {
                    const int c = cb + s * LPR + gl;
                    if (!row_ok || c >= nch) continue;
                    Chunk kc;
                    chunk_decode<DT>(c, rw[s], mw[s], kc);
#pragma unroll
                    for (int i = 0; i < kPairGroup; ++i) {
                        if (p0 + i < u.npairs) {
                            const int64_t pos = u.pos0 + p0 + i;
                            acc[i] += chunk_dot<DT>(kc, a.act + pos * a.act_ld, a.asum16 + pos * as_ld);
                        }
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < kPairGroup; ++i) {
                const float v = group_sum<LPR>(acc[i]);
                if (gl == 0 && row_ok && p0 + i < u.npairs) a.y[(int64_t)(u.pos0 + p0 + i) * a.d + n] = v;
            }
        }
    }
}

template <int DT>
cudaError_t gateup_dt(const GemvArgs& a, bool shared, cudaStream_t s) {
    if (!shared) {
        const int grid = a.max_active * (a.F / 16);
        if (grid > 0) gateup_kernel<DT, false><<<grid, 128, 0, s>>>(a);
    } else {
        gateup_kernel<DT, true><<<a.Fs / 16, 128, 0, s>>>(a);
    }
    return cudaGetLastError();
}

int pick_lpr(int nch) { return nch >= 64 ? 32 : nch >= 32 ? 16 : 8; }

template <int DT, int LPR>
cudaError_t down_dt_lpr(const GemvArgs& a, bool shared, cudaStream_t s) {
    const int rows_per_cta = 4 * (32 / LPR) * 2;
    const int groups = (a.d + rows_per_cta - 1) / rows_per_cta;
    if (!shared) {
        const int grid = a.max_active * groups;
        if (grid > 0) down_kernel<DT, LPR, false><<<grid, 128, 0, s>>>(a, rows_per_cta);
    } else {
        down_kernel<DT, LPR, true><<<groups, 128, 0, s>>>(a, rows_per_cta);
    }
    return cudaGetLastError();
}

template <int DT>
cudaError_t down_dt(const GemvArgs& a, bool shared, cudaStream_t s) {
    const int lpr = pick_lpr(qm_chunks_per_row(DT, shared ? a.Fs : a.F));
    if (lpr == 32) return down_dt_lpr<DT, 32>(a, shared, s);
    if (lpr == 16) return down_dt_lpr<DT, 16>(a, shared, s);
    return down_dt_lpr<DT, 8>(a, shared, s);
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
