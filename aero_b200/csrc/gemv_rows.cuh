// Row-dot building blocks of the CUDA-core GEMVs (gemv.cu's grouped expert
// products and the decoder's dense projections): a row of K quantised values
// is split into 16-byte code chunks, lane gl of a row's LPR lanes holding chunks
// base + gl + LPR i (i < CPL). The input rows come as integer codes (QInput),
// so each 16-value run is two dp4a chains over the raw code bytes; the products
// follow the reference factorisation of the quantised dot (src/kernels.cpp:78-84,
// 123-156): Q8_0 d * sum(q x), Q4_K d sc * sum(q x) - dmin m * sum(x).
#pragma once

#include "internal.h"

namespace aero {
namespace {

template <int DT>
struct Layout;
// Q8_0 row of K values: K bytes of codes, a f16 scale per 32 values. Chunk c =
// values [16 c, 16 c + 16).
template <>
struct Layout<AERO_DT_Q8_0> {
    static constexpr int kVals = 16;  // values per chunk
    static constexpr int kWords = 1;  // 16-byte loads per chunk
    static __host__ __device__ __forceinline__ int chunks(int K) { return K / 16; }
};
// Q4_K row: 256-value super-blocks of 128 code bytes and a 16-byte header.
// Chunk c = code bytes [16 c, 16 c + 16): super-block c / 8, byte group
// g = (c % 8) / 2 of 32 bytes, half h = c % 2; its low nibbles are values
// 64 g + 16 h + [0, 16) (sub-block 2 g) and its high nibbles 64 g + 32 + 16 h +
// [0, 16) (sub-block 2 g + 1) of the super-block.
template <>
struct Layout<AERO_DT_Q4_K> {
    static constexpr int kVals = 32;
    static constexpr int kWords = 1;
    static __host__ __device__ __forceinline__ int chunks(int K) { return K / 32; }
};
// F32 (padded to 16) row: chunk c = values [16 c, 16 c + 16), four 16-byte loads.
template <>
struct Layout<AERO_DT_F32> {
    static constexpr int kVals = 16;
    static constexpr int kWords = 4;
    static __host__ __device__ __forceinline__ int chunks(int K) { return K / 16; }
};

// First input index of each run of chunk c (two 16-value runs for Q4_K).
template <int DT>
__device__ __forceinline__ int run0(int c) {
    if (DT == AERO_DT_Q4_K) return (c >> 3) * 256 + ((c & 7) >> 1) * 64 + (c & 1) * 16;
    return c * Layout<DT>::kVals;
}

// A lane's share of one row: its chunks' raw bytes and per-chunk scale data.
template <int DT, int CPL>
struct RowRaw {
    uint4 q[CPL][Layout<DT>::kWords];
    uint4 m[DT == AERO_DT_Q4_K ? CPL : 1];  // Q4_K: header of each chunk's super-block
    uint32_t sc[DT == AERO_DT_Q8_0 ? CPL : 1];  // Q8_0: f16 scale of each chunk's block
};

template <int DT, int LPR, int CPL>
__device__ __forceinline__ void row_load(const QMat& M, int e, int r, int gl, int nch, RowRaw<DT, CPL>& w,
                                         int base = 0) {
    const uint8_t* qs = qm_row_qs(M, e, r);
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = base + gl + LPR * i;
        if (c < nch) {
#pragma unroll
            for (int k = 0; k < Layout<DT>::kWords; ++k) {
                if (DT == AERO_DT_F32)
                    w.q[i][k] = __ldg(reinterpret_cast<const uint4*>(qs + (int64_t)c * 64) + k);
                else
                    w.q[i][k] = ld_stream16(qs + (int64_t)c * 16);
            }
        }
    }
    if (DT == AERO_DT_Q4_K) {
        const uint8_t* mt = qm_row_meta(M, e, r);
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = base + gl + LPR * i;
            if (c < nch) w.m[i] = __ldg(reinterpret_cast<const uint4*>(mt + (int64_t)(c >> 3) * 16));
        }
    } else if (DT == AERO_DT_Q8_0) {
        const unsigned short* mt = reinterpret_cast<const unsigned short*>(qm_row_meta(M, e, r));
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int c = base + gl + LPR * i;
            if (c < nch) w.sc[i] = __ldg(mt + (c >> 1));
        }
    }
}

// The lane's input for its chunks. F32: the values. Q8_0 / Q4_K: per 16-value
// run the two int8 code planes (4 words each), the block scale and the exact
// sum of the run.
template <int DT, int CPL>
struct LaneInput {
    static constexpr int kRuns = DT == AERO_DT_Q4_K ? 2 : 1;
    float v[DT == AERO_DT_F32 ? CPL : 1][DT == AERO_DT_F32 ? 16 : 1];
    uint32_t hi[DT == AERO_DT_F32 ? 1 : CPL][kRuns][4], lo[DT == AERO_DT_F32 ? 1 : CPL][kRuns][4];
    float sx[DT == AERO_DT_F32 ? 1 : CPL][kRuns], s16[DT == AERO_DT_F32 ? 1 : CPL][kRuns];
};

template <int DT, int LPR, int CPL>
__device__ __forceinline__ void input_load(const float* x, const QInput& q, int64_t row, int gl, int nch,
                                           LaneInput<DT, CPL>& in, int base = 0) {
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = base + gl + LPR * i;
        if (c >= nch) continue;
        if (DT == AERO_DT_F32) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                const float4 f = ld_f4(x + row * q.K + run0<DT>(c) + j);
                in.v[i][j] = f.x;
                in.v[i][j + 1] = f.y;
                in.v[i][j + 2] = f.z;
                in.v[i][j + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int r = 0; r < LaneInput<DT, CPL>::kRuns; ++r) {
                const int v0 = run0<DT>(c) + 32 * r;  // first value of the run
                const uint4 h = __ldg(reinterpret_cast<const uint4*>(q.q1 + row * q.K + v0));
                const uint4 l = __ldg(reinterpret_cast<const uint4*>(q.q0 + row * q.K + v0));
                in.hi[i][r][0] = h.x;
                in.hi[i][r][1] = h.y;
                in.hi[i][r][2] = h.z;
                in.hi[i][r][3] = h.w;
                in.lo[i][r][0] = l.x;
                in.lo[i][r][1] = l.y;
                in.lo[i][r][2] = l.z;
                in.lo[i][r][3] = l.w;
                in.sx[i][r] = __ldg(q.sx + row * (q.K / 32) + (v0 >> 5));
                in.s16[i][r] = __ldg(q.s16 + row * (q.K / 16) + (v0 >> 4));
            }
        }
    }
}

// sum over 16 values of code * input code (128 hi + lo), from 4 words of code bytes.
__device__ __forceinline__ int dot16(const uint32_t (&w)[4], const uint32_t (&hi)[4], const uint32_t (&lo)[4]) {
    int a = 0, b = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        a = __dp4a((int)w[k], (int)hi[k], a);
        b = __dp4a((int)w[k], (int)lo[k], b);
    }
    return a * 128 + b;
}

// This lane's part of the row dot.
template <int DT, int LPR, int CPL>
__device__ __forceinline__ float row_dot(const RowRaw<DT, CPL>& w, const LaneInput<DT, CPL>& in, int gl, int nch,
                                         int base = 0) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        const int c = base + gl + LPR * i;
        if (c >= nch) continue;
        const uint32_t raw[4] = {w.q[i][0].x, w.q[i][0].y, w.q[i][0].z, w.q[i][0].w};
        if (DT == AERO_DT_Q4_K) {
            const uint4 m = w.m[i];
            const float d = __half2float(__ushort_as_half((unsigned short)(m.x & 0xFFFFu)));
            const float dmin = __half2float(__ushort_as_half((unsigned short)(m.x >> 16)));
            const int g = (c & 7) >> 1;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                // run r: low (r = 0) or high nibbles of the chunk, sub-block 2g + r
                int sc, mn;
                q4k_sc_m_words(m.y, m.z, m.w, 2 * g + r, sc, mn);
                uint32_t nib[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) nib[k] = (r ? raw[k] >> 4 : raw[k]) & 0x0F0F0F0Fu;
                const int sq = dot16(nib, in.hi[i][r], in.lo[i][r]);
                acc += (d * (float)sc) * in.sx[i][r] * (float)sq - (dmin * (float)mn) * in.s16[i][r];
            }
        } else if (DT == AERO_DT_Q8_0) {
            const int sq = dot16(raw, in.hi[i][0], in.lo[i][0]);
            acc = fmaf(__half2float(__ushort_as_half((unsigned short)w.sc[i])) * in.sx[i][0], (float)sq, acc);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                acc = fmaf(__uint_as_float(w.q[i][k].x), in.v[i][4 * k], acc);
                acc = fmaf(__uint_as_float(w.q[i][k].y), in.v[i][4 * k + 1], acc);
                acc = fmaf(__uint_as_float(w.q[i][k].z), in.v[i][4 * k + 2], acc);
                acc = fmaf(__uint_as_float(w.q[i][k].w), in.v[i][4 * k + 3], acc);
            }
        }
    }
    return acc;
}

template <int LPR>
__device__ __forceinline__ float lanes_sum(float v) {
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace
}  // namespace aero
