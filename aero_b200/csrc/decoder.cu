// The decoder around the MoE layer (include/aero_cuda_decoder.h): one step of
// the reference's block loop (src/model.cpp:234-330, qwen layers) for T tokens,
// each of its own sequence at its own position.
//
// Kernels per layer (all on the decoder's stream):
//   norm_kernel          x (+)= the previous residual term; h = RMSNorm(x, w)
//                        (src/tensor.cpp:128-134), written as f32 rows and/or as
//                        the integer-coded input rows of the GEMVs (QInput)
//   dense_gemv_kernel    y = W h for Q8_0 / Q4_K rows (the fused q|k|v matrix,
//                        the output projection, the head): one warp per row, its
//                        32 lanes splitting the row into 16-byte code chunks,
//                        dp4a over the coded input, f32 accumulation; a CTA takes
//                        up to 16 tokens so a row is read once for all of them
//   qk_rope_kv_kernel    per (token, head): q/k RMSNorm over the head, neox RoPE
//                        (src/transformer.cpp:27-91), k and v stored f16 into the
//                        sequence's cache rows
//   attn_partial_kernel  per (64-position chunk, token, kv head): the chunk's K/V
//                        rows staged in shared memory once for the kv head's
//                        group of query heads, causal scores, chunk softmax
//                        (max, sum) and P V
//   attn_combine_kernel  merges the chunks of each (token, head)
//                        (src/transformer.cpp:120-205 computes the same online
//                        softmax in 1024-position blocks) and codes the head's
//                        values as the output projection's input
//   the MoE layer        aero_cuda_moe_forward on the layer's handle, device
//                        pointers, same stream
// and per step the embedding row gather (Q8_0, the reference's dequantised row,
// src/model.cpp:296-313) and, for the tokens whose logits are asked for, the
// final RMSNorm and the head GEMV.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <set>
#include <tuple>
#include <string>
#include <utility>
#include <vector>

#include "../../include/aero_cuda_decoder.h"
#include "gemv_rows.cuh"
#include "gguf_loader.h"
#include "internal.h"

namespace aero {
namespace {

constexpr int kTokGroup = 16;   // tokens per dense GEMV CTA: a weight row is read once for all of them
// 16-byte chunks per lane per pass over a row (Q4_K chunks carry two runs of input codes)
template <int DT>
__host__ __device__ constexpr int gemv_cpl() { return DT == AERO_DT_Q4_K ? 2 : 4; }
constexpr int kAttnChunk = 64;  // cache positions per attention CTA
constexpr int kMaxGroup = 16;   // query heads per kv head

// Coded input rows (the QInput codes and scales) in the integer tensor-core layout
// of the dense projections: per group of 16 rows and 32-value block, the 16 rows'
// 32 code bytes of the high plane, then of the low plane (a warp's fragment load of
// 8 rows x 32 bytes reads 256 contiguous bytes), and the block's 16 scales sx.
struct QFrag {
    int8_t* q;  // [groups][K / 32][2][16][32]
    float* sx;  // [groups][K / 32][16]
    int K;
};
inline size_t qfrag_bytes(int rows, int K) { return (size_t)((rows + 15) / 16) * (size_t)(K / 32) * (1024 + 64); }
inline QFrag qfrag_at(void* base, int rows, int K) {
    const size_t groups = (size_t)((rows + 15) / 16);
    int8_t* q = static_cast<int8_t*>(base);
    return QFrag{q, reinterpret_cast<float*>(q + groups * (size_t)(K / 32) * 1024), K};
}
// Rows [16 g, ...) onward: the layout of rows starting at a group boundary.
inline QFrag qfrag_from_group(const QFrag& f, int g) {
    if (!f.q) return f;
    const int64_t nb = f.K / 32;
    return QFrag{f.q + (int64_t)g * nb * 1024, f.sx + (int64_t)g * nb * 16, f.K};
}
__device__ __forceinline__ int8_t* qfrag_code(const QFrag& f, int row, int col, int plane) {
    const int64_t nb = f.K / 32;
    return f.q + (((int64_t)(row >> 4) * nb + (col >> 5)) * 2 + plane) * 512 + (row & 15) * 32 + (col & 31);
}
__device__ __forceinline__ float* qfrag_sx(const QFrag& f, int row, int blk) {
    return f.sx + ((int64_t)(row >> 4) * (f.K / 32) + blk) * 16 + (row & 15);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// every group but the most recent N committed by this thread has landed
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// (a, b) as f16 pairs hi = f16(v), lo = f16(v - hi): hi + lo carries v to about 2^-22.
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
    hi = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
    lo = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}
// D (16x8 f32) += A (16x16 f16, row-major fragments a[4]) x B (16x8 f16, b0 / b1)
// Four 8x8 f16 matrices from shared memory (lane i addresses row i % 8 of matrix
// i / 8): r[m] is matrix m's fragment (row g, columns 2 tq, 2 tq + 1), or with TRANS
// its transpose's (rows 2 tq, 2 tq + 1 of column g). Row addresses 16-byte aligned.
template <bool TRANS>
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* row_addr) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(row_addr);
    if (TRANS)
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                     : "r"(a));
    else
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                     : "r"(a));
}

// (not volatile: the compiler may issue later loads ahead of an MMA waiting on its operands)
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------ embedding gather
// x[t] = the Q8_0 row tok[t] dequantised: d * q with one f32 rounding (the
// reference's dequant_ref, src/kernels.cpp:337-350). One thread per 32-value block.
__global__ void embed_q8_kernel(QMat E, const int32_t* __restrict__ tok, int T, float* __restrict__ x) {
    const int d = E.cols, nb = d / 32;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * nb) return;
    const int t = (int)(i / nb), b = (int)(i % nb);
    const int r = tok[t];
    const uint8_t* qs = qm_row_qs(E, 0, r) + 32 * b;
    const float sc =
        __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(qm_row_meta(E, 0, r)) + b)));
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(qs)), c = __ldg(reinterpret_cast<const uint4*>(qs + 16));
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    float4* o = reinterpret_cast<float4*>(x + (int64_t)t * d + 32 * b);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        float4 v;
        v.x = __fmul_rn(sc, (float)(int8_t)(w[k] & 0xFFu));
        v.y = __fmul_rn(sc, (float)(int8_t)((w[k] >> 8) & 0xFFu));
        v.z = __fmul_rn(sc, (float)(int8_t)((w[k] >> 16) & 0xFFu));
        v.w = __fmul_rn(sc, (float)(int8_t)(w[k] >> 24));
        o[k] = v;
    }
}

// ------------------------------------------------------------------ RMSNorm
// Row r0 + b of x (b = blockIdx.x): with add non-null, x += add first (the
// residual, written back); then h = x * inv * w, inv = 1 / sqrt(mean(x^2) + eps)
// (src/tensor.cpp:128-134). Output row b of h32 (f32) and/or of hq (the coded
// GEMV input), either may be null. Thread t holds the 8-value groups t, t + 256,
// ... (all loads issued at once); the four threads of a 32-value block code it
// together (max and 16-value sums by shuffles within the quad). d <= 8192.
constexpr int kNormGroups = 4;  // 8-value groups per thread at most: d <= 4 * 256 * 8
template <int NG>
__global__ void __launch_bounds__(256) norm_kernel(float* __restrict__ x, int d, const float* __restrict__ add,
                                                   const float* __restrict__ w, float eps, int r0,
                                                   float* __restrict__ h32, QInput hq, QFrag hf) {
    __shared__ float red[8];
    const int t = r0 + (int)blockIdx.x, o = (int)blockIdx.x;
    const int ng = d / 8;
    float* xr = x + (int64_t)t * d;
    float v[NG][8], wv[NG][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        const int g = threadIdx.x + 256 * k;
        if (g < ng) {
            float4 a0 = *reinterpret_cast<const float4*>(xr + 8 * g), a1 = *reinterpret_cast<const float4*>(xr + 8 * g + 4);
            const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + 8 * g)),
                         w1 = __ldg(reinterpret_cast<const float4*>(w + 8 * g + 4));
            if (add) {
                const float4 b0 = *reinterpret_cast<const float4*>(add + (int64_t)t * d + 8 * g),
                             b1 = *reinterpret_cast<const float4*>(add + (int64_t)t * d + 8 * g + 4);
                a0.x += b0.x, a0.y += b0.y, a0.z += b0.z, a0.w += b0.w;
                a1.x += b1.x, a1.y += b1.y, a1.z += b1.z, a1.w += b1.w;
                *reinterpret_cast<float4*>(xr + 8 * g) = a0;
                *reinterpret_cast<float4*>(xr + 8 * g + 4) = a1;
            }
            const float vv[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                v[k][i] = vv[i];
                wv[k][i] = ww[i];
                ss = fmaf(vv[i], vv[i], ss);
            }
        }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = 1.0f / sqrtf(tot / (float)d + eps);
    const int q = threadIdx.x & 3;  // this thread's quarter of its 32-value blocks
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        const int g = threadIdx.x + 256 * k;
        const bool on = g < ng;
        float h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = on ? v[k][i] * inv * wv[k][i] : 0.f;
        if (on && h32) {
            float* hp = h32 + (int64_t)o * d + 8 * g;
            *reinterpret_cast<float4*>(hp) = make_float4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<float4*>(hp + 4) = make_float4(h[4], h[5], h[6], h[7]);
        }
        if (!hq.q1) continue;
        float mx = 0.f, sum8 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            mx = fmaxf(mx, fabsf(h[i]));
            sum8 += h[i];
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float s16 = sum8 + __shfl_xor_sync(0xffffffffu, sum8, 1);
        if (!on) continue;
        const float cinv = mx > 0.f ? 16383.0f / mx : 0.f;
        uint32_t p1[2] = {0u, 0u}, p0[2] = {0u, 0u};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int c = __float2int_rn(h[i] * cinv);  // |c| <= 16383
            p1[i >> 2] |= (uint32_t)(c >> 7 & 0xFF) << (8 * (i & 3));
            p0[i >> 2] |= (uint32_t)(c & 127) << (8 * (i & 3));
        }
        const int64_t col = 8 * (int64_t)g;
        *reinterpret_cast<uint2*>(hq.q1 + (int64_t)o * hq.K + col) = make_uint2(p1[0], p1[1]);
        *reinterpret_cast<uint2*>(hq.q0 + (int64_t)o * hq.K + col) = make_uint2(p0[0], p0[1]);
        if (q == 0) hq.sx[(int64_t)o * (hq.K / 32) + (col >> 5)] = mx / 16383.0f;
        if (hf.q) {
            *reinterpret_cast<uint2*>(qfrag_code(hf, o, (int)col, 0)) = make_uint2(p1[0], p1[1]);
            *reinterpret_cast<uint2*>(qfrag_code(hf, o, (int)col, 1)) = make_uint2(p0[0], p0[1]);
            if (q == 0) *qfrag_sx(hf, o, (int)(col >> 5)) = mx / 16383.0f;
        }
        if ((q & 1) == 0) hq.s16[(int64_t)o * (hq.K / 16) + (col >> 4)] = s16;
    }
}

cudaError_t launch_norm(float* x, int T, int d, const float* add, const float* w, float eps, float* h32, QInput hq,
                        QFrag hf, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const int ng = (d / 8 + 255) / 256;
    if (ng <= 1)
        norm_kernel<1><<<(unsigned)T, 256, 0, s>>>(x, d, add, w, eps, 0, h32, hq, hf);
    else if (ng == 2)
        norm_kernel<2><<<(unsigned)T, 256, 0, s>>>(x, d, add, w, eps, 0, h32, hq, hf);
    else
        norm_kernel<kNormGroups><<<(unsigned)T, 256, 0, s>>>(x, d, add, w, eps, 0, h32, hq, hf);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ dense GEMV
// y[t][r] = W[r] . in[t] for the tokens t0 + [0, 16) of blockIdx.y. One warp per
// row at a time (rows blockIdx.x * 8 + warp, stepping over the grid); a row is
// loaded once per pass of 32 x gemv_cpl chunks and dotted with every token of the
// CTA. ONE: a single token whose row fits one pass: its input stays in
// registers and the next row's chunks are prefetched while the current one is
// reduced.
template <int DT, bool ONE>
__global__ void __launch_bounds__(256, 2) dense_gemv_kernel(QMat W, QInput in, int T, float* __restrict__ y,
                                                            int ldy) {
    constexpr int CPL = gemv_cpl<DT>(), LPR = 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = Layout<DT>::chunks(W.cols);
    const int t0 = (int)blockIdx.y * kTokGroup;
    const int nt = min(kTokGroup, T - t0);
    const int stride = (int)gridDim.x * 8;
    int r = (int)blockIdx.x * 8 + warp;
    if (ONE) {
        LaneInput<DT, CPL> xin;
        input_load<DT, LPR, CPL>(nullptr, in, t0, lane, nch, xin);
        RowRaw<DT, CPL> w{}, nx{};
        if (r < W.rows) row_load<DT, LPR, CPL>(W, 0, r, lane, nch, w);
        for (; r < W.rows; r += stride) {
            if (r + stride < W.rows) row_load<DT, LPR, CPL>(W, 0, r + stride, lane, nch, nx);
            const float v = warp_sum(row_dot<DT, LPR, CPL>(w, xin, lane, nch));
            if (lane == 0) y[(int64_t)t0 * ldy + r] = v;
            w = nx;
        }
        return;
    }
    // several tokens: one copy of the dot in the code (a loop over the tokens, not
    // unrolled: the kernel body stays small), each token's sum reduced across the
    // warp at once and kept by lane 0 in shared memory across the row's passes
    __shared__ float acc_s[8][kTokGroup];
    for (; r < W.rows; r += stride) {
        for (int base = 0; base < nch; base += LPR * CPL) {
            RowRaw<DT, CPL> w;
            row_load<DT, LPR, CPL>(W, 0, r, lane, nch, w, base);
#pragma unroll 1
            for (int j = 0; j < nt; ++j) {
                LaneInput<DT, CPL> xin;
                input_load<DT, LPR, CPL>(nullptr, in, t0 + j, lane, nch, xin, base);
                const float v = warp_sum(row_dot<DT, LPR, CPL>(w, xin, lane, nch, base));
                if (lane == 0) acc_s[warp][j] = base == 0 ? v : acc_s[warp][j] + v;
            }
        }
        if (lane < nt) y[(int64_t)(t0 + lane) * ldy + r] = acc_s[warp][lane];
        __syncwarp();
    }
}

// ------------------------------------------- dense Q8_0 rows x tokens, tensor cores
// y[t][r] = W[r] . in[t] for Q8_0 rows and 2..16 tokens of blockIdx.y's group: the
// same integer sums as the row dots above, on the tensor cores. Per 32-value block
// (one Q8_0 scale d, one input scale sx) the block's codes give two integer MMAs
// (m16n8k32, s8 x s8 -> s32): the weight codes against the input's high and low
// code planes, 128 hi + lo exactly in int32, then d sx times that in f32. A CTA
// owns 16 rows; its 8 warps take every 8th block of K (tensor-core A: the 16 rows,
// B: 8 tokens per tile) and their partial sums meet in shared memory in warp order.
// Thread (g, q) of a warp loads bytes [8 q, 8 q + 8) of a block for row g and row
// g + 8 (one 8-byte load each) and the same bytes of token g's codes: the MMA sums
// over k, so one permutation of k applied to both operands (the fragment's k
// positions 4q..4q+3 and 16+4q..16+4q+3 read bytes 8q..8q+7) leaves the sums
// unchanged.
constexpr int kMmaWarps = 8;

// Neither asm is volatile: the weights are read-only for the launch, and the
// compiler may then issue the loads of later blocks ahead of the MMAs that wait.
__device__ __forceinline__ uint2 ld_stream8(const void* p) {
    uint2 v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

template <int NT>  // 8-token tiles per CTA (1: up to 8 tokens, 2: up to 16)
__global__ void __launch_bounds__(256) dense_mma_q8_kernel(QMat W, QFrag in, int T, float* __restrict__ y, int ldy) {
    constexpr int U = 4;  // blocks whose loads are issued together
    __shared__ float red[kMmaWarps][16][16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q = lane & 3;
    const int r0 = (int)blockIdx.x * 16, t0 = (int)blockIdx.y * 16;
    const int nt = min(16, T - t0);
    const int nblk = W.cols / 32;
    // rows past the matrix read its last row and are not stored
    const int ra = min(r0 + g, W.rows - 1), rb = min(r0 + g + 8, W.rows - 1);
    const uint8_t* qa = W.qs + (int64_t)ra * W.cols + 8 * q;
    const uint8_t* qb = W.qs + (int64_t)rb * W.cols + 8 * q;
    const unsigned short* ma = reinterpret_cast<const unsigned short*>(W.meta + (int64_t)ra * nblk * 2);
    const unsigned short* mb = reinterpret_cast<const unsigned short*>(W.meta + (int64_t)rb * nblk * 2);
    // this thread's B token (8 j + g) and accumulator tokens (8 j + 2 q, + 1) per
    // tile, in the group's tensor-core layout (t0 is a multiple of 16); products of
    // tokens past the call's are computed on stale codes and never stored
    const int64_t grp = t0 >> 4;
    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    // warp w takes the contiguous blocks [w nper, (w + 1) nper) (nper a multiple of U),
    // U at a time: the U scales of a row are one 8-byte load (nblk is a multiple of U)
    const int nper = ((nblk + kMmaWarps - 1) / kMmaWarps + U - 1) / U * U;
    const int bend = min(nblk, (warp + 1) * nper);
    for (int b0 = warp * nper; b0 < bend; b0 += U) {
        uint2 wa[U], wb[U], h[U][NT], l[U][NT];
        float s0[U][NT], s1[U][NT];
        const uint2 sa4 = __ldg(reinterpret_cast<const uint2*>(ma + b0)), sb4 = __ldg(reinterpret_cast<const uint2*>(mb + b0));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int b = b0 + u;  // < nblk: b0 + U <= nblk
            wa[u] = ld_stream8(qa + (int64_t)b * 32);
            wb[u] = ld_stream8(qb + (int64_t)b * 32);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                const int8_t* f = in.q + ((grp * nblk + b) * 2) * 512 + (8 * j + g) * 32 + 8 * q;
                h[u][j] = *reinterpret_cast<const uint2*>(f);
                l[u][j] = *reinterpret_cast<const uint2*>(f + 512);
                const float2 sv = *reinterpret_cast<const float2*>(in.sx + (grp * nblk + b) * 16 + 8 * j + 2 * q);
                s0[u][j] = sv.x;
                s1[u][j] = sv.y;
            }
        }
        const uint32_t sav[2] = {sa4.x, sa4.y}, sbv[2] = {sb4.x, sb4.y};
#pragma unroll
        for (int u = 0; u < U; ++u) {
            if (b0 + u >= bend) break;
            const uint32_t A[4] = {wa[u].x, wb[u].x, wa[u].y, wb[u].y};
            const float da = __half2float(__ushort_as_half((unsigned short)(sav[u >> 1] >> (16 * (u & 1)))));
            const float db = __half2float(__ushort_as_half((unsigned short)(sbv[u >> 1] >> (16 * (u & 1)))));
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                int ch[4], cl[4];
                mma_s8(ch, A, h[u][j].x, h[u][j].y);
                mma_s8(cl, A, l[u][j].x, l[u][j].y);
                acc[j][0] = fmaf((float)(128 * ch[0] + cl[0]), da * s0[u][j], acc[j][0]);
                acc[j][1] = fmaf((float)(128 * ch[1] + cl[1]), da * s1[u][j], acc[j][1]);
                acc[j][2] = fmaf((float)(128 * ch[2] + cl[2]), db * s0[u][j], acc[j][2]);
                acc[j][3] = fmaf((float)(128 * ch[3] + cl[3]), db * s1[u][j], acc[j][3]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int tc = 8 * j + 2 * q;
        red[warp][g][tc] = acc[j][0];
        red[warp][g][tc + 1] = acc[j][1];
        red[warp][g + 8][tc] = acc[j][2];
        red[warp][g + 8][tc + 1] = acc[j][3];
    }
    __syncthreads();
    const int row = threadIdx.x >> 4, tk = threadIdx.x & 15;
    if (tk < nt && tk < 8 * NT && r0 + row < W.rows) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) v += red[w][row][tk];
        y[(int64_t)(t0 + tk) * ldy + r0 + row] = v;
    }
}

// One token over rows of up to two passes (32 x gemv_cpl chunks each): a CTA takes 4
// rows, two warps per row, each with its half's input in registers and its half of the
// row; the halves are added in order (first, then second) in shared memory.
template <int DT>
__global__ void __launch_bounds__(256) dense_gemv_split_kernel(QMat W, QInput in, float* __restrict__ y) {
    constexpr int CPL = gemv_cpl<DT>(), LPR = 32;
    __shared__ float part[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = Layout<DT>::chunks(W.cols);
    const int r = (int)blockIdx.x * 4 + (warp >> 1), base = (warp & 1) * LPR * CPL;
    float v = 0.f;
    if (r < W.rows) {
        LaneInput<DT, CPL> xin;
        input_load<DT, LPR, CPL>(nullptr, in, 0, lane, nch, xin, base);
        RowRaw<DT, CPL> w{};
        row_load<DT, LPR, CPL>(W, 0, r, lane, nch, w, base);
        v = warp_sum(row_dot<DT, LPR, CPL>(w, xin, lane, nch, base));
    }
    if (lane == 0) part[warp] = v;
    __syncthreads();
    if (threadIdx.x < 4) {
        const int rr = (int)blockIdx.x * 4 + (int)threadIdx.x;
        if (rr < W.rows) y[rr] = part[2 * threadIdx.x] + part[2 * threadIdx.x + 1];
    }
}

// ---------------------------------------------------- q/k norm, RoPE, cache
// One warp per (token, head j) of the step's q|k|v rows (j < H: query head,
// then H_kv key heads, then H_kv value heads); lane l holds values i * 32 + l,
// so the neox pairs (p, p + D/2) are lane-local. Queries are written back f32,
// keys and values f16 into the cache row (seq, head, pos).
template <int NV>
__global__ void __launch_bounds__(128) qk_rope_kv_kernel(float* __restrict__ qkv, int T, int H, int HK, int ld,
                                                         const float* __restrict__ q_norm,
                                                         const float* __restrict__ k_norm, float eps, float rope_base,
                                                         const int64_t* __restrict__ pos,
                                                         const int32_t* __restrict__ seq, __half* __restrict__ kc,
                                                         __half* __restrict__ vc, int n_ctx) {
    constexpr int D = NV * 32, HV = NV / 2;
    const int item = (int)blockIdx.x * 4 + (int)(threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int per = H + 2 * HK;
    if (item >= T * per) return;
    const int t = item / per, j = item % per;
    float* src = qkv + (int64_t)t * ld + (int64_t)j * D;
    float v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = src[i * 32 + lane];
    const int64_t p = pos[t];
    if (j < H + HK) {
        const float* w = j < H ? q_norm : k_norm;
        if (w) {
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < NV; ++i) ss = fmaf(v[i], v[i], ss);
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = v[i] * inv * w[i * 32 + lane];
        }
#pragma unroll
        for (int i = 0; i < HV; ++i) {
            const int pi = i * 32 + lane;
            const float e = (float)pi * 2.0f / (float)D;
            const float invf = 1.0f / powf(rope_base, e);
            const float ang = (float)p * invf;
            const float c = cosf(ang), s = sinf(ang);
            const float x0 = v[i], x1 = v[i + HV];
            v[i] = x0 * c - x1 * s;
            v[i + HV] = x0 * s + x1 * c;
        }
    }
    if (j < H) {
#pragma unroll
        for (int i = 0; i < NV; ++i) src[i * 32 + lane] = v[i];
        return;
    }
    const bool is_k = j < H + HK;
    const int hk = is_k ? j - H : j - H - HK;
    __half* dst = (is_k ? kc : vc) + (((int64_t)seq[t] * HK + hk) * n_ctx + p) * D;
#pragma unroll
    for (int i = 0; i < NV; ++i) dst[i * 32 + lane] = __float2half_rn(v[i]);
}

// The A fragment (m16n8k16, row-major 16 x 16) of rows g, g + 8 (zero at or past
// `rows`) and columns c0 + 2 tq, + 1, + 8, + 9 of an f32 matrix with row stride ld,
// split into f16 hi and lo halves: written as two uint4 (hi a0..a3, lo a0..a3).
__device__ __forceinline__ void make_a_frag(const float* m, int ld, int rows, int c0, int lane, uint4* dst) {
    const int g = lane >> 2, tq = lane & 3, col = c0 + 2 * tq;
    const bool r0 = g < rows, r1 = g + 8 < rows;
    const float* m0 = m + g * ld;
    const float* m1 = m + (g + 8) * ld;
    uint32_t h[4], l[4];
    split_pair(r0 ? m0[col] : 0.f, r0 ? m0[col + 1] : 0.f, h[0], l[0]);
    split_pair(r1 ? m1[col] : 0.f, r1 ? m1[col + 1] : 0.f, h[1], l[1]);
    split_pair(r0 ? m0[col + 8] : 0.f, r0 ? m0[col + 9] : 0.f, h[2], l[2]);
    split_pair(r1 ? m1[col + 8] : 0.f, r1 ? m1[col + 9] : 0.f, h[3], l[3]);
    dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
    dst[1] = make_uint4(l[0], l[1], l[2], l[3]);
}

// ------------------------------------------------------------------ attention
// CTA = (nch consecutive chunks of 64 positions, token t, kv head hk): each
// chunk's K and V rows of (seq[t], hk) staged in shared memory by asynchronous
// copies, two buffers so the next chunk's copies fly while this one is computed
// (rows padded to an odd number of 16-byte units; the queries and their MMA
// fragments made once per CTA), per chunk the scores of the group's R <= 16
// query heads for positions <= pos[t] (masked to -inf otherwise, scaled by
// 1/sqrt(D)) and P V as warp-level tensor-core MMAs (m16n8k16, f16 operands with
// the f32 queries and probabilities split into hi + lo halves, f32 accumulation),
// the chunk's max m and sum l of exp(s - m) in f32.
// part[t][h][c] = (m, l, -, -, acc[D]) (acc 16-byte aligned).
template <int NV>
__global__ void __launch_bounds__(256) attn_partial_kernel(const float* __restrict__ qkv, int ld, int H, int HK,
                                                           const __half* __restrict__ kc,
                                                           const __half* __restrict__ vc, int n_ctx,
                                                           const int64_t* __restrict__ pos,
                                                           const int32_t* __restrict__ seq, float scale,
                                                           float* __restrict__ part, int n_chunk, int nch) {
    constexpr int D = NV * 32;
    constexpr int KS = D * 2 + 16;
    constexpr int C = kAttnChunk;
    const int t = (int)blockIdx.y / HK, hk = (int)blockIdx.y % HK;
    const int64_t qp = pos[t];
    const int c0 = (int)blockIdx.x * nch;
    if ((int64_t)c0 * C > qp) return;
    const int c1 = (int)min((int64_t)min(n_chunk, c0 + nch), qp / C + 1);  // chunks [c0, c1) hold positions <= qp
    const int R = H / HK;
    extern __shared__ __align__(16) uint8_t sm[];
    uint8_t* kbuf = sm;                    // [2][C][KS]
    uint8_t* vbuf = kbuf + 2 * C * KS;     // [2][C][KS]
    float* qs = reinterpret_cast<float*>(vbuf + 2 * C * KS);
    float* S = qs + R * D;
    // the MMAs' A fragments (every warp uses the same ones): per 16-column step and
    // lane, the four f16x2 registers of hi then of lo
    uint4* qa = reinterpret_cast<uint4*>(S + R * C);  // [D / 16][32][2]
    uint4* pa = qa + (D / 16) * 64;                   // [C / 16][32][2]
    // running max and sum of each head over the CTA's chunks, and the chunk's
    // rescale factors (old sums, this chunk's) for the accumulators
    float* mrun = reinterpret_cast<float*>(pa + (C / 16) * 64);  // [R]
    float* lrun = mrun + kMaxGroup;                              // [R]
    float2* fac = reinterpret_cast<float2*>(lrun + kMaxGroup);   // [R]
    const int64_t sbase = ((int64_t)seq[t] * HK + hk) * n_ctx;
    // chunk c's rows into buffer b, copied asynchronously (one commit group per
    // chunk and thread); rows past the query's position are zeroed
    constexpr int pieces = D / 8;
    auto stage = [&](int c, int b) {
        const int nvc = (int)min((int64_t)C, qp - (int64_t)c * C + 1);
        const int64_t base = (sbase + (int64_t)c * C) * D;
        uint8_t* ks = kbuf + b * C * KS;
        uint8_t* vs = vbuf + b * C * KS;
        for (int i = threadIdx.x; i < nvc * pieces; i += blockDim.x) {
            const int row = i / pieces, pc = i % pieces;
            cp_async16(ks + row * KS + pc * 16, kc + base + (int64_t)row * D + pc * 8);
            cp_async16(vs + row * KS + pc * 16, vc + base + (int64_t)row * D + pc * 8);
        }
        for (int i = threadIdx.x; i < (C - nvc) * pieces; i += blockDim.x) {
            const int row = nvc + i / pieces, pc = i % pieces;
            *reinterpret_cast<uint4*>(ks + row * KS + pc * 16) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(vs + row * KS + pc * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        cp_async_commit();
    };
    stage(c0, 0);
    for (int i = threadIdx.x; i < R * D; i += blockDim.x)
        qs[i] = qkv[(int64_t)t * ld + (int64_t)(hk * R) * D + i];
    if (threadIdx.x < R) {
        mrun[threadIdx.x] = -INFINITY;
        lrun[threadIdx.x] = 0.f;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, tq = lane & 3;  // the MMA fragments' row group and column pair
    for (int kk = warp; kk < D / 16; kk += 8) make_a_frag(qs, D, R, kk * 16, lane, qa + (kk * 32 + lane) * 2);
    __syncthreads();
    // heads of up to 128 values keep the query fragments in registers for every chunk
    // (a warp reads them from shared memory once instead of once per chunk)
    constexpr bool kQReg = NV <= 4;
    uint4 qf[kQReg ? D / 16 : 1][2];
    if constexpr (kQReg) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            qf[kk][0] = qa[(kk * 32 + lane) * 2];
            qf[kk][1] = qa[(kk * 32 + lane) * 2 + 1];
        }
    }
    // the P V accumulators of this thread's tiles (heads g, g + 8), merged over the chunks
    constexpr int NT = D / 64;
    float accr[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) accr[i][0] = accr[i][1] = accr[i][2] = accr[i][3] = 0.f;
    for (int c = c0; c < c1; ++c) {
    const int cb = (c - c0) & 1;
    if (c + 1 < c1) {
        stage(c + 1, cb ^ 1);  // the other buffer's chunk was finished before the last barrier
        cp_async_wait_group<1>();
    } else {
        cp_async_wait_group<0>();
    }
    __syncthreads();
    const uint8_t* ks = kbuf + cb * C * KS;
    const uint8_t* vs = vbuf + cb * C * KS;
    const int nv = (int)min((int64_t)C, qp - (int64_t)c * C + 1);
    // scores on the tensor cores: S (query heads x positions) = Q K^T with Q split
    // into f16 hi + lo parts (two MMAs per 16 dims, f32 accumulation; K is f16 as
    // cached); warp w takes positions 8w .. 8w + 7, heads beyond R are zero rows
    {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        // lane i addresses position 8 warp + i % 8, dims 32 kp + 8 (i / 8): two k-steps per load
        const uint8_t* kr = ks + (8 * warp + (lane & 7)) * KS + (lane >> 3) * 16;
        const bool r0 = g < R, r1 = g + 8 < R;
#pragma unroll
        for (int kp = 0; kp < D / 32; ++kp) {
            uint32_t b[4];
            ldsm_x4<false>(b, kr + kp * 64);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int kk = 2 * kp + h;
                uint4 fh, fl;
                if constexpr (kQReg) {
                    fh = qf[kk][0];
                    fl = qf[kk][1];
                } else {
                    fh = qa[(kk * 32 + lane) * 2];
                    fl = qa[(kk * 32 + lane) * 2 + 1];
                }
                const uint32_t ah[4] = {fh.x, fh.y, fh.z, fh.w}, al[4] = {fl.x, fl.y, fl.z, fl.w};
                mma_f16(acc, ah, b[2 * h], b[2 * h + 1]);
                mma_f16(acc, al, b[2 * h], b[2 * h + 1]);
            }
        }
        const int j = 8 * warp + 2 * tq;
        if (r0) {
            S[g * C + j] = j < nv ? acc[0] * scale : -INFINITY;
            S[g * C + j + 1] = j + 1 < nv ? acc[1] * scale : -INFINITY;
        }
        if (r1) {
            S[(g + 8) * C + j] = j < nv ? acc[2] * scale : -INFINITY;
            S[(g + 8) * C + j + 1] = j + 1 < nv ? acc[3] * scale : -INFINITY;
        }
    }
    __syncthreads();
    for (int r = warp; r < R; r += 8) {
        const float s0 = S[r * C + lane], s1 = S[r * C + lane + 32];
        const float m = warp_max(fmaxf(s0, s1));  // finite: position start is always kept
        const float p0 = lane < nv ? expf(s0 - m) : 0.f;
        const float p1 = lane + 32 < nv ? expf(s1 - m) : 0.f;
        S[r * C + lane] = p0;
        S[r * C + lane + 32] = p1;
        const float l = warp_sum(p0 + p1);
        if (lane == 0) {
            // online merge with the CTA's earlier chunks (src/transformer.cpp:120-205
            // merges its 1024-position blocks the same way)
            const float mo = mrun[r], mn = fmaxf(mo, m);
            const float alpha = expf(mo - mn), beta = expf(m - mn);
            lrun[r] = alpha * lrun[r] + beta * l;
            mrun[r] = mn;
            fac[r] = make_float2(alpha, beta);
        }
    }
    __syncthreads();
    for (int kk = warp; kk < C / 16; kk += 8) make_a_frag(S, C, R, kk * 16, lane, pa + (kk * 32 + lane) * 2);
    __syncthreads();
    // P V on the tensor cores: (heads x dims) = P (heads x positions, f16 hi + lo)
    // times V (positions x dims, f16); warp w takes dims 8 nt .. 8 nt + 7 for
    // nt = w, w + 8, ...; positions past nv have P = 0 and zeroed V rows
    {
        // warp w takes the D / 64 tiles of 8 dims nt = w, w + 8, ..., all in one pass
        // over the P fragments (read once per warp)
        float acc[NT][4];
#pragma unroll
        for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        const bool r0 = g < R, r1 = g + 8 < R;
#pragma unroll
        for (int kp = 0; kp < C / 32; ++kp) {
            uint4 fh[2], fl[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                fh[h] = pa[((2 * kp + h) * 32 + lane) * 2];
                fl[h] = pa[((2 * kp + h) * 32 + lane) * 2 + 1];
            }
#pragma unroll
            for (int i = 0; i < NT; ++i) {
                const int nt = warp + 8 * i;
                // lane l addresses position 32 kp + l, dims 8 nt .. 8 nt + 7 (transposed: two k-steps)
                uint32_t b[4];
                ldsm_x4<true>(b, vs + (kp * 32 + lane) * KS + nt * 16);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t ah[4] = {fh[h].x, fh[h].y, fh[h].z, fh[h].w};
                    const uint32_t al[4] = {fl[h].x, fl[h].y, fl[h].z, fl[h].w};
                    mma_f16(acc[i], ah, b[2 * h], b[2 * h + 1]);
                    mma_f16(acc[i], al, b[2 * h], b[2 * h + 1]);
                }
            }
        }
        const float2 fa = r0 ? fac[g] : make_float2(0.f, 0.f), fb = r1 ? fac[g + 8] : make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < NT; ++i) {
            accr[i][0] = fmaf(fa.x, accr[i][0], fa.y * acc[i][0]);
            accr[i][1] = fmaf(fa.x, accr[i][1], fa.y * acc[i][1]);
            accr[i][2] = fmaf(fb.x, accr[i][2], fb.y * acc[i][2]);
            accr[i][3] = fmaf(fb.x, accr[i][3], fb.y * acc[i][3]);
        }
    }
    __syncthreads();  // the buffers, the scores, the P fragments and the factors are reused
    }
    // the CTA's merged partial: part[t][h][blockIdx.x] = (m, l, -, -, acc[D])
    const bool r0 = g < R, r1 = g + 8 < R;
    float* outp = part + (((int64_t)t * H + (int64_t)hk * R) * n_chunk + blockIdx.x) * (D + 4);
    if (threadIdx.x < R) {
        float* op = outp + (int64_t)threadIdx.x * n_chunk * (D + 4);
        op[0] = mrun[threadIdx.x];
        op[1] = lrun[threadIdx.x];
    }
#pragma unroll
    for (int i = 0; i < NT; ++i) {
        const int col = 4 + (warp + 8 * i) * 8 + 2 * tq;
        if (r0) {
            float* op = outp + (int64_t)g * n_chunk * (D + 4);
            op[col] = accr[i][0];
            op[col + 1] = accr[i][1];
        }
        if (r1) {
            float* op = outp + (int64_t)(g + 8) * n_chunk * (D + 4);
            op[col] = accr[i][2];
            op[col + 1] = accr[i][3];
        }
    }
}

// CTA = (token, head), kCombThreads threads: out = sum_c e^(m_c - M) acc_c / sum_c e^(m_c - M) l_c
// over the head's partials c (one per group of nch chunks). The partials' (m, l) are read
// in parallel (one partial per thread, block max and sum); then warp w adds the acc
// rows of partials w, w + kCombWarps, ... (float4 per lane) and the warps' sums meet in
// shared memory.
constexpr int kCombWarps = 8;
constexpr int kCombThreads = 32 * kCombWarps;
__global__ void __launch_bounds__(kCombThreads) attn_combine_kernel(const float* __restrict__ part, int H, int D,
                                                                    int n_chunk, int nch,
                                                                    const int64_t* __restrict__ pos,
                                                                    float* __restrict__ att, QInput aq, QFrag af) {
    __shared__ float ew[1024];  // e^(m_c - M), partial c (n_chunk <= 1024)
    __shared__ float red[kCombWarps];
    __shared__ float4 accs[kCombWarps][64];
    const int t = (int)blockIdx.x / H, h = (int)blockIdx.x % H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nc = (int)(pos[t] / kAttnChunk) / nch + 1;  // the partials: one per group of nch chunks
    const float* pb = part + ((int64_t)t * H + h) * n_chunk * (D + 4);
    float m = -INFINITY;
    for (int c = threadIdx.x; c < nc; c += kCombThreads) m = fmaxf(m, pb[(int64_t)c * (D + 4)]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    float M = red[0];
#pragma unroll
    for (int w = 1; w < kCombWarps; ++w) M = fmaxf(M, red[w]);
    __syncthreads();
    float L = 0.f;
    for (int c = threadIdx.x; c < nc; c += kCombThreads) {
        const float e = expf(pb[(int64_t)c * (D + 4)] - M);
        ew[c] = e;
        L = fmaf(e, pb[(int64_t)c * (D + 4) + 1], L);
    }
    L = warp_sum(L);
    if (lane == 0) red[warp] = L;
    __syncthreads();
    float Ls = 0.f;
#pragma unroll
    for (int w = 0; w < kCombWarps; ++w) Ls += red[w];
    const int nq = D / 4;  // float4 per acc row (<= 64)
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = lane; q < nq; q += 32) {
        a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = warp; c < nc; c += kCombWarps) {
            const float e = ew[c];
            const float4 v = *reinterpret_cast<const float4*>(pb + (int64_t)c * (D + 4) + 4 + 4 * q);
            a.x = fmaf(e, v.x, a.x);
            a.y = fmaf(e, v.y, a.y);
            a.z = fmaf(e, v.z, a.z);
            a.w = fmaf(e, v.w, a.w);
        }
        accs[warp][q] = a;
    }
    __syncthreads();
    const float inv = 1.0f / fmaxf(Ls, 1e-30f);
    for (int q = threadIdx.x; q < nq; q += kCombThreads) {
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kCombWarps; ++w) {
            const float4 aw = accs[w][q];
            o.x += aw.x, o.y += aw.y, o.z += aw.z, o.w += aw.w;
        }
        o.x *= inv, o.y *= inv, o.z *= inv, o.w *= inv;
        *reinterpret_cast<float4*>(att + ((int64_t)t * H + h) * D + 4 * q) = o;
        accs[0][q] = o;
    }
    // the head's D values coded as the output projection's input (row t, columns h * D ...)
    __syncthreads();
    if (threadIdx.x < D / 32) {
        const int b = threadIdx.x, c = h * D + 32 * b;
        qinput_block(reinterpret_cast<const float*>(&accs[0][0]) + 32 * b, aq.q1 + (int64_t)t * aq.K + c,
                     aq.q0 + (int64_t)t * aq.K + c, aq.sx + (int64_t)t * (aq.K / 32) + (c >> 5),
                     aq.s16 + (int64_t)t * (aq.K / 16) + (c >> 4));
        if (af.q) {
            // the block this thread just coded, copied into the tensor-core layout
            const uint4* h1 = reinterpret_cast<const uint4*>(aq.q1 + (int64_t)t * aq.K + c);
            const uint4* h0 = reinterpret_cast<const uint4*>(aq.q0 + (int64_t)t * aq.K + c);
            uint4* f1 = reinterpret_cast<uint4*>(qfrag_code(af, t, c, 0));
            uint4* f0 = reinterpret_cast<uint4*>(qfrag_code(af, t, c, 1));
            f1[0] = h1[0], f1[1] = h1[1], f0[0] = h0[0], f0[1] = h0[1];
            *qfrag_sx(af, t, c >> 5) = aq.sx[(int64_t)t * (aq.K / 32) + (c >> 5)];
        }
    }
}

// ------------------------------------------------------------------ launchers
template <int DT>
cudaError_t gemv_dense_dt(const QMat& W, const QInput& in, const QFrag& fr, int T, float* y, int ldy, int n_sm,
                          cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const int nch = Layout<DT>::chunks(W.cols);
    const dim3 grid((unsigned)std::max(1, std::min((W.rows + 7) / 8, n_sm * 4)), (unsigned)((T + kTokGroup - 1) / kTokGroup));
    if (DT == AERO_DT_Q8_0 && T >= 2 && fr.q && W.cols % 128 == 0 && fr.K == W.cols) {
        // several tokens: the integer tensor-core form (a CTA per 16 rows)
        const dim3 mg((unsigned)((W.rows + 15) / 16), (unsigned)((T + kTokGroup - 1) / kTokGroup));
        if (T <= 8)
            dense_mma_q8_kernel<1><<<mg, 256, 0, s>>>(W, fr, T, y, ldy);
        else
            dense_mma_q8_kernel<2><<<mg, 256, 0, s>>>(W, fr, T, y, ldy);
        return cudaGetLastError();
    }
    if (T == 1 && nch > 32 * gemv_cpl<DT>() && nch <= 64 * gemv_cpl<DT>()) {
        dense_gemv_split_kernel<DT><<<(unsigned)((W.rows + 3) / 4), 256, 0, s>>>(W, in, y);
        return cudaGetLastError();
    }
    if (T == 1 && nch <= 32 * gemv_cpl<DT>())
        dense_gemv_kernel<DT, true><<<grid, 256, 0, s>>>(W, in, T, y, ldy);
    else
        dense_gemv_kernel<DT, false><<<grid, 256, 0, s>>>(W, in, T, y, ldy);
    return cudaGetLastError();
}

// fr: the same input rows in the tensor-core layout (fr.q null: the CUDA-core form only)
cudaError_t gemv_dense(const QMat& W, const QInput& in, const QFrag& fr, int T, float* y, int ldy, int n_sm,
                       cudaStream_t s) {
    if (W.dtype == AERO_DT_Q8_0) return gemv_dense_dt<AERO_DT_Q8_0>(W, in, fr, T, y, ldy, n_sm, s);
    if (W.dtype == AERO_DT_Q4_K) return gemv_dense_dt<AERO_DT_Q4_K>(W, in, fr, T, y, ldy, n_sm, s);
    return cudaErrorInvalidValue;
}

template <int NV>
size_t attn_smem(int R) {
    // two buffers of K and V rows, the queries, the scores, the A fragments of Q and of
    // P, the running max / sum and rescale factors of the heads
    return (size_t)4 * kAttnChunk * (NV * 64 + 16) + (size_t)R * NV * 32 * 4 + (size_t)R * kAttnChunk * 4 +
           (size_t)(NV * 2) * 32 * 32 + (size_t)(kAttnChunk / 16) * 32 * 32 + (size_t)kMaxGroup * 16;
}

template <int NV>
cudaError_t attention_nv(float* qkv, int ld, int T, int H, int HK, const float* qn, const float* kn, float eps,
                         float base, const int64_t* pos, const int32_t* seq, __half* kc, __half* vc, int n_ctx,
                         float* part, int n_chunk, float* att, QInput aq, QFrag af, cudaStream_t s) {
    const int per = H + 2 * HK;
    qk_rope_kv_kernel<NV><<<(unsigned)((T * per + 3) / 4), 128, 0, s>>>(qkv, T, H, HK, ld, qn, kn, eps, base, pos, seq,
                                                                        kc, vc, n_ctx);
    const int R = H / HK;
    const size_t smem = attn_smem<NV>(R);
    static thread_local size_t smem_set = 0;
    if (smem > 48 * 1024 && smem > smem_set) {
        const cudaError_t e =
            cudaFuncSetAttribute(attn_partial_kernel<NV>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        smem_set = smem;
    }
    const float scale = 1.0f / std::sqrt((float)(NV * 32));
    // chunks per CTA: enough CTAs for about two rounds of two per SM, at most 8 chunks each
    const int n_sm = 148;
    const int nch = std::max(1, std::min(8, (int)(((int64_t)n_chunk * T * HK) / (4 * n_sm))));
    attn_partial_kernel<NV><<<dim3((unsigned)((n_chunk + nch - 1) / nch), (unsigned)(T * HK)), 256, smem, s>>>(
        qkv, ld, H, HK, kc, vc, n_ctx, pos, seq, scale, part, n_chunk, nch);
    attn_combine_kernel<<<(unsigned)(T * H), kCombThreads, 0, s>>>(part, H, NV * 32, n_chunk, nch, pos, att, aq, af);
    return cudaGetLastError();
}

cudaError_t attention(int D, float* qkv, int ld, int T, int H, int HK, const float* qn, const float* kn, float eps,
                      float base, const int64_t* pos, const int32_t* seq, __half* kc, __half* vc, int n_ctx,
                      float* part, int n_chunk, float* att, QInput aq, QFrag af, cudaStream_t s) {
    switch (D) {
        case 64: return attention_nv<2>(qkv, ld, T, H, HK, qn, kn, eps, base, pos, seq, kc, vc, n_ctx, part, n_chunk, att, aq, af, s);
        case 128: return attention_nv<4>(qkv, ld, T, H, HK, qn, kn, eps, base, pos, seq, kc, vc, n_ctx, part, n_chunk, att, aq, af, s);
        case 192: return attention_nv<6>(qkv, ld, T, H, HK, qn, kn, eps, base, pos, seq, kc, vc, n_ctx, part, n_chunk, att, aq, af, s);
        case 256: return attention_nv<8>(qkv, ld, T, H, HK, qn, kn, eps, base, pos, seq, kc, vc, n_ctx, part, n_chunk, att, aq, af, s);
    }
    return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ host side
struct DLayer {
    QMat qkv{}, o{};
    float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    void* moe = nullptr;
    bool own_moe = false;
    __half *kc = nullptr, *vc = nullptr;
};

struct Decoder {
    int device = 0;
    cudaStream_t stream = nullptr, own_stream = nullptr;
    int n_layer = 0, d = 0, H = 0, HK = 0, D = 0, vocab = 0, n_seq = 0, n_ctx = 0, n_chunk = 0, n_sm = 148;
    float eps = 1e-6f, rope_base = 10000.f;
    QMat embd{}, head{};
    float* out_norm = nullptr;
    std::vector<DLayer> L;
    struct Alloc {
        void* p;
        size_t bytes;
        int cls;
    };
    std::vector<Alloc> allocs;
    // step scratch, for up to cap tokens
    int cap = 0;
    void* sbase = nullptr;
    size_t sbytes = 0;
    float *x = nullptr, *h32 = nullptr, *qkv = nullptr, *att = nullptr, *o = nullptr, *dm = nullptr, *part = nullptr,
          *logits = nullptr;
    int32_t *tok = nullptr, *seq = nullptr;
    int64_t* pos = nullptr;
    QInput hq{}, aq{};
    QFrag hf{}, af{};  // hq and aq in the dense projections' tensor-core layout
    std::string err;
    // CUDA graphs of decode steps (T <= kDecodeMaxTokens): keyed by (T, first head
    // row, head rows, logits pointer); a key runs eagerly once (sizing every
    // scratch and setting kernel attributes), is captured on its second call and
    // replayed from then on. Dropped when the decoder's scratch is reallocated or a
    // step larger than any before runs (the MoE layers may then reallocate theirs).
    bool use_graphs = true;
    int max_T = 0;
    std::set<std::tuple<int, int, int, uintptr_t>> seen;
    std::map<std::tuple<int, int, int, uintptr_t>, cudaGraphExec_t> graphs;
    void drop_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
        seen.clear();
    }
    // profiling
    bool prof = false;
    double ms[5] = {};
    std::vector<cudaEvent_t> ev;
    std::vector<int> ev_phase;
    int n_ev = 0;

    bool fail(const char* fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        err = buf;
        return false;
    }
    bool ok(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        cudaGetLastError();
        return fail("%s: %s", what, cudaGetErrorString(e));
    }
    void* alloc(size_t bytes, int cls, const char* what) {
        void* p = nullptr;
        if (guarded_malloc(&p, bytes, cls) != cudaSuccess) {
            cudaGetLastError();
            fail("device allocation of %zu bytes for %s refused (memory guard budget or device memory)", bytes, what);
            return nullptr;
        }
        allocs.push_back({p, bytes, cls});
        return p;
    }
    void mark(int phase) {
        if (!prof) return;
        if (n_ev == (int)ev.size()) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            ev.push_back(e);
            ev_phase.push_back(0);
        }
        ev_phase[(size_t)n_ev] = phase;
        cudaEventRecord(ev[(size_t)n_ev++], stream);
    }
    void collect() {
        if (!prof || n_ev < 2) {
            n_ev = 0;
            return;
        }
        cudaEventSynchronize(ev[(size_t)n_ev - 1]);
        for (int i = 0; i + 1 < n_ev; ++i) {
            float m = 0.f;
            cudaEventElapsedTime(&m, ev[(size_t)i], ev[(size_t)i + 1]);
            ms[ev_phase[(size_t)i]] += m;
        }
        n_ev = 0;
    }
    ~Decoder() {
        if (stream) cudaStreamSynchronize(stream);
        drop_graphs();
        // borrowed MoE handles go back to their own streams
        for (auto& l : L)
            if (!l.own_moe && l.moe) aero_cuda_moe_set_stream(l.moe, nullptr);
        for (auto& l : L)
            if (l.own_moe && l.moe) aero_cuda_moe_close(l.moe);
        for (auto& a : allocs) guarded_free(a.p, a.bytes, a.cls);
        if (sbase) guarded_free(sbase, sbytes, kScratch);
        for (auto e : ev) cudaEventDestroy(e);
        if (own_stream) cudaStreamDestroy(own_stream);
    }
};

int64_t row_bytes_gguf(int dt, int cols) {
    return dt == AERO_DT_Q8_0 ? (int64_t)cols / 32 * 34 : dt == AERO_DT_Q4_K ? (int64_t)cols / 256 * 144 : -1;
}

// A (rows, cols) quantised matrix for the dense GEMVs: planes allocated here,
// filled by put_rows.
bool alloc_qmat(Decoder& g, int dt, int rows, int cols, QMat& m, const char* what) {
    if (dt != AERO_DT_Q8_0 && dt != AERO_DT_Q4_K)
        return g.fail("%s: ggml type %d (the decoder reads Q8_0 and Q4_K projections)", what, dt);
    if (cols % (dt == AERO_DT_Q8_0 ? 32 : 256))
        return g.fail("%s: row width %d is not a multiple of the block", what, cols);
    m.dtype = dt;
    m.rows = rows;
    m.cols = cols;
    m.n_expert = 1;
    m.qs_estride = align128((int64_t)rows * qm_row_qs_bytes(dt, cols));
    m.meta_estride = align128((int64_t)rows * qm_row_meta_bytes(dt, cols));
    m.qs = (const uint8_t*)g.alloc((size_t)m.qs_estride, kWeightsResident, what);
    m.meta = m.qs ? (const uint8_t*)g.alloc((size_t)m.meta_estride, kWeightsResident, what) : nullptr;
    return m.meta != nullptr;
}

bool put_rows(Decoder& g, QMat& m, int row0, const aero_cuda_tensor& t, int rows, const char* what) {
    if (t.dtype != m.dtype) return g.fail("%s: ggml type %d, expected %d", what, t.dtype, m.dtype);
    const int64_t rb = row_bytes_gguf(m.dtype, m.cols);
    const int64_t need = rb * rows;
    if (!t.data || t.nbytes < need) return g.fail("%s: %lld bytes given, %lld needed", what, (long long)t.nbytes, (long long)need);
    const bool dev = is_device_ptr(t.data);
    const uint8_t* src = static_cast<const uint8_t*>(t.data);
    void* stage = nullptr;
    const int64_t chunk_rows = std::max<int64_t>(1, std::min<int64_t>(rows, (128ll << 20) / rb));
    if (!dev) {
        if (guarded_malloc(&stage, (size_t)(chunk_rows * rb), kScratch) != cudaSuccess) {
            cudaGetLastError();
            return g.fail("%s: staging buffer refused", what);
        }
    } else if (m.dtype == AERO_DT_Q4_K && ((uintptr_t)src & 15) != 0) {
        return g.fail("%s: device source is not 16-byte aligned", what);
    }
    bool good = true;
    uint8_t* qs = const_cast<uint8_t*>(m.qs) + (int64_t)row0 * qm_row_qs_bytes(m.dtype, m.cols);
    uint8_t* meta = const_cast<uint8_t*>(m.meta) + (int64_t)row0 * qm_row_meta_bytes(m.dtype, m.cols);
    for (int64_t r0 = 0; r0 < rows && good; r0 += chunk_rows) {
        const int64_t n = std::min<int64_t>(chunk_rows, rows - r0);
        const uint8_t* s = src + r0 * rb;
        if (!dev) {
            good = g.ok(cudaMemcpyAsync(stage, s, (size_t)(n * rb), cudaMemcpyHostToDevice, g.stream), what);
            s = static_cast<const uint8_t*>(stage);
        }
        if (good)
            good = g.ok(launch_repack(m.dtype, s, n, m.cols, (int)n, 0, qs + r0 * qm_row_qs_bytes(m.dtype, m.cols),
                                      meta + r0 * qm_row_meta_bytes(m.dtype, m.cols), m.qs_estride, m.meta_estride,
                                      g.stream),
                        what);
        if (good) good = g.ok(cudaStreamSynchronize(g.stream), what);
    }
    if (stage) guarded_free(stage, (size_t)(chunk_rows * rb), kScratch);
    return good;
}

float* put_f32(Decoder& g, const float* src, int n, const char* what) {
    if (!src) {
        g.fail("%s is required", what);
        return nullptr;
    }
    float* p = (float*)g.alloc((size_t)n * 4, kWeightsResident, what);
    if (!p) return nullptr;
    if (!g.ok(cudaMemcpyAsync(p, src, (size_t)n * 4, is_device_ptr(src) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                              g.stream),
              what))
        return nullptr;
    return p;
}

bool ensure_step_scratch(Decoder& g, int T) {
    if (T <= g.cap && g.sbase) return true;
    const int cap = std::max(T, std::max(2 * g.cap, 16));
    const int HD = g.H * g.D, KD = g.HK * g.D, qkv_ld = HD + 2 * KD;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += (b + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_x = take((size_t)cap * g.d * 4), o_h = take((size_t)cap * g.d * 4);
    const size_t o_qkv = take((size_t)cap * qkv_ld * 4), o_att = take((size_t)cap * HD * 4);
    const size_t o_o = take((size_t)cap * g.d * 4), o_dm = take((size_t)cap * g.d * 4);
    const size_t o_part = take((size_t)cap * g.H * g.n_chunk * (g.D + 4) * 4);
    const size_t o_hq = take(qinput_bytes(cap, g.d)), o_aq = take(qinput_bytes(cap, HD));
    const size_t o_hf = take(qfrag_bytes(cap, g.d)), o_af = take(qfrag_bytes(cap, HD));
    const size_t o_tok = take((size_t)cap * 4), o_seq = take((size_t)cap * 4), o_pos = take((size_t)cap * 8);
    const size_t o_lg = take((size_t)cap * g.vocab * 4);
    void* p = nullptr;
    if (guarded_malloc(&p, off, kScratch) != cudaSuccess) {
        cudaGetLastError();
        return g.fail("step scratch of %zu bytes for %d tokens refused", off, cap);
    }
    if (g.sbase) {
        cudaStreamSynchronize(g.stream);
        guarded_free(g.sbase, g.sbytes, kScratch);
    }
    g.drop_graphs();
    g.sbase = p;
    g.sbytes = off;
    g.cap = cap;
    uint8_t* b = static_cast<uint8_t*>(p);
    g.x = (float*)(b + o_x);
    g.h32 = (float*)(b + o_h);
    g.qkv = (float*)(b + o_qkv);
    g.att = (float*)(b + o_att);
    g.o = (float*)(b + o_o);
    g.dm = (float*)(b + o_dm);
    g.part = (float*)(b + o_part);
    g.hq = qinput_at(b + o_hq, cap, g.d);
    g.aq = qinput_at(b + o_aq, cap, HD);
    g.hf = qfrag_at(b + o_hf, cap, g.d);
    g.af = qfrag_at(b + o_af, cap, HD);
    g.tok = (int32_t*)(b + o_tok);
    g.seq = (int32_t*)(b + o_seq);
    g.pos = (int64_t*)(b + o_pos);
    g.logits = (float*)(b + o_lg);
    return true;
}

// The step on device buffers: head rows [r0, r0 + nh) of the step get logits
// into lg (row stride vocab), nh = 0: none.
bool run_step(Decoder& g, int T, int r0, int nh, float* lg) {
    cudaStream_t s = g.stream;
    const int HD = g.H * g.D, KD = g.HK * g.D, qkv_ld = HD + 2 * KD;
    g.mark(0);
    const int64_t nb = (int64_t)T * (g.d / 32);
    embed_q8_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(g.embd, g.tok, T, g.x);
    if (!g.ok(cudaGetLastError(), "embedding")) return false;
    for (int l = 0; l < g.n_layer; ++l) {
        DLayer& Ly = g.L[(size_t)l];
        g.mark(0);
        if (!g.ok(launch_norm(g.x, T, g.d, l > 0 ? g.dm : nullptr, Ly.attn_norm, g.eps, nullptr, g.hq,
                              T >= 2 ? g.hf : QFrag{}, s),
                  "norm"))
            return false;
        g.mark(1);
        if (!g.ok(gemv_dense(Ly.qkv, g.hq, T >= 2 ? g.hf : QFrag{}, T, g.qkv, qkv_ld, g.n_sm, s), "q/k/v projection"))
            return false;
        g.mark(2);
        if (!g.ok(attention(g.D, g.qkv, qkv_ld, T, g.H, g.HK, Ly.q_norm, Ly.k_norm, g.eps, g.rope_base, g.pos, g.seq,
                            Ly.kc, Ly.vc, g.n_ctx, g.part, g.n_chunk, g.att, g.aq, T >= 2 ? g.af : QFrag{}, s),
                  "attention"))
            return false;
        g.mark(1);
        if (!g.ok(gemv_dense(Ly.o, g.aq, T >= 2 ? g.af : QFrag{}, T, g.o, g.d, g.n_sm, s), "output projection"))
            return false;
        g.mark(0);
        if (!g.ok(launch_norm(g.x, T, g.d, g.o, Ly.ffn_norm, g.eps, g.h32, QInput{}, QFrag{}, s), "norm")) return false;
        g.mark(3);
        if (aero_cuda_moe_forward(Ly.moe, l, g.h32, T, g.d, g.dm) != 1)
            return g.fail("layer %d MoE: %s", l, aero_cuda_moe_last_error(Ly.moe));
    }
    g.mark(0);
    // the last layer's FFN output joins the residual for every row; the head rows are normed
    // the head rows start at r0: the tensor-core layout serves them when r0 is a group boundary
    const bool head_frag = nh >= 2 && r0 % 16 == 0;
    if (!g.ok(launch_norm(g.x, T, g.d, g.dm, g.out_norm, g.eps, nullptr, nh > 0 ? g.hq : QInput{},
                          head_frag ? g.hf : QFrag{}, s),
              "output norm"))
        return false;
    if (nh > 0) {
        g.mark(4);
        QInput hq = g.hq;
        hq.q1 += (int64_t)r0 * hq.K;
        hq.q0 += (int64_t)r0 * hq.K;
        hq.sx += (int64_t)r0 * (hq.K / 32);
        hq.s16 += (int64_t)r0 * (hq.K / 16);
        if (!g.ok(gemv_dense(g.head, hq, head_frag ? qfrag_from_group(g.hf, r0 / 16) : QFrag{}, nh, lg, g.vocab,
                             g.n_sm, s),
                  "head"))
            return false;
    }
    g.mark(0);
    return true;
}

// run_step through a CUDA graph where one applies (see Decoder::graphs). A
// capture that fails (an error in the step, or a call the capture refuses)
// switches graphs off for this decoder and runs the step eagerly.
bool run_graphed(Decoder& g, int T, int r0, int nh, float* lg) {
    if (!g.use_graphs || g.prof || T > kDecodeMaxTokens) return run_step(g, T, r0, nh, lg);
    const auto key = std::make_tuple(T, r0, nh, (uintptr_t)lg);
    auto it = g.graphs.find(key);
    if (it != g.graphs.end()) return g.ok(cudaGraphLaunch(it->second, g.stream), "step graph");
    if (g.seen.insert(key).second) return run_step(g, T, r0, nh, lg);
    if (cudaStreamBeginCapture(g.stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        g.use_graphs = false;
        return run_step(g, T, r0, nh, lg);
    }
    const bool ran = run_step(g, T, r0, nh, lg);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(g.stream, &graph);
    cudaGraphExec_t exec = nullptr;
    const bool captured = ran && e == cudaSuccess && graph &&
                          cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
    if (graph) cudaGraphDestroy(graph);
    if (!captured) {
        cudaGetLastError();
        g.use_graphs = false;
        g.err.clear();
        return run_step(g, T, r0, nh, lg);
    }
    g.graphs[key] = exec;
    return g.ok(cudaGraphLaunch(exec, g.stream), "step graph");
}

bool step_entry(Decoder& g, const int32_t* tokens, const int32_t* seqs, const int64_t* positions, int T, float* logits,
                bool last_only) {
    if (T <= 0) return g.fail("T=%d", T);
    if (!tokens || !positions) return g.fail("null tokens or positions");
    std::set<std::pair<int32_t, int64_t>> seen;
    for (int i = 0; i < T; ++i) {
        const int32_t sq = seqs ? seqs[i] : 0;
        if (tokens[i] < 0 || tokens[i] >= g.vocab) return g.fail("token %d = %d outside [0, %d)", i, tokens[i], g.vocab);
        if (sq < 0 || sq >= g.n_seq) return g.fail("sequence %d = %d outside [0, %d)", i, sq, g.n_seq);
        if (positions[i] < 0 || positions[i] >= g.n_ctx)
            return g.fail("position %d = %lld outside [0, %d)", i, (long long)positions[i], g.n_ctx);
        if (!seen.insert({sq, positions[i]}).second)
            return g.fail("sequence %d position %lld appears twice in the step", sq, (long long)positions[i]);
    }
    if (cudaSetDevice(g.device) != cudaSuccess) return g.fail("cudaSetDevice(%d) failed", g.device);
    if (!ensure_step_scratch(g, T)) return false;
    // pageable host sources: each copy has taken the bytes when the call returns
    if (!g.ok(cudaMemcpyAsync(g.tok, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, g.stream), "tokens") ||
        !g.ok(cudaMemcpyAsync(g.pos, positions, (size_t)T * 8, cudaMemcpyHostToDevice, g.stream), "positions"))
        return false;
    if (seqs) {
        if (!g.ok(cudaMemcpyAsync(g.seq, seqs, (size_t)T * 4, cudaMemcpyHostToDevice, g.stream), "sequences")) return false;
    } else if (!g.ok(cudaMemsetAsync(g.seq, 0, (size_t)T * 4, g.stream), "sequences")) {
        return false;
    }
    const int r0 = last_only ? T - 1 : 0, nh = logits ? (last_only ? 1 : T) : 0;
    const bool dev_out = logits && is_device_ptr(logits);
    float* lg = dev_out ? logits : g.logits;
    if (T > g.max_T) {
        g.drop_graphs();
        g.max_T = T;
    }
    if (!run_graphed(g, T, r0, nh, lg)) return false;
    if (logits && !dev_out) {
        if (!g.ok(cudaMemcpyAsync(logits, g.logits, (size_t)nh * g.vocab * 4, cudaMemcpyDeviceToHost, g.stream), "logits"))
            return false;
        if (!g.ok(cudaStreamSynchronize(g.stream), "step")) return false;
        for (auto& l : g.L)
            if (aero_cuda_moe_status(l.moe) != 0) return g.fail("a MoE layer's device wait gave up: the step is invalid");
    }
    g.collect();
    return true;
}

Decoder* open_decoder(const aero_cuda_decoder_desc* d, std::string* why, bool own_moe) {
    if (!d) {
        *why = "null descriptor";
        return nullptr;
    }
    auto* g = new Decoder();
    auto bad = [&](const std::string& m) {
        *why = m.empty() ? g->err : m;
        delete g;  // closes the MoE handles it owns
        return (Decoder*)nullptr;
    };
    if (d->n_layer > 0 && d->n_layer <= 4096 && d->layers) {
        // take the handles first, so an owned one is closed whatever fails below
        g->L.resize((size_t)d->n_layer);
        for (int l = 0; l < d->n_layer; ++l) {
            g->L[(size_t)l].moe = d->layers[l].moe;
            g->L[(size_t)l].own_moe = own_moe;
        }
    }
    g->device = d->device;
    g->n_layer = d->n_layer;
    g->d = d->n_embd;
    g->H = d->n_head;
    g->HK = d->n_head_kv;
    g->D = d->head_dim;
    g->vocab = d->vocab;
    g->n_seq = d->n_seq;
    g->n_ctx = d->n_ctx;
    g->eps = d->eps;
    g->rope_base = d->rope_base;
    if (g->n_layer <= 0 || g->n_layer > 4096 || g->d <= 0 || g->d % 32 || g->vocab <= 0 || g->n_seq <= 0 || g->n_ctx <= 0)
        return bad("n_layer, vocab, n_seq, n_ctx must be positive and n_embd a multiple of 32");
    if (g->n_ctx > 1024 * kAttnChunk) return bad("n_ctx above 65536 positions per sequence");
    if (g->d > kNormGroups * 256 * 8) return bad("n_embd above 8192");
    if (g->H <= 0 || g->HK <= 0 || g->H % g->HK || g->H / g->HK > kMaxGroup)
        return bad("n_head must be a multiple of n_head_kv with at most 16 query heads per kv head");
    if (g->D != 64 && g->D != 128 && g->D != 192 && g->D != 256) return bad("head_dim must be 64, 128, 192 or 256");
    if (!d->layers) return bad("layers are required");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return bad("no CUDA device is available (this library has no CPU path)");
    }
    if (g->device < 0 || g->device >= ndev) return bad("device does not exist");
    cudaSetDevice(g->device);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, g->device) == cudaSuccess) g->n_sm = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&g->own_stream, cudaStreamNonBlocking) != cudaSuccess) return bad("stream creation failed");
    g->stream = g->own_stream;
    g->n_chunk = (g->n_ctx + kAttnChunk - 1) / kAttnChunk;
    if (const char* v = std::getenv("AERO_DECODER_GRAPHS")) g->use_graphs = std::atoi(v) != 0;
    const int HD = g->H * g->D, KD = g->HK * g->D;
    // plan the whole load (weights and caches; the MoE handles planned their own)
    // before allocating (admit_plan, src/memory_guard.cpp:192-213)
    {
        const size_t plan = (size_t)aero_cuda_decoder_plan_bytes(d, nullptr);
        char why2[256];
        if (!aero_cuda_guard_admit_plan(plan, why2, sizeof(why2))) return bad(std::string("load refused: ") + why2);
    }
    // weights
    if (d->token_embd.dtype != AERO_DT_Q8_0) return bad("token_embd must be Q8_0");
    if (!alloc_qmat(*g, AERO_DT_Q8_0, g->vocab, g->d, g->embd, "token_embd") ||
        !put_rows(*g, g->embd, 0, d->token_embd, g->vocab, "token_embd"))
        return bad("");
    if (d->output.data) {
        if (!alloc_qmat(*g, d->output.dtype, g->vocab, g->d, g->head, "output") ||
            !put_rows(*g, g->head, 0, d->output, g->vocab, "output"))
            return bad("");
    } else {
        g->head = g->embd;
    }
    g->out_norm = put_f32(*g, d->output_norm, g->d, "output_norm");
    if (!g->out_norm) return bad("");
    const size_t kv_bytes = (size_t)g->n_seq * g->HK * g->n_ctx * g->D * 2;
    for (int l = 0; l < g->n_layer; ++l) {
        const aero_cuda_decoder_layer& s = d->layers[l];
        DLayer& Ly = g->L[(size_t)l];
        if (!s.moe) return bad("layer " + std::to_string(l) + ": no MoE handle");
        int32_t info[8] = {0};
        aero_cuda_moe_info(s.moe, info);
        if (info[0] != g->d) return bad("layer " + std::to_string(l) + ": the MoE handle's n_embd differs");
        char what[64];
        std::snprintf(what, sizeof(what), "blk.%d.attn_qkv", l);
        if (s.attn_q.dtype != s.attn_k.dtype || s.attn_q.dtype != s.attn_v.dtype)
            return bad(std::string(what) + ": q, k and v must share one ggml type");
        if (!alloc_qmat(*g, s.attn_q.dtype, HD + 2 * KD, g->d, Ly.qkv, what) ||
            !put_rows(*g, Ly.qkv, 0, s.attn_q, HD, what) || !put_rows(*g, Ly.qkv, HD, s.attn_k, KD, what) ||
            !put_rows(*g, Ly.qkv, HD + KD, s.attn_v, KD, what))
            return bad("");
        std::snprintf(what, sizeof(what), "blk.%d.attn_output", l);
        if (!alloc_qmat(*g, s.attn_output.dtype, g->d, HD, Ly.o, what) || !put_rows(*g, Ly.o, 0, s.attn_output, g->d, what))
            return bad("");
        Ly.attn_norm = put_f32(*g, s.attn_norm, g->d, "attn_norm");
        Ly.ffn_norm = Ly.attn_norm ? put_f32(*g, s.ffn_norm, g->d, "post_attention_norm") : nullptr;
        if (!Ly.ffn_norm) return bad("");
        if (s.q_norm && !(Ly.q_norm = put_f32(*g, s.q_norm, g->D, "attn_q_norm"))) return bad("");
        if (s.k_norm && !(Ly.k_norm = put_f32(*g, s.k_norm, g->D, "attn_k_norm"))) return bad("");
        Ly.kc = (__half*)g->alloc(kv_bytes, kKVCache, "key cache");
        Ly.vc = Ly.kc ? (__half*)g->alloc(kv_bytes, kKVCache, "value cache") : nullptr;
        if (!Ly.vc) return bad("");
        if (!g->ok(cudaMemsetAsync(Ly.kc, 0, kv_bytes, g->stream), "cache") ||
            !g->ok(cudaMemsetAsync(Ly.vc, 0, kv_bytes, g->stream), "cache"))
            return bad("");
        aero_cuda_moe_set_stream(s.moe, g->stream);
    }
    if (!g->ok(cudaStreamSynchronize(g->stream), "upload")) return bad("");
    return g;
}

}  // namespace
}  // namespace aero

using aero::Decoder;

extern "C" int64_t aero_cuda_decoder_plan_bytes(const aero_cuda_decoder_desc* d, int64_t* by_class) {
    if (!d || d->n_layer <= 0 || d->n_embd <= 0 || d->vocab <= 0) return -1;
    auto qmat = [](int dt, int64_t rows, int64_t cols) -> int64_t {
        if (dt != AERO_DT_Q8_0 && dt != AERO_DT_Q4_K) return 0;
        return align128(rows * qm_row_qs_bytes(dt, (int)cols)) +
               align128(rows * qm_row_meta_bytes(dt, (int)cols));
    };
    const int64_t dm = d->n_embd, HD = (int64_t)d->n_head * d->head_dim, KD = (int64_t)d->n_head_kv * d->head_dim;
    int64_t w = qmat(AERO_DT_Q8_0, d->vocab, dm) + dm * 4;
    if (d->output.data) w += qmat(d->output.dtype, d->vocab, dm);
    int64_t kv = 0;
    for (int l = 0; l < d->n_layer; ++l) {
        const int dt = d->layers ? d->layers[l].attn_q.dtype : AERO_DT_Q8_0;
        const int dto = d->layers ? d->layers[l].attn_output.dtype : AERO_DT_Q8_0;
        w += qmat(dt, HD + 2 * KD, dm) + qmat(dto, dm, HD) + 2 * dm * 4;
        if (d->layers && d->layers[l].q_norm) w += (int64_t)d->head_dim * 4;
        if (d->layers && d->layers[l].k_norm) w += (int64_t)d->head_dim * 4;
        kv += 2 * (int64_t)d->n_seq * KD * d->n_ctx * 2;
    }
    if (by_class) {
        by_class[0] = w;   // weights resident
        by_class[1] = kv;  // KV cache
    }
    return w + kv;
}

extern "C" {

void* aero_cuda_decoder_open(const aero_cuda_decoder_desc* desc, char* err, int errlen) {
    std::string why;
    Decoder* g = aero::open_decoder(desc, &why, false);
    if (!g && err && errlen > 0) std::snprintf(err, (size_t)errlen, "%s", why.c_str());
    return g;
}

void* aero_cuda_decoder_open_gguf(const char* path, int device, int n_seq, int n_ctx, char* err, int errlen) {
    auto put = [&](const std::string& m) {
        if (err && errlen > 0) std::snprintf(err, (size_t)errlen, "%s", m.c_str());
        return (void*)nullptr;
    };
    aero::GgufFile f;
    std::string why;
    if (!path || !f.open(path, &why)) return put(path ? why : "null path");
    const std::string arch = f.arch();
    auto hp = [&](const char* key, int64_t def) {
        int64_t v = def;
        if (!f.get_int(arch + "." + key, &v)) f.get_int(key, &v);
        return v;
    };
    auto hpf = [&](const char* key, double def) {
        double v = def;
        if (!f.get_float(arch + "." + key, &v)) f.get_float(key, &v);
        return v;
    };
    aero_cuda_decoder_desc d{};
    d.n_layer = (int)hp("block_count", 0);
    d.n_embd = (int)hp("embedding_length", 0);
    d.n_head = (int)hp("attention.head_count", 0);
    d.n_head_kv = (int)hp("attention.head_count_kv", d.n_head);
    d.head_dim = (int)hp("attention.key_length", d.n_head > 0 ? d.n_embd / d.n_head : 0);
    if (hp("attention.value_length", d.head_dim) != d.head_dim) return put("value_length != key_length is not supported");
    if (hp("rope.dimension_count", d.head_dim) != d.head_dim) return put("partial RoPE is not supported");
    d.eps = (float)hpf("attention.layer_norm_rms_epsilon", 1e-6);
    d.rope_base = (float)hpf("rope.freq_base", 10000.0);
    d.n_seq = n_seq;
    d.n_ctx = n_ctx;
    d.device = device;
    const aero::GgufTensor* te = f.find("token_embd.weight");
    const aero::GgufTensor* to = f.find("output.weight");
    const aero::GgufTensor* tn = f.find("output_norm.weight");
    if (!te || te->dims.size() != 2 || !tn || tn->type != 0) return put("token_embd.weight / output_norm.weight (F32) missing");
    d.vocab = (int)te->shape(0);
    d.token_embd = {te->type, 0, f.data(*te), te->nbytes};
    if (to) d.output = {to->type, 0, f.data(*to), to->nbytes};
    d.output_norm = reinterpret_cast<const float*>(f.data(*tn));
    if (d.n_layer <= 0 || d.n_layer > 4096) return put(arch + ".block_count missing or out of range");
    std::vector<aero_cuda_decoder_layer> layers((size_t)d.n_layer);
    std::vector<void*> moes;
    auto close_moes = [&]() {
        for (void* m : moes) aero_cuda_moe_close(m);
    };
    for (int l = 0; l < d.n_layer; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        auto T = [&](const char* n) { return f.find(p + n); };
        const aero::GgufTensor *an = T("attn_norm.weight"), *pn = T("post_attention_norm.weight");
        if (!pn) pn = T("ffn_norm.weight");
        const aero::GgufTensor *q = T("attn_q.weight"), *k = T("attn_k.weight"), *v = T("attn_v.weight"),
                               *o = T("attn_output.weight"), *qn = T("attn_q_norm.weight"), *kn = T("attn_k_norm.weight");
        if (!an || !pn || !q || !k || !v || !o || an->type != 0 || pn->type != 0 || (qn && qn->type != 0) ||
            (kn && kn->type != 0)) {
            close_moes();
            return put(p + "attention tensors or F32 norms missing");
        }
        char e2[512] = {0};
        void* m = aero_cuda_moe_open_gguf(path, l, device, 0, 0, e2, sizeof(e2));
        if (!m) {
            close_moes();
            return put(p + "MoE: " + e2);
        }
        moes.push_back(m);
        aero_cuda_decoder_layer& L = layers[(size_t)l];
        L.attn_q = {q->type, 0, f.data(*q), q->nbytes};
        L.attn_k = {k->type, 0, f.data(*k), k->nbytes};
        L.attn_v = {v->type, 0, f.data(*v), v->nbytes};
        L.attn_output = {o->type, 0, f.data(*o), o->nbytes};
        L.attn_norm = reinterpret_cast<const float*>(f.data(*an));
        L.ffn_norm = reinterpret_cast<const float*>(f.data(*pn));
        L.q_norm = qn ? reinterpret_cast<const float*>(f.data(*qn)) : nullptr;
        L.k_norm = kn ? reinterpret_cast<const float*>(f.data(*kn)) : nullptr;
        L.moe = m;
    }
    d.layers = layers.data();
    Decoder* g = aero::open_decoder(&d, &why, true);  // owns the MoE handles, closed on failure too
    if (!g) return put(why);
    return g;
}

int aero_cuda_decoder_forward(void* dec, const int32_t* tokens, int n_tokens, const int64_t* positions, float* logits) {
    auto* g = static_cast<Decoder*>(dec);
    if (!g || !logits) return 0;
    return aero::step_entry(*g, tokens, nullptr, positions, n_tokens, logits, true) ? 1 : 0;
}

int aero_cuda_decoder_step(void* dec, const int32_t* tokens, const int32_t* seqs, const int64_t* positions, int T,
                           float* logits) {
    auto* g = static_cast<Decoder*>(dec);
    if (!g) return -1;
    return aero::step_entry(*g, tokens, seqs, positions, T, logits, false) ? 0 : -1;
}

int aero_cuda_decoder_set_stream(void* dec, void* stream) {
    auto* g = static_cast<Decoder*>(dec);
    if (!g) return -1;
    cudaStreamSynchronize(g->stream);
    g->stream = stream ? static_cast<cudaStream_t>(stream) : g->own_stream;
    for (auto& l : g->L)
        if (l.moe) aero_cuda_moe_set_stream(l.moe, g->stream);
    return 0;
}

int aero_cuda_decoder_kv(void* dec, int layer, void** k, void** v) {
    auto* g = static_cast<Decoder*>(dec);
    if (!g || layer < 0 || layer >= g->n_layer || !k || !v) return -1;
    *k = g->L[(size_t)layer].kc;
    *v = g->L[(size_t)layer].vc;
    return 0;
}

int aero_cuda_decoder_profile(void* dec, int on, double* ms) {
    auto* g = static_cast<Decoder*>(dec);
    if (!g) return -1;
    if (ms) {
        for (int i = 0; i < 5; ++i) ms[i] = g->ms[i];
        for (double& m : g->ms) m = 0.0;
    }
    g->prof = on != 0;
    return 0;
}

int aero_cuda_decoder_info(void* dec, int64_t* out8) {
    auto* g = static_cast<Decoder*>(dec);
    if (!g || !out8) return -1;
    const int64_t v[8] = {g->n_layer, g->d, g->H, g->HK, g->D, g->vocab, g->n_seq, g->n_ctx};
    for (int i = 0; i < 8; ++i) out8[i] = v[i];
    return 0;
}

const char* aero_cuda_decoder_last_error(void* dec) {
    auto* g = static_cast<Decoder*>(dec);
    return g ? g->err.c_str() : "null decoder";
}

void aero_cuda_decoder_close(void* dec) { delete static_cast<Decoder*>(dec); }

}  // extern "C"
