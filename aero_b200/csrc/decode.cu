// Decode (calls of up to 32 tokens): the whole MoE layer in one cooperative
// launch (two CTAs per SM), five phases separated by grid barriers.
//
//   A  router logits (f32, x . W_r + bias, plus the shared-gate column) and the
//      call's x rows coded as integer input                         | barrier
//   B  top-k per token (src/moe.cpp:26-66, the same selection as the top-k
//      kernel): in every CTA for calls of up to 8 tokens, else one warp per
//      token over the grid followed by a barrier; then, in every CTA, the
//      dispatch of the T*k pairs into expert segments (stable in (token, slot)
//      order: one warp's bitonic sort for up to 32 pairs, a counting sort
//      above), kept in shared memory
//   C  gate/up GEMVs over the active experts and the shared expert:
//      act[pair][row] = silu(gate . x) * (up . x) in f32       | barrier
//   D  down GEMVs: y[pair][row] = down row . act[pair], act coded as integer
//      input by each lane for its own 64 values                 | barrier
//   E  combine: out[t] = sum over slots in order of w * y + sgate * y_shared
//      (src/moe.cpp:68-120)
//
// GEMV lanes. A lane owns 64 consecutive values of a row: for Q4_K the 32 code
// bytes of sub-blocks 2g and 2g+1 of one super-block plus that super-block's
// 16-byte header (one header load and one scale decode per row and lane); for
// Q8_0 two whole 32-value blocks and their two fp16 scales. Rows of K values
// take a group of G = pow2(K/64) >= 4 lanes; a warp covers 32/G rows per pass.
// Phases C and D are streams of chunks of 4 row dots (a unit = an expert with
// its pairs, or the shared expert; per unit its input rows, blocks of rows, and
// the chunks of a block): each warp takes a contiguous range of chunks, keeps
// kRing rows' weights in flight across chunk boundaries, accumulates one
// partial per row dot, and a partial reduce-scatter across the lane group
// leaves each lane with the full sum of one row dot of the chunk. Only the
// selected experts' blocks are read from HBM, once per pair (an expert's second
// token re-reads its rows from L2); accumulation is f32.
//
// Integer input (x and act), per 16 values: a 15-bit code split into two int8
// planes (v ~= sx * (128 q1 + q0), |128 q1 + q0| <= 16383) and the exact f32 sum
// of the 16 values (the Q4_K min term). A lane's 64 values are four blocks:
// sum(q x) is two chains of dp4a over the raw code bytes per block, and the
// per-sub-block factorisation of the quantised dot (src/kernels.cpp:78-84,
// 123-156) applies the scales once per block:
//   Q8_0: d * sum(q x)          Q4_K: d sc * sum(q x) - dmin m * sum(x)
// The input coding error is at most 2^-15 of each 16-value block's largest |v|.
//
// Every grid-barrier wait is bounded (%globaltimer): a CTA that gives up
// records an error code (device word and the handle's host-mapped word) and
// returns; the host reports it at its next synchronisation or call.
#include <cuda_runtime.h>

#include <algorithm>
#include <cub/block/block_scan.cuh>

#include "internal.h"
#include "topk.cuh"

namespace aero {
namespace {

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kScanItems = (1024 + kDecThreads) / kDecThreads;  // items per thread: E + 1 <= 1025 values
constexpr int kRouterTokGroup = 4;  // tokens per router warp task
constexpr int kTopkInCta = 8;       // calls of up to this many tokens select their experts in every CTA
constexpr int kJBlock = 16;         // rows of gate and of up per block of the gate/up stream
constexpr int kRing = 2;            // weight rows in flight per lane (two CTAs per SM)
constexpr int kErrBarrier = 31;

__device__ __forceinline__ uint64_t dec_gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier b of this launch: every CTA adds one to the counter, which
// starts the launch at zero (barrier b completes when it reaches
// (b + 1) * gridDim.x). False when the wait ran out (the error is recorded).
__device__ bool grid_barrier(const DecodeArgs& a, int b, volatile int* abort_s) {
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t target = ((uint32_t)b + 1u) * gridDim.x;
        __threadfence();
        atomicAdd(a.bar, 1u);
        const uint64_t t0 = dec_gtimer();
        while ((int32_t)(ld_acquire_gpu(a.bar) - target) < 0) {
            if (dec_gtimer() - t0 > a.wait_ns) {
                if (atomicCAS(a.err, 0, kErrBarrier) == 0 && a.err_host) {
                    *reinterpret_cast<volatile int32_t*>(a.err_host) = kErrBarrier;
                    __threadfence_system();
                }
                *abort_s = 1;
                break;
            }
            __nanosleep(64);
        }
        __threadfence();
    }
    __syncthreads();
    return *abort_s == 0;
}

// ------------------------------------------------------------ integer input
// Row of K values: q1 [K] int8, q0 [K] int8, then (sx, s16) per 16 values.
__host__ __device__ inline int64_t qx_row_bytes(int K) { return (int64_t)K * 2 + (int64_t)K / 2; }

// Codes the 16 values v[0..16) into the row at column c (a multiple of 16).
__device__ __forceinline__ void qx_code16(const float* v, uint8_t* row, int K, int c) {
    float mx = 0.f, s = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        mx = fmaxf(mx, fabsf(v[i]));
        s += v[i];
    }
    const float inv = mx > 0.f ? 16383.0f / mx : 0.f;
    uint32_t w1[4], w0[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t p1 = 0, p0 = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q = __float2int_rn(v[4 * i + j] * inv);  // |q| <= 16383
            p1 |= (uint32_t)(q >> 7 & 0xFF) << (8 * j);
            p0 |= (uint32_t)(q & 127) << (8 * j);
        }
        w1[i] = p1;
        w0[i] = p0;
    }
    *reinterpret_cast<uint4*>(row + c) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
    *reinterpret_cast<uint4*>(row + K + c) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    *reinterpret_cast<float2*>(row + 2 * K + (c / 16) * 8) = make_float2(mx / 16383.0f, s);
}

// A lane's 64 values of one input row: both code planes and the four blocks' (sx, s16).
struct XSlice {
    uint32_t h[16], l[16];
    float sx[4], s16[4];
};

__device__ __forceinline__ void xs_load(const uint8_t* row, int K, int gl, XSlice& s) {
    const uint4* ph = reinterpret_cast<const uint4*>(row + 64 * gl);
    const uint4* pl = reinterpret_cast<const uint4*>(row + K + 64 * gl);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 a = ph[i], b = pl[i];
        s.h[4 * i] = a.x, s.h[4 * i + 1] = a.y, s.h[4 * i + 2] = a.z, s.h[4 * i + 3] = a.w;
        s.l[4 * i] = b.x, s.l[4 * i + 1] = b.y, s.l[4 * i + 2] = b.z, s.l[4 * i + 3] = b.w;
    }
    const float4* ps = reinterpret_cast<const float4*>(row + 2 * K + 32 * gl);
    const float4 s0 = ps[0], s1 = ps[1];
    s.sx[0] = s0.x, s.s16[0] = s0.y, s.sx[1] = s0.z, s.s16[1] = s0.w;
    s.sx[2] = s1.x, s.s16[2] = s1.y, s.sx[3] = s1.z, s.s16[3] = s1.w;
}

// ------------------------------------------------------------ weight slices
template <int DT>
struct WSlice;
template <>
struct WSlice<AERO_DT_Q4_K> {
    uint4 a, b, hdr;  // 32 code bytes, the super-block header
};
template <>
struct WSlice<AERO_DT_Q8_0> {
    uint4 q[4];
    uint32_t sc;  // the two blocks' fp16 scales
};

__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

// Row r of one expert's matrix, from the expert's plane bases (qs, meta).
template <int DT>
__device__ __forceinline__ void ws_load(const uint8_t* qs, const uint8_t* mt, int64_t qs_row, int64_t mt_row, int r,
                                        int gl, WSlice<DT>& w) {
    qs += (int64_t)r * qs_row;
    mt += (int64_t)r * mt_row;
    if constexpr (DT == AERO_DT_Q4_K) {
        w.a = ldg16(qs + 32 * gl);
        w.b = ldg16(qs + 32 * gl + 16);
        w.hdr = ldg16(mt + 16 * (gl >> 2));
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) w.q[i] = ldg16(qs + 64 * gl + 16 * i);
        w.sc = __ldg(reinterpret_cast<const uint32_t*>(mt + 4 * gl));
    }
}

// dp4a with unsigned bytes in a and signed bytes in b
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// sum over 16 values (4 words of unsigned codes) of code * (128 q1 + q0)
__device__ __forceinline__ int dot16u(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, const uint32_t* h,
                                      const uint32_t* l) {
    int a = dp4a_us(w0, h[0], 0), b = dp4a_us(w0, l[0], 0);
    a = dp4a_us(w1, h[1], a), b = dp4a_us(w1, l[1], b);
    a = dp4a_us(w2, h[2], a), b = dp4a_us(w2, l[2], b);
    a = dp4a_us(w3, h[3], a), b = dp4a_us(w3, l[3], b);
    return a * 128 + b;
}
// sum over 16 values (4 words of codes) of code * (128 q1 + q0)
__device__ __forceinline__ int dot16(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, const uint32_t* h,
                                     const uint32_t* l) {
    int a = __dp4a((int)w0, (int)h[0], 0), b = __dp4a((int)w0, (int)l[0], 0);
    a = __dp4a((int)w1, (int)h[1], a), b = __dp4a((int)w1, (int)l[1], b);
    a = __dp4a((int)w2, (int)h[2], a), b = __dp4a((int)w2, (int)l[2], b);
    a = __dp4a((int)w3, (int)h[3], a), b = __dp4a((int)w3, (int)l[3], b);
    return a * 128 + b;
}

// The 6-bit scales and mins of sub-blocks j and j + 1 (j = 2g even) from the
// three words of packed scale bytes q[0..12) (src/kernels.cpp:65-73), two
// 16-bit lanes at a time and without a branch on j < 4 (lanes of one warp hold
// different j): for j < 4 sc = q[j] & 63, m = q[j + 4] & 63; otherwise
// sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4), m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4).
// sc2 / m2 hold sub-block j in bits 0-7 and j + 1 in bits 16-23.
__device__ __forceinline__ void q4k_sc_m_pair(uint32_t w0, uint32_t w1, uint32_t w2, int j, uint32_t& sc2,
                                              uint32_t& m2) {
    const int sh = 8 * (j & 3);
    // bytes j, j + 1 (mod 4) of each word, spread to bits 0-7 and 16-23
    const uint32_t y = __byte_perm(w0 >> sh, 0, 0x5140), z = __byte_perm(w1 >> sh, 0, 0x5140),
                   w = __byte_perm(w2 >> sh, 0, 0x5140);
    const uint32_t hy = (y & 0x00C000C0u) >> 2, hz = (z & 0x00C000C0u) >> 2;
    const bool lo = j < 4;
    sc2 = lo ? (y & 0x003F003Fu) : ((w & 0x000F000Fu) | hy);
    m2 = lo ? (z & 0x003F003Fu) : (((w >> 4) & 0x000F000Fu) | hz);
}

// This lane's part of (row . input).
template <int DT>
__device__ __forceinline__ float ws_dot(const WSlice<DT>& w, int gl, const XSlice& x) {
    if constexpr (DT == AERO_DT_Q4_K) {
        const uint32_t q[8] = {w.a.x, w.a.y, w.a.z, w.a.w, w.b.x, w.b.y, w.b.z, w.b.w};
        // low nibbles as bytes; high nibbles kept in place (16 x the code, an
        // unsigned byte), the factor 16 folded into the scale below
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = q[i] & 0x0F0F0F0Fu;
            hi[i] = q[i] & 0xF0F0F0F0u;
        }
        const float d = __half2float(__ushort_as_half((unsigned short)(w.hdr.x & 0xFFFFu)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(w.hdr.x >> 16)));
        uint32_t sc2, m2;
        q4k_sc_m_pair(w.hdr.y, w.hdr.z, w.hdr.w, 2 * (gl & 3), sc2, m2);
        // low nibbles: sub-block 2g (values 0-31 = blocks 0, 1); high: 2g+1 (blocks 2, 3)
        const int s0 = dot16u(lo[0], lo[1], lo[2], lo[3], x.h, x.l);
        const int s1 = dot16u(lo[4], lo[5], lo[6], lo[7], x.h + 4, x.l + 4);
        const int s2 = dot16u(hi[0], hi[1], hi[2], hi[3], x.h + 8, x.l + 8);
        const int s3 = dot16u(hi[4], hi[5], hi[6], hi[7], x.h + 12, x.l + 12);
        const float p0 = fmaf(x.sx[0], (float)s0, x.sx[1] * (float)s1);
        const float p1 = fmaf(x.sx[2], (float)s2, x.sx[3] * (float)s3);
        const float sc0 = (float)(sc2 & 0xFFu), sc1 = (float)(sc2 >> 16);
        const float m0 = (float)(m2 & 0xFFu), m1 = (float)(m2 >> 16);
        return (d * sc0 * p0 - dmin * m0 * (x.s16[0] + x.s16[1])) +
               (d * sc1 * 0.0625f * p1 - dmin * m1 * (x.s16[2] + x.s16[3]));
    } else {
        const float d0 = __half2float(__ushort_as_half((unsigned short)(w.sc & 0xFFFFu)));
        const float d1 = __half2float(__ushort_as_half((unsigned short)(w.sc >> 16)));
        const int s0 = dot16(w.q[0].x, w.q[0].y, w.q[0].z, w.q[0].w, x.h, x.l);
        const int s1 = dot16(w.q[1].x, w.q[1].y, w.q[1].z, w.q[1].w, x.h + 4, x.l + 4);
        const int s2 = dot16(w.q[2].x, w.q[2].y, w.q[2].z, w.q[2].w, x.h + 8, x.l + 8);
        const int s3 = dot16(w.q[3].x, w.q[3].y, w.q[3].z, w.q[3].w, x.h + 12, x.l + 12);
        return d0 * fmaf(x.sx[0], (float)s0, x.sx[1] * (float)s1) + d1 * fmaf(x.sx[2], (float)s2, x.sx[3] * (float)s3);
    }
}

constexpr int kChunk = 4;  // row dots reduced together

// v[i] (i < 4) holds this lane's partial of chunk item i, for lane groups of
// G >= 4 lanes (runtime). Two halving steps over the top two bits of the
// group's lane index, then sums over the remaining bits: v[0] ends with the
// group's full sum of item (lane % G) / (G / 4).
__device__ __forceinline__ void chunk_reduce(float (&v)[kChunk], int G, int lane) {
    {
        const int o = G >> 1;
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float send = up ? v[i] : v[i + 2];
            const float keep = up ? v[i + 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    {
        const int o = G >> 2;
        const bool up = (lane & o) != 0;
        const float send = up ? v[0] : v[1];
        const float keep = up ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
    for (int o = G >> 3; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
}

__host__ __device__ inline int pow2_at_least(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}

// The lane's 64 values [64 gl, 64 gl + 64) of an f32 row, coded in registers
// (the same 16-value blocks as qx_code16).
__device__ __forceinline__ void xs_code_f32(const float* row, int gl, XSlice& x) {
    const float4* src = reinterpret_cast<const float4*>(row + 64 * gl);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 f = src[4 * b + j];
            v[4 * j] = f.x, v[4 * j + 1] = f.y, v[4 * j + 2] = f.z, v[4 * j + 3] = f.w;
        }
        float mx = 0.f, s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            mx = fmaxf(mx, fabsf(v[i]));
            s += v[i];
        }
        const float inv = mx > 0.f ? 16383.0f / mx : 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t p1 = 0, p0 = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int q = __float2int_rn(v[4 * i + j] * inv);
                p1 |= (uint32_t)(q >> 7 & 0xFF) << (8 * j);
                p0 |= (uint32_t)(q & 127) << (8 * j);
            }
            x.h[4 * b + i] = p1;
            x.l[4 * b + i] = p0;
        }
        x.sx[b] = mx / 16383.0f;
        x.s16[b] = s;
    }
}

// A warp's position in a stream of GEMV chunks (4 row dots each). The stream
// runs over units (experts, then the shared expert), the unit's input rows,
// blocks of rows, and the chunks of a block; `pre` holds each unit's first
// chunk. Gate/up: blocks of 16 rows of gate and up, chunk c = items 4c..4c+3,
// item q = 2 * pass + matrix (0 gate, 1 up), pass p covering rows p * (32 / G)
// + sub of the block. Down: blocks of 32 rows, item q = pass q.
struct Cursor {
    int u, i, blk, c;   // unit, its input row, block, chunk of the block
    int n_i, n_blk, n_c;
    int lg;             // log2 of the lane group G = pow2(K / 64)
    int k64;            // K / 64: lanes of a group that hold values
    bool sh;
    // the unit's expert matrices (gate/up: 0 gate, 1 up; down: 0) and row strides
    const uint8_t *q0, *m0, *q1, *m1;
    int64_t qs_row, mt_row;
};

// ------------------------------------------------------------ shared state
// Per-CTA tables of the call's routing (phase B).
struct DecShared {
    int32_t* cnt;     // [E] pairs per expert, then the scatter's cursor
    int32_t* off;     // [E + 1] expert offsets
    int32_t* idx;     // [P] selected expert of pair p = t * k + s
    float* w;         // [P]
    int32_t* perm;    // [P] sorted position -> pair
    int32_t* inv;     // [P] pair -> sorted position
    float* sgate;     // [T]
    int32_t* u_e;     // [U] unit expert (-1: the shared expert)
    int32_t* u_pos;   // [U] first sorted position (shared: P)
    int32_t* u_n;     // [U] pairs (shared: T)
    int32_t* gu_pre;  // [U + 1] first gate/up chunk of each unit
    int32_t* dn_pre;  // [U + 1] first down chunk of each unit
};

// Exclusive scan of v[0..n) in place (n <= kScanItems * blockDim.x); returns the total.
template <typename Scan>
__device__ int block_excl_scan(int32_t* v, int n, typename Scan::TempStorage& tmp) {
    int in[kScanItems], out[kScanItems], tot;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int i = kScanItems * threadIdx.x + j;
        in[j] = i < n ? v[i] : 0;
    }
    Scan(tmp).ExclusiveSum(in, out, tot);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
        const int i = kScanItems * threadIdx.x + j;
        if (i < n) v[i] = out[j];
    }
    __syncthreads();
    return tot;
}

// The last u with pre[u] <= task (pre[0] = 0, U >= 1).
__device__ __forceinline__ int find_unit(const int32_t* pre, int U, int task) {
    int lo = 0, hi = U - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (pre[mid] <= task)
            lo = mid;
        else
            hi = mid - 1;
    }
    return lo;
}

__host__ __device__ inline int log2_pow2(int p) {
    int l = 0;
    while ((1 << l) < p) ++l;
    return l;
}

// Unit parameters of a cursor (gateup: the gate/up stream, else the down stream).
__device__ __forceinline__ void cursor_unit(Cursor& c, const DecShared& S, const DecodeArgs& a, bool gateup) {
    c.sh = S.u_e[c.u] < 0;
    c.n_i = S.u_n[c.u];
    const int e = c.sh ? 0 : S.u_e[c.u];
    int K;
    const QMat *A, *B;
    if (gateup) {
        K = a.dp;
        c.n_blk = (c.sh ? a.Fs : a.F) / kJBlock;
        A = c.sh ? &a.sg : &a.gate;
        B = c.sh ? &a.su : &a.up;
    } else {
        K = c.sh ? a.Fs : a.F;
        c.n_blk = a.dp / 32;
        A = B = c.sh ? &a.sd : &a.down;
    }
    c.k64 = K / 64;
    c.lg = log2_pow2(c.k64);
    c.n_c = (1 << c.lg) / kChunk;
    c.q0 = A->qs + (int64_t)e * A->qs_estride;
    c.m0 = A->meta + (int64_t)e * A->meta_estride;
    c.q1 = B->qs + (int64_t)e * B->qs_estride;
    c.m1 = B->meta + (int64_t)e * B->meta_estride;
    c.qs_row = qm_row_qs_bytes(A->dtype, A->cols);
    c.mt_row = qm_row_meta_bytes(A->dtype, A->cols);
}

__device__ __forceinline__ void cursor_at(Cursor& c, int chunk, const int32_t* pre, int U, const DecShared& S,
                                          const DecodeArgs& a, bool gateup) {
    c.u = find_unit(pre, U, chunk);
    cursor_unit(c, S, a, gateup);
    int rel = chunk - pre[c.u];
    c.c = rel % c.n_c;
    rel /= c.n_c;
    c.blk = rel % c.n_blk;
    c.i = rel / c.n_blk;
}

__device__ __forceinline__ void cursor_next(Cursor& c, const DecShared& S, const DecodeArgs& a, bool gateup, int U) {
    if (++c.c < c.n_c) return;
    c.c = 0;
    if (++c.blk < c.n_blk) return;
    c.blk = 0;
    if (++c.i < c.n_i) return;
    c.i = 0;
    if (++c.u < U) cursor_unit(c, S, a, gateup);
}

// Weights of item s of the cursor's chunk for this lane.
template <int DT>
__device__ __forceinline__ void cursor_load(const Cursor& c, int s, bool gateup, int lane, WSlice<DT>& w) {
    const int gl = lane & ((1 << c.lg) - 1), sub = lane >> c.lg;
    if (gl >= c.k64) return;
    const int q = kChunk * c.c + s;
    const int shr = 5 - c.lg;  // log2 of the rows a pass covers
    if (gateup) {
        const int row = c.blk * kJBlock + ((q >> 1) << shr) + sub;
        if (q & 1)
            ws_load<DT>(c.q1, c.m1, c.qs_row, c.mt_row, row, gl, w);
        else
            ws_load<DT>(c.q0, c.m0, c.qs_row, c.mt_row, row, gl, w);
    } else {
        ws_load<DT>(c.q0, c.m0, c.qs_row, c.mt_row, c.blk * 32 + (q << shr) + sub, gl, w);
    }
}

// A warp's contiguous range [lo, hi) of a chunk stream: 4 row dots per chunk,
// kRing rows in flight across chunk boundaries; the input slice is (re)made when
// the unit or its input row changes; emit(cursor, v) gets each chunk's result
// (v = the full dot of item (lane % G) / (G / 4) of the chunk, in every lane).
template <int DT, typename MakeX, typename Emit>
__device__ __forceinline__ void gemv_stream(int lo, int hi, const int32_t* pre, int U, const DecShared& S,
                                            const DecodeArgs& a, bool gateup, int lane, MakeX make_x, Emit emit) {
    if (lo >= hi) return;
    Cursor cc, lc;
    cursor_at(cc, lo, pre, U, S, a, gateup);
    lc = cc;
    int ls = 0;                      // loader: item of its chunk
    int left = (hi - lo) * kChunk;   // items still to load
    WSlice<DT> ring[kRing];
    auto advance_load = [&]() {
        --left;
        if (++ls == kChunk) {
            ls = 0;
            if (left > 0) cursor_next(lc, S, a, gateup, U);
        }
    };
#pragma unroll
    for (int r = 0; r < kRing; ++r)
        if (left > 0) {
            cursor_load<DT>(lc, ls, gateup, lane, ring[r]);
            advance_load();
        }
    XSlice x;
    int xu = -1, xi = -1;
    for (int chunk = lo; chunk < hi; ++chunk) {
        const int gl = lane & ((1 << cc.lg) - 1);
        const bool on = gl < cc.k64;
        if (cc.u != xu || cc.i != xi) {
            if (on) make_x(cc, gl, x);
            xu = cc.u;
            xi = cc.i;
        }
        float acc[kChunk];
#pragma unroll
        for (int s = 0; s < kChunk; ++s) {
            acc[s] = on ? ws_dot<DT>(ring[s % kRing], gl, x) : 0.f;
            if (left > 0) {
                cursor_load<DT>(lc, ls, gateup, lane, ring[s % kRing]);
                advance_load();
            }
        }
        chunk_reduce(acc, 1 << cc.lg, lane);
        emit(cc, acc[0]);
        if (chunk + 1 < hi) cursor_next(cc, S, a, gateup, U);
    }
}

template <int DT, int PER>
__global__ void __launch_bounds__(kDecThreads, 2) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) uint8_t dsm[];
    using Scan = cub::BlockScan<int, kDecThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ int abort_s, n_units_s;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int T = a.T, E = a.E, k = a.k, P = T * k;
    const int n_warps = gridDim.x * kDecWarps;
    const int gwarp = blockIdx.x * kDecWarps + warp;
    // top-k by one warp per token over the grid (and one more barrier) for calls of
    // more than 8 tokens; up to 8, every CTA selects them itself (measured: at 16
    // tokens two selections per warp take longer than the spread and its barrier)
    const bool topk_spread = T > kTopkInCta;
    int nb = 0;                              // grid barriers passed
    if (threadIdx.x == 0) abort_s = 0;
    auto stamp = [&](int i) {
        if (a.stamps && blockIdx.x == 0 && threadIdx.x == 0) a.stamps[i] = dec_gtimer();
    };
    auto barrier = [&]() { return grid_barrier(a, nb++, &abort_s); };
    stamp(0);

    // ---------------------------------------------------------------- phase A
    {
        const int n_rows = a.logits_in ? (a.has_shared ? 1 : 0) : E + (a.has_shared ? 1 : 0);
        const int row0 = a.logits_in ? E : 0;
        // tokens per task: up to kRouterTokGroup (a router row read once for them), fewer
        // while that leaves warps idle (each token of a task is one more round trip)
        const int per_task = max(1, min(kRouterTokGroup, (T * n_rows + n_warps - 1) / max(1, n_warps)));
        const int n_tg = (T + per_task - 1) / per_task;
        const int n_tasks = n_rows * n_tg;
        const int nf4 = a.dp / 128;  // float4 per lane (dp <= 2048: at most 16)
        for (int task = gwarp; task < n_tasks; task += n_warps) {
            const int tg = task / n_rows, r = row0 + task % n_rows;
            const float* wr = a.router + (int64_t)r * a.dp;
            float4 wv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i < nf4) wv[i] = __ldg(reinterpret_cast<const float4*>(wr) + lane + 32 * i);
            for (int t = tg * per_task; t < min(T, (tg + 1) * per_task); ++t) {
                const float4* xr = reinterpret_cast<const float4*>(a.x + (int64_t)t * a.dp);
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    if (i < nf4) {
                        const float4 xv = __ldg(xr + lane + 32 * i);
                        acc = fmaf(wv[i].x, xv.x, acc);
                        acc = fmaf(wv[i].y, xv.y, acc);
                        acc = fmaf(wv[i].z, xv.z, acc);
                        acc = fmaf(wv[i].w, xv.w, acc);
                    }
                acc = warp_sum(acc);
                if (lane == 0) a.logits[(int64_t)t * a.lg_ld + r] = acc + (r < E && a.bias ? a.bias[r] : 0.f);
            }
        }
        // the call's x rows as integer input (one thread per 16 values)
        const int nb16 = a.dp / 16;
        for (int i = blockIdx.x * kDecThreads + threadIdx.x; i < T * nb16; i += gridDim.x * kDecThreads) {
            const int t = i / nb16, c = (i % nb16) * 16;
            float v[16];
            const float4* src = reinterpret_cast<const float4*>(a.x + (int64_t)t * a.dp + c);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 f = __ldg(src + j);
                v[4 * j] = f.x, v[4 * j + 1] = f.y, v[4 * j + 2] = f.z, v[4 * j + 3] = f.w;
            }
            qx_code16(v, a.xq + (int64_t)t * qx_row_bytes(a.dp), a.dp, c);
        }
    }
    if (!barrier()) return;
    stamp(1);

    // ---------------------------------------------------------------- phase B
    DecShared S;
    {
        uint8_t* p = dsm;
        auto take = [&](size_t bytes) {
            uint8_t* q = p;
            p += (bytes + 15) & ~(size_t)15;
            return q;
        };
        const int Umax = min(P, E) + 1;
        S.cnt = (int32_t*)take((size_t)E * 4);
        S.off = (int32_t*)take((size_t)(E + 1) * 4);
        S.idx = (int32_t*)take((size_t)P * 4);
        S.w = (float*)take((size_t)P * 4);
        S.perm = (int32_t*)take((size_t)P * 4);
        S.inv = (int32_t*)take((size_t)P * 4);
        S.sgate = (float*)take((size_t)T * 4);
        S.u_e = (int32_t*)take((size_t)Umax * 4);
        S.u_pos = (int32_t*)take((size_t)Umax * 4);
        S.u_n = (int32_t*)take((size_t)Umax * 4);
        S.gu_pre = (int32_t*)take((size_t)(Umax + 1) * 4);
        S.dn_pre = (int32_t*)take((size_t)(Umax + 1) * 4);
    }
    const float* lg_base = a.logits_in ? a.logits_in : a.logits;
    const int lg_ld = a.logits_in ? a.ld_in : a.lg_ld;
    if (topk_spread) {
        // one warp per token over the grid, then every CTA reads the T * k choices
        for (int t = gwarp; t < T; t += n_warps) {
            int sel_i = 0;
            topk_warp<PER>(lg_base + (int64_t)t * lg_ld, E, k, a.norm, a.idx_out + t * k, a.w_out + t * k, &sel_i);
            if (lane == 0) a.sgate_out[t] = a.has_shared ? sigmoid_f(a.logits[(int64_t)t * a.lg_ld + E]) : 0.f;
        }
        if (!barrier()) return;
        for (int p = threadIdx.x; p < P; p += kDecThreads) {
            S.idx[p] = __ldcg(a.idx_out + p);
            S.w[p] = __ldcg(a.w_out + p);
        }
        for (int t = threadIdx.x; t < T; t += kDecThreads) S.sgate[t] = __ldcg(a.sgate_out + t);
    } else {
        for (int t = warp; t < T; t += kDecWarps) {
            int sel_i = 0;
            topk_warp<PER>(lg_base + (int64_t)t * lg_ld, E, k, a.norm, S.idx + t * k, S.w + t * k, &sel_i);
            if (lane == 0 && a.has_shared) S.sgate[t] = sigmoid_f(a.logits[(int64_t)t * a.lg_ld + E]);
        }
    }
    __syncthreads();
    if (P <= 32) {
        // one warp: the pairs sorted by (expert, pair) with a bitonic exchange
        // across the lanes; lane = sorted position
        if (warp == 0) {
            const bool valid = lane < P;
            uint32_t key = valid ? ((uint32_t)S.idx[lane] << 5) | (uint32_t)lane : 0xFFFFFFFFu;
#pragma unroll
            for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, key, stride);
                    const bool keep_min = ((lane & stride) == 0) == ((lane & size) == 0);
                    key = keep_min ? min(key, other) : max(key, other);
                }
            const int pr = (int)(key & 31u), e = (int)(key >> 5);
            if (valid) {
                S.perm[lane] = pr;
                S.inv[pr] = lane;
            }
            const int prev_e = __shfl_up_sync(0xffffffffu, e, 1);
            const bool start = valid && (lane == 0 || prev_e != e);
            const unsigned starts = __ballot_sync(0xffffffffu, start);
            if (start) {
                const int u = __popc(starts & ((1u << lane) - 1u));
                const unsigned later = starts & ~((2u << lane) - 1u);
                const int end = later ? __ffs(later) - 1 : P;
                S.u_e[u] = e;
                S.u_pos[u] = lane;
                S.u_n[u] = end - lane;
            }
            if (lane == 0) {
                int U = __popc(starts);
                if (a.has_shared) {
                    S.u_e[U] = -1;
                    S.u_pos[U] = P;
                    S.u_n[U] = T;
                    ++U;
                }
                n_units_s = U;
            }
        }
        __syncthreads();
    } else {
        for (int e = threadIdx.x; e < E; e += kDecThreads) S.cnt[e] = 0;
        __syncthreads();
        for (int p = threadIdx.x; p < P; p += kDecThreads) atomicAdd(&S.cnt[S.idx[p]], 1);
        __syncthreads();
        // expert offsets (exclusive prefix of the counts)
        for (int e = threadIdx.x; e < E; e += kDecThreads) S.off[e] = S.cnt[e];
        __syncthreads();
        block_excl_scan<Scan>(S.off, E, scan_tmp);
        if (threadIdx.x == 0) S.off[E] = P;
        // the active units: experts in ascending order, then the shared expert
        {
            int in[kScanItems], out[kScanItems], tot;
    #pragma unroll
            for (int j = 0; j < kScanItems; ++j) {
                const int e = kScanItems * threadIdx.x + j;
                in[j] = e < E && S.cnt[e] > 0 ? 1 : 0;
            }
            Scan(scan_tmp).ExclusiveSum(in, out, tot);
    #pragma unroll
            for (int j = 0; j < kScanItems; ++j) {
                const int e = kScanItems * threadIdx.x + j;
                if (in[j]) {
                    S.u_e[out[j]] = e;
                    S.u_pos[out[j]] = S.off[e];
                    S.u_n[out[j]] = S.cnt[e];
                }
            }
            if (threadIdx.x == 0) {
                int U = tot;
                if (a.has_shared) {
                    S.u_e[U] = -1;
                    S.u_pos[U] = P;
                    S.u_n[U] = T;
                    ++U;
                }
                n_units_s = U;
            }
        }
        __syncthreads();
        // stable scatter (warp 0): pairs in order, equal experts ranked by __match_any_sync
        for (int e = threadIdx.x; e < E; e += kDecThreads) S.cnt[e] = S.off[e];  // cursor
        __syncthreads();
        if (warp == 0) {
            for (int base = 0; base < P; base += 32) {
                const int p = base + lane;
                const bool valid = p < P;
                const int e = valid ? S.idx[p] : -1 - lane;
                const unsigned peers = __match_any_sync(0xffffffffu, e);
                const int rank = __popc(peers & ((1u << lane) - 1u));
                const int pos = valid ? S.cnt[e] + rank : 0;
                __syncwarp();
                if (valid) {
                    S.perm[pos] = p;
                    S.inv[p] = pos;
                    if ((peers >> lane) == 1u) S.cnt[e] = pos + 1;
                }
                __syncwarp();
            }
        }
        __syncthreads();
    }
    const int U = n_units_s;
    // chunks per unit: input rows x blocks x (G / 4), and their exclusive prefixes (one
    // warp's shuffle scan for up to 32 units, a block scan above)
    auto unit_chunks = [&](int u, int& gu, int& dn) {
        const bool sh = S.u_e[u] < 0;
        const int Fu = sh ? a.Fs : a.F;
        gu = S.u_n[u] * (Fu / kJBlock) * (pow2_at_least(a.dp / 64) / kChunk);
        dn = S.u_n[u] * (a.dp / 32) * (pow2_at_least(Fu / 64) / kChunk);
    };
    __shared__ int tot_s[2];
    int n_gu, n_dn;
    if (U <= 32) {
        if (warp == 0) {
            int gu = 0, dn = 0;
            if (lane < U) unit_chunks(lane, gu, dn);
            int ig = gu, id = dn;  // inclusive prefixes
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int tg = __shfl_up_sync(0xffffffffu, ig, o), td = __shfl_up_sync(0xffffffffu, id, o);
                if (lane >= o) ig += tg, id += td;
            }
            if (lane < U) {
                S.gu_pre[lane] = ig - gu;
                S.dn_pre[lane] = id - dn;
            }
            if (lane == 31) tot_s[0] = ig, tot_s[1] = id;
        }
        __syncthreads();
        n_gu = tot_s[0];
        n_dn = tot_s[1];
    } else {
        for (int u = threadIdx.x; u < U; u += kDecThreads) unit_chunks(u, S.gu_pre[u], S.dn_pre[u]);
        __syncthreads();
        n_gu = block_excl_scan<Scan>(S.gu_pre, U, scan_tmp);
        n_dn = block_excl_scan<Scan>(S.dn_pre, U, scan_tmp);
    }
    if (blockIdx.x == 0) {
        // the call's routing for the host (stats, profiling)
        if (!topk_spread)
            for (int p = threadIdx.x; p < P; p += kDecThreads) {
                a.idx_out[p] = S.idx[p];
                a.w_out[p] = S.w[p];
            }
        if (threadIdx.x == 0) {
            *a.n_active_out = U - (a.has_shared ? 1 : 0);
            *a.p_real_out = P;
        }
    }
    __syncthreads();
    stamp(2);

    // ---------------------------------------------------------------- phase C
    // act[pair][row] = silu(gate . x) * (up . x) in f32; a warp streams its
    // contiguous range of chunks (2 rows of gate and up each)
    {
        const int per = (n_gu + n_warps - 1) / n_warps;
        const int lo = gwarp * per, hi = min(n_gu, lo + per);
        auto make_x = [&](const Cursor& c, int gl, XSlice& x) {
            const int tok = c.sh ? c.i : S.perm[S.u_pos[c.u] + c.i] / k;
            xs_load(a.xq + (int64_t)tok * qx_row_bytes(a.dp), a.dp, gl, x);
        };
        auto emit = [&](const Cursor& c, float v) {
            const int gl = lane & ((1 << c.lg) - 1), ls = c.lg - 2;  // log2 of the lanes sharing an item
            const int q = kChunk * c.c + (gl >> ls);                // this lane's item of the chunk
            const float partner = __shfl_xor_sync(0xffffffffu, v, 1 << ls);  // the other matrix of the row
            if ((q & 1) == 0 && (gl & ((1 << ls) - 1)) == 0) {
                const int row = c.blk * kJBlock + ((q >> 1) << (5 - c.lg)) + (lane >> c.lg);
                a.act[(int64_t)(S.u_pos[c.u] + c.i) * a.act_ld + row] = silu_f(v) * partner;
            }
        };
        gemv_stream<DT>(lo, hi, S.gu_pre, U, S, a, true, lane, make_x, emit);
    }
    if (!barrier()) return;
    stamp(3);

    // ---------------------------------------------------------------- phase D
    // y[pair][row] = down row . act[pair] (act coded per lane as it is first used)
    {
        const int per = (n_dn + n_warps - 1) / n_warps;
        const int lo = gwarp * per, hi = min(n_dn, lo + per);
        auto make_x = [&](const Cursor& c, int gl, XSlice& x) {
            xs_code_f32(a.act + (int64_t)(S.u_pos[c.u] + c.i) * a.act_ld, gl, x);
        };
        auto emit = [&](const Cursor& c, float v) {
            const int gl = lane & ((1 << c.lg) - 1), ls = c.lg - 2;
            if ((gl & ((1 << ls) - 1)) == 0) {
                const int row = c.blk * 32 + ((kChunk * c.c + (gl >> ls)) << (5 - c.lg)) + (lane >> c.lg);
                a.y[(int64_t)(S.u_pos[c.u] + c.i) * a.dp + row] = v;
            }
        };
        gemv_stream<DT>(lo, hi, S.dn_pre, U, S, a, false, lane, make_x, emit);
    }
    if (!barrier()) return;
    stamp(4);
    // Every CTA has passed the last barrier and no longer reads the counter: the
    // last one here zeroes it (and the exit count), so the next launch, or a
    // replay of this one, starts from zero.
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.bar + 2, 1u) == gridDim.x - 1) {
            atomicExch(a.bar, 0u);
            atomicExch(a.bar + 2, 0u);
        }
    }

    // ---------------------------------------------------------------- phase E
    // out[t][n] = sum_s w[t][s] * y[inv(t, s)][n] (slot order) + sgate[t] * y[P + t][n]
    {
        const int d4 = a.dp / 4;
        for (int i = blockIdx.x * kDecThreads + threadIdx.x; i < T * d4; i += gridDim.x * kDecThreads) {
            const int t = i / d4, c = (i % d4) * 4;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s = 0; s < k; ++s) {
                const float ws = S.w[t * k + s];
                const float4 v = __ldcg(reinterpret_cast<const float4*>(a.y + (int64_t)S.inv[t * k + s] * a.dp + c));
                o.x += ws * v.x, o.y += ws * v.y, o.z += ws * v.z, o.w += ws * v.w;
            }
            if (a.has_shared) {
                const float g = S.sgate[t];
                const float4 v = __ldcg(reinterpret_cast<const float4*>(a.y + (int64_t)(P + t) * a.dp + c));
                o.x += g * v.x, o.y += g * v.y, o.z += g * v.z, o.w += g * v.w;
            }
            *reinterpret_cast<float4*>(a.out + (int64_t)t * a.dp + c) = o;
        }
    }
    __syncthreads();
    stamp(5);
}

template <int DT>
const void* decode_kernel_for(int E) {
    if (E <= 128) return (const void*)decode_kernel<DT, 4>;
    if (E <= 256) return (const void*)decode_kernel<DT, 8>;
    if (E <= 512) return (const void*)decode_kernel<DT, 16>;
    return (const void*)decode_kernel<DT, 32>;
}

size_t decode_smem_bytes(int T, int E, int k) {
    const int P = T * k, Umax = std::min(P, E) + 1;
    auto al = [](size_t b) { return (b + 15) & ~(size_t)15; };
    return al((size_t)E * 4) + al((size_t)(E + 1) * 4) + 4 * al((size_t)P * 4) + al((size_t)T * 4) +
           3 * al((size_t)Umax * 4) + 2 * al((size_t)(Umax + 1) * 4);
}

}  // namespace

int64_t decode_qx_row_bytes(int K) { return qx_row_bytes(K); }

bool decode_supported(int dtype, int T, int E, int k, int dp, int F, int Fs, int has_shared) {
    if (dtype != AERO_DT_Q4_K && dtype != AERO_DT_Q8_0) return false;
    if (T < 1 || T > kDecodeMaxTokens || k < 1 || k > 32 || E < k || E > 1024) return false;
    if (std::min(T * k, E) + (has_shared ? 1 : 0) > kScanItems * kDecThreads) return false;
    // lane groups of at least 4 lanes: rows of at least 192 values
    if (dp % 128 || dp > 2048 || dp < 256 || F % 64 || F > 2048 || F < 192) return false;
    if (has_shared && (Fs % 64 || Fs > 2048 || Fs < 192)) return false;
    return true;
}

int decode_barriers(int T) { return T > kTopkInCta ? 4 : 3; }

cudaError_t launch_decode(const DecodeArgs& args, int n_sm, cudaStream_t s, int* grid_out) {
    DecodeArgs a = args;
    const void* fn = a.gate.dtype == AERO_DT_Q4_K ? decode_kernel_for<AERO_DT_Q4_K>(a.E)
                                                  : decode_kernel_for<AERO_DT_Q8_0>(a.E);
    const int grid = 2 * n_sm;  // two CTAs per SM (checked below against the occupancy)
    const size_t smem = decode_smem_bytes(a.T, a.E, a.k);
    // the dynamic shared memory each instantiation has been allowed so far (the
    // attribute call and the occupancy check run when it has to grow, not per call)
    struct Allowed {
        const void* fn;
        size_t smem;
    };
    static thread_local Allowed allowed[32] = {};
    Allowed* slot = nullptr;
    for (auto& x : allowed)
        if (x.fn == fn || x.fn == nullptr) {
            slot = &x;
            break;
        }
    if (!slot || slot->fn != fn || slot->smem < smem) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDecThreads, smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 2) return cudaErrorCooperativeLaunchTooLarge;
        if (slot) *slot = Allowed{fn, smem};
    }
    *grid_out = grid;
    void* params[] = {&a};
    return cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kDecThreads), params, smem, s);
}

}  // namespace aero
