// Shared device helpers for the B200 MoE library.
//
// Weight planes. Each expert tensor family (E experts x rows x cols, GGUF
// row-major (out, in)) is repacked once at load into two expert-major planes,
// every expert starting on a 128-byte boundary:
//   Q8_0  qs   int8   [E][rows][cols]            (the 32 int8 of each block)
//         meta fp16   [E][rows][cols/32]         (the block scale d)
//   Q4_K  qs   u8     [E][rows][cols/256][128]   (the 128 nibble bytes, as stored)
//         meta 16 B   [E][rows][cols/256]        (d, dmin, 12 packed scale bytes)
//   F32   qs   f32    [E][rows][cols]            (meta unused)
// A "chunk" is 16 bytes of qs: 16 values of one Q8_0 block, 32 values of one
// Q4_K super-block (16 low nibbles of sub-block 2g and 16 high nibbles of
// sub-block 2g+1), or 4 f32 values.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define AERO_DT_F32 0
#define AERO_DT_Q8_0 8
#define AERO_DT_Q4_K 12

struct QMat {
    const uint8_t* qs;
    const uint8_t* meta;
    int64_t qs_estride;    // bytes between experts in qs
    int64_t meta_estride;  // bytes between experts in meta
    int32_t dtype, rows, cols, n_expert;
};

__host__ __device__ inline int64_t qm_row_qs_bytes(int dtype, int cols) {
    return dtype == AERO_DT_Q8_0 ? (int64_t)cols
         : dtype == AERO_DT_Q4_K ? (int64_t)cols / 2
                                 : (int64_t)cols * 4;
}
__host__ __device__ inline int64_t qm_row_meta_bytes(int dtype, int cols) {
    return dtype == AERO_DT_Q8_0 ? (int64_t)cols / 32 * 2
         : dtype == AERO_DT_Q4_K ? (int64_t)cols / 256 * 16
                                 : 0;
}
__host__ __device__ inline int qm_chunks_per_row(int dtype, int cols) {
    return dtype == AERO_DT_Q8_0 ? cols / 16 : dtype == AERO_DT_Q4_K ? cols / 32 : cols / 4;
}
__host__ __device__ inline int64_t align128(int64_t v) { return (v + 127) & ~(int64_t)127; }

__device__ __forceinline__ const uint8_t* qm_row_qs(const QMat& m, int e, int r) {
    return m.qs + (int64_t)e * m.qs_estride + (int64_t)r * qm_row_qs_bytes(m.dtype, m.cols);
}
__device__ __forceinline__ const uint8_t* qm_row_meta(const QMat& m, int e, int r) {
    return m.meta + (int64_t)e * m.meta_estride + (int64_t)r * qm_row_meta_bytes(m.dtype, m.cols);
}

#if defined(__CUDACC__)
// Streaming 16-byte load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float4 ld_f4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
template <int W>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = W / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Unsigned byte i of w as an exact float: the byte lands in the low mantissa
// bits of 2^23, and subtracting 2^23 leaves its integer value.
__device__ __forceinline__ float ubyte_to_f(uint32_t w, int i) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + (uint32_t)i)) - 8388608.0f;
}
// Signed int8 in byte i of w: bias by 128 first (w ^ 0x80 per byte), then remove
// 2^23 + 128.
__device__ __forceinline__ float sbyte_biased_to_f(uint32_t wb, int i) {
    return __uint_as_float(__byte_perm(wb, 0x4B000000u, 0x7540u + (uint32_t)i)) - 8388736.0f;
}

// Q4_K 6-bit scale/min of sub-block j from the 12 packed bytes (restates
// src/kernels.cpp:65-73): j<4: sc=q[j]&63, m=q[j+4]&63; j>=4: sc=(q[j+4]&15)|((q[j-4]>>6)<<4),
// m=(q[j+4]>>4)|((q[j]>>6)<<4).
__device__ __forceinline__ void q4k_sc_m(const uint8_t* q, int j, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// The same, with the 12 packed scale bytes as three little-endian words (bytes
// 0-3, 4-7, 8-11): register-only, no byte array to index.
__device__ __forceinline__ void q4k_sc_m_words(uint32_t w0, uint32_t w1, uint32_t w2, int j, int& sc, int& m) {
    const int sh = 8 * (j & 3);
    const int b0 = (int)((w0 >> sh) & 0xFFu), b1 = (int)((w1 >> sh) & 0xFFu), b2 = (int)((w2 >> sh) & 0xFFu);
    if (j < 4) {
        sc = b0 & 63;  // q[j]
        m = b1 & 63;   // q[j + 4]
    } else {
        sc = (b2 & 15) | ((b0 >> 6) << 4);  // q[j + 4], q[j - 4]
        m = (b2 >> 4) | ((b1 >> 6) << 4);   // q[j + 4], q[j]
    }
}

// One 32-value block of an input row into its integer form (see QInput):
// writes q1[0..32), q0[0..32), *sx and s16[0..2). Called by one thread.
__device__ __forceinline__ void qinput_block(const float* x, int8_t* q1, int8_t* q0, float* sx, float* s16) {
    float v[32];
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 f = *reinterpret_cast<const float4*>(x + i);
        v[i] = f.x;
        v[i + 1] = f.y;
        v[i + 2] = f.z;
        v[i + 3] = f.w;
    }
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) a += v[i];
#pragma unroll
    for (int i = 16; i < 32; ++i) b += v[i];
    s16[0] = a;
    s16[1] = b;
#pragma unroll
    for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
    const float inv = mx > 0.f ? 16383.0f / mx : 0.f;
    *sx = mx / 16383.0f;
    uint32_t w1[8], w0[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
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
    uint4* d1 = reinterpret_cast<uint4*>(q1);
    uint4* d0 = reinterpret_cast<uint4*>(q0);
    d1[0] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
    d1[1] = make_uint4(w1[4], w1[5], w1[6], w1[7]);
    d0[0] = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    d0[1] = make_uint4(w0[4], w0[5], w0[6], w0[7]);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

// A chunk decoded into registers: its values in column order of two 16-column
// runs (Q4_K: lo run and hi run; Q8_0: one run of 16 in v[0..15]), plus the
// affine coefficients that turn a dot with q into a dot with the weights:
//   Q8_0: dot = a0 * sum(v[0..16) * x)
//   Q4_K: dot = a0 * sum(lo*x_lo) - b0 * sum(x_lo) + a1 * sum(hi*x_hi) - b1 * sum(x_hi)
struct Chunk {
    float v[32];
    float a0, b0, a1, b1;
    int col_lo, col_hi;
};

template <int DT>
__device__ __forceinline__ void chunk_load(const QMat& m, const uint8_t* row_qs, const uint8_t* row_meta,
                                           int c, uint4& raw, uint4& meta) {
    raw = ld_stream16(row_qs + (int64_t)c * 16);
    if (DT == AERO_DT_Q4_K) {
        meta = __ldg(reinterpret_cast<const uint4*>(row_meta + (int64_t)(c >> 3) * 16));
    } else if (DT == AERO_DT_Q8_0) {
        meta.x = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(row_meta) + (c >> 1));
    }
}

template <int DT>
__device__ __forceinline__ void chunk_decode(int c, const uint4& raw, const uint4& meta, Chunk& k) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    if (DT == AERO_DT_Q8_0) {
        const float d = __half2float(__ushort_as_half((unsigned short)meta.x));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t wb = w[i] ^ 0x80808080u;
#pragma unroll
            for (int b = 0; b < 4; ++b) k.v[4 * i + b] = sbyte_biased_to_f(wb, b);
        }
        k.a0 = d;
        k.b0 = k.a1 = k.b1 = 0.f;
        k.col_lo = c * 16;
        k.col_hi = 0;
    } else if (DT == AERO_DT_Q4_K) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                k.v[4 * i + b] = ubyte_to_f(lo, b);
                k.v[16 + 4 * i + b] = ubyte_to_f(hi, b);
            }
        }
        const uint8_t* mb = reinterpret_cast<const uint8_t*>(&meta);
        const float d = __half2float(__ushort_as_half((unsigned short)(mb[0] | (mb[1] << 8))));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(mb[2] | (mb[3] << 8))));
        const int g = (c >> 1) & 3, hh = c & 1, s = c >> 3;
        int sc0, m0, sc1, m1;
        q4k_sc_m(mb + 4, 2 * g, sc0, m0);
        q4k_sc_m(mb + 4, 2 * g + 1, sc1, m1);
        k.a0 = d * (float)sc0;
        k.b0 = dmin * (float)m0;
        k.a1 = d * (float)sc1;
        k.b1 = dmin * (float)m1;
        k.col_lo = s * 256 + g * 64 + hh * 16;
        k.col_hi = k.col_lo + 32;
    } else {
        k.v[0] = __uint_as_float(w[0]);
        k.v[1] = __uint_as_float(w[1]);
        k.v[2] = __uint_as_float(w[2]);
        k.v[3] = __uint_as_float(w[3]);
        k.a0 = 1.f;
        k.b0 = k.a1 = k.b1 = 0.f;
        k.col_lo = c * 4;
        k.col_hi = 0;
    }
}

// Dot of a decoded chunk with the matching columns of x (f32 row) — xs16 holds
// sums of x over aligned 16-column groups (used by Q4_K's min term).
template <int DT>
__device__ __forceinline__ float chunk_dot(const Chunk& k, const float* x, const float* xs16) {
    if (DT == AERO_DT_Q8_0) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 xv = ld_f4(x + k.col_lo + i);
            s = fmaf(k.v[i], xv.x, s);
            s = fmaf(k.v[i + 1], xv.y, s);
            s = fmaf(k.v[i + 2], xv.z, s);
            s = fmaf(k.v[i + 3], xv.w, s);
        }
        return k.a0 * s;
    } else if (DT == AERO_DT_Q4_K) {
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
            const float4 xl = ld_f4(x + k.col_lo + i);
            const float4 xh = ld_f4(x + k.col_hi + i);
            s0 = fmaf(k.v[i], xl.x, s0);
            s0 = fmaf(k.v[i + 1], xl.y, s0);
            s0 = fmaf(k.v[i + 2], xl.z, s0);
            s0 = fmaf(k.v[i + 3], xl.w, s0);
            s1 = fmaf(k.v[16 + i], xh.x, s1);
            s1 = fmaf(k.v[16 + i + 1], xh.y, s1);
            s1 = fmaf(k.v[16 + i + 2], xh.z, s1);
            s1 = fmaf(k.v[16 + i + 3], xh.w, s1);
        }
        const float sx0 = __ldg(xs16 + (k.col_lo >> 4)), sx1 = __ldg(xs16 + (k.col_hi >> 4));
        return (k.a0 * s0 - k.b0 * sx0) + (k.a1 * s1 - k.b1 * sx1);
    } else {
        const float4 xv = ld_f4(x + k.col_lo);
        float s = k.v[0] * xv.x;
        s = fmaf(k.v[1], xv.y, s);
        s = fmaf(k.v[2], xv.z, s);
        s = fmaf(k.v[3], xv.w, s);
        return s;
    }
}

#endif  // __CUDACC__

#define AERO_CUDA_CHECK(expr)                                                    \
    do {                                                                         \
        cudaError_t _e = (expr);                                                 \
        if (_e != cudaSuccess) return _e;                                        \
    } while (0)
