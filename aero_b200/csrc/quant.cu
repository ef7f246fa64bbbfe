// Device-side GGUF block work: repack into the SoA expert planes, exact
// dequantisation, and the block quantisers.
//
// Dequantisation restates src/kernels.cpp:337-373 (engine/quant.py:133-181)
// with the same single-rounding f32 operations (products and differences are
// written with __fmul_rn / __fsub_rn so the compiler cannot fuse them into an
// FMA), which makes it bit-identical to the reference's fp32 values.
//
// The quantisers restate the rules documented in aero_b200/quant.py with the
// same IEEE operations, so host and device produce identical bytes.
#include "internal.h"

namespace aero {
namespace {

__device__ __forceinline__ float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// ------------------------------------------------------------------ repack
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ src, int64_t n_rows, int cols, int rows_per_expert,
                                   int64_t expert0, uint8_t* __restrict__ qs, uint8_t* __restrict__ meta,
                                   int64_t qs_es, int64_t meta_es) {
    const int bpr = cols / 32;
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= n_rows * bpr) return;
    const int64_t row = blk / bpr;
    const int b = (int)(blk % bpr);
    const uint8_t* s = src + blk * 34;
    const int64_t e = expert0 + row / rows_per_expert, r = row % rows_per_expert;
    uint8_t* dq = qs + e * qs_es + r * (int64_t)cols + b * 32;
    uint8_t* dm = meta + e * meta_es + r * (int64_t)bpr * 2 + b * 2;
    dm[0] = s[0];
    dm[1] = s[1];
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        w[i] = (uint32_t)s[2 + 4 * i] | ((uint32_t)s[3 + 4 * i] << 8) | ((uint32_t)s[4 + 4 * i] << 16) |
               ((uint32_t)s[5 + 4 * i] << 24);
    reinterpret_cast<uint4*>(dq)[0] = make_uint4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<uint4*>(dq)[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void repack_q4_k_kernel(const uint8_t* __restrict__ src, int64_t n_rows, int cols, int rows_per_expert,
                                   int64_t expert0, uint8_t* __restrict__ qs, uint8_t* __restrict__ meta,
                                   int64_t qs_es, int64_t meta_es) {
    const int bpr = cols / 256;
    const int64_t blk = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (blk >= n_rows * bpr) return;
    const int64_t row = blk / bpr;
    const int b = (int)(blk % bpr);
    const uint4* s = reinterpret_cast<const uint4*>(src + blk * 144);  // 144 = 9 x 16, source 16-B aligned
    const int64_t e = expert0 + row / rows_per_expert, r = row % rows_per_expert;
    uint4* dq = reinterpret_cast<uint4*>(qs + e * qs_es + (r * bpr + b) * 128);
    uint4* dm = reinterpret_cast<uint4*>(meta + e * meta_es + (r * bpr + b) * 16);
    dm[0] = s[0];
#pragma unroll
    for (int i = 0; i < 8; ++i) dq[i] = s[1 + i];
}

// ------------------------------------------------------------------ dequant
__global__ void dequant_q8_0_kernel(const uint8_t* __restrict__ src, int64_t nb, float* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const uint8_t* s = src + b * 34;
    const float d = h2f_bits((uint16_t)(s[0] | (s[1] << 8)));
    for (int i = 0; i < 32; ++i) out[b * 32 + i] = __fmul_rn(d, (float)(int8_t)s[2 + i]);
}

__global__ void dequant_q4_k_kernel(const uint8_t* __restrict__ src, int64_t nb, float* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const uint8_t* s = src + b * 144;
    const float d = h2f_bits((uint16_t)(s[0] | (s[1] << 8)));
    const float dmin = h2f_bits((uint16_t)(s[2] | (s[3] << 8)));
    float* o = out + b * 256;
    for (int g = 0; g < 4; ++g) {
        int s1, m1, s2, m2;
        q4k_sc_m(s + 4, 2 * g, s1, m1);
        q4k_sc_m(s + 4, 2 * g + 1, s2, m2);
        const float f1 = __fmul_rn(d, (float)s1), g1 = __fmul_rn(dmin, (float)m1);
        const float f2 = __fmul_rn(d, (float)s2), g2 = __fmul_rn(dmin, (float)m2);
        for (int i = 0; i < 32; ++i) {
            const uint8_t q = s[16 + 32 * g + i];
            o[64 * g + i] = __fsub_rn(__fmul_rn(f1, (float)(q & 15)), g1);
            o[64 * g + 32 + i] = __fsub_rn(__fmul_rn(f2, (float)(q >> 4)), g2);
        }
    }
}

__global__ void f16_to_f32_kernel(const uint16_t* __restrict__ in, int64_t n, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = h2f_bits(in[i]);
}

// ------------------------------------------------------------------ quantise
// round half away from zero, as floor(a) + floor(2 (a - floor(a))) with sign
__device__ __forceinline__ float rnd_away(float v) {
    const float a = fabsf(v);
    const float f = floorf(a);
    const float r = __fadd_rn(f, floorf(__fmul_rn(2.0f, __fsub_rn(a, f))));
    return v < 0.f ? -r : (v > 0.f ? r : 0.f * r);
}

__global__ void quantize_q8_0_kernel(const float* __restrict__ x, int64_t nb, uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const float* xb = x + b * 32;
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(xb[i]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d == 0.f ? 0.f : __fdiv_rn(1.0f, d);
    // the 34-byte block is 2-byte aligned: write it as 17 little-endian u16 words
    unsigned short* o = reinterpret_cast<unsigned short*>(out + b * 34);
    o[0] = __half_as_ushort(__float2half_rn(d));
    for (int i = 0; i < 32; i += 2) {
        const uint32_t q0 = (uint32_t)(uint8_t)(int8_t)(int)rnd_away(__fmul_rn(xb[i], id));
        const uint32_t q1 = (uint32_t)(uint8_t)(int8_t)(int)rnd_away(__fmul_rn(xb[i + 1], id));
        o[1 + i / 2] = (unsigned short)(q0 | (q1 << 8));
    }
}

__global__ void quantize_q4_k_kernel(const float* __restrict__ x, int64_t nb, uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nb) return;
    const float* xb = x + b * 256;
    float span[8], mval[8];
    float dmax = 0.f, mmax = 0.f;
    for (int j = 0; j < 8; ++j) {
        float lo = xb[32 * j], hi = xb[32 * j];
        for (int i = 1; i < 32; ++i) {
            lo = fminf(lo, xb[32 * j + i]);
            hi = fmaxf(hi, xb[32 * j + i]);
        }
        lo = fminf(lo, 0.f);
        span[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        mval[j] = -lo;
        dmax = j == 0 ? span[j] : fmaxf(dmax, span[j]);
        mmax = j == 0 ? mval[j] : fmaxf(mmax, mval[j]);
    }
    const float d = __fdiv_rn(dmax, 63.0f), dmin = __fdiv_rn(mmax, 63.0f);
    const __half d16 = __float2half_rn(d), dm16 = __float2half_rn(dmin);
    const float dq = __half2float(d16), dmq = __half2float(dm16);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = dq > 0.f ? (int)fminf(rnd_away(__fdiv_rn(span[j], dq)), 63.f) : 0;
        mn[j] = dmq > 0.f ? (int)fminf(rnd_away(__fdiv_rn(mval[j], dmq)), 63.f) : 0;
    }
    uint8_t* o = out + b * 144;
    const uint16_t db = __half_as_ushort(d16), mb = __half_as_ushort(dm16);
    o[0] = (uint8_t)(db & 0xFF);
    o[1] = (uint8_t)(db >> 8);
    o[2] = (uint8_t)(mb & 0xFF);
    o[3] = (uint8_t)(mb >> 8);
    for (int j = 0; j < 4; ++j) {
        o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        o[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        o[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    for (int g = 0; g < 4; ++g) {
        int qv[2][32];
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * g + h;
            const float es = __fmul_rn(dq, (float)sc[j]);
            const float em = __fmul_rn(dmq, (float)mn[j]);
            for (int i = 0; i < 32; ++i) {
                int q = 0;
                if (es > 0.f) {
                    const float r = rnd_away(__fdiv_rn(__fadd_rn(xb[32 * j + i], em), es));
                    q = (int)fminf(fmaxf(r, 0.f), 15.f);
                }
                qv[h][i] = q;
            }
        }
        for (int i = 0; i < 32; ++i) o[16 + 32 * g + i] = (uint8_t)(qv[0][i] | (qv[1][i] << 4));
    }
}

}  // namespace

cudaError_t launch_repack(int dtype, const uint8_t* gguf, int64_t n_rows_total, int cols, int rows_per_expert,
                          int64_t expert0, uint8_t* qs, uint8_t* meta, int64_t qs_estride, int64_t meta_estride,
                          cudaStream_t s) {
    if (dtype == AERO_DT_Q8_0) {
        const int64_t nb = n_rows_total * (cols / 32);
        repack_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(gguf, n_rows_total, cols, rows_per_expert,
                                                                       expert0, qs, meta, qs_estride, meta_estride);
    } else if (dtype == AERO_DT_Q4_K) {
        const int64_t nb = n_rows_total * (cols / 256);
        repack_q4_k_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(gguf, n_rows_total, cols, rows_per_expert,
                                                                       expert0, qs, meta, qs_estride, meta_estride);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant_gguf(int dtype, const uint8_t* gguf, int64_t n_values, float* out, cudaStream_t s) {
    if (dtype == AERO_DT_Q8_0) {
        const int64_t nb = n_values / 32;
        dequant_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(gguf, nb, out);
    } else if (dtype == AERO_DT_Q4_K) {
        const int64_t nb = n_values / 256;
        dequant_q4_k_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, s>>>(gguf, nb, out);
    } else if (dtype == AERO_DT_F32) {
        return cudaMemcpyAsync(out, gguf, (size_t)n_values * 4, cudaMemcpyDeviceToDevice, s);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_quantize(int dtype, const float* x, int64_t n_values, uint8_t* out, cudaStream_t s) {
    if (dtype == AERO_DT_Q8_0) {
        const int64_t nb = n_values / 32;
        quantize_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(x, nb, out);
    } else if (dtype == AERO_DT_Q4_K) {
        const int64_t nb = n_values / 256;
        quantize_q4_k_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, s>>>(x, nb, out);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_f16_to_f32(const uint16_t* in, int64_t n, float* out, cudaStream_t s) {
    if (n <= 0) return cudaSuccess;
    f16_to_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in, n, out);
    return cudaGetLastError();
}

}  // namespace aero
