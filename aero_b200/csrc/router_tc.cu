// Router projection for prefill batches on the tensor cores.
//
// logits[t][e] = x_t . W[e] (+ bias[e]) for the E router rows (the reference's
// caller-side router, engine/model.py:665-666, an f32 GEMM). FP32 accuracy on
// TF32 tensor cores by operand splitting: every f32 value v is written as
// hi + lo with hi = v rounded to TF32 (10 mantissa bits) and lo = v - hi
// (exact in f32), and the product is accumulated in f32 as
//   x_hi W_hi + x_hi W_lo + x_lo W_hi
// (the x_lo W_lo term is below f32 resolution). W's split is made once at open;
// x is split in shared memory as it arrives.
//
// The tensor core's accumulation into TMEM rounds toward zero, so the error of
// a long accumulation chain grows with its length (one step per MMA). The
// chains are kept short: the hi x hi products of even and odd K stages go to
// two accumulators and the small hi x lo / lo x hi terms to a third; the
// epilogue adds the three in f32.
//
// One CTA per 128 tokens x N router rows (N <= 128; three TMEM accumulators of
// N f32 columns), K in stages of 32 values (128-byte rows, 128B swizzle), three
// stages:
//   warp 0      TMA producer: x tile (128 rows) and the W_hi / W_lo tiles
//   warp 1      one thread issues the 3 x 4 MMAs of a stage (128 x N x 8 each)
//   warps 2-5   split the x tile in place (hi) and into the lo buffer, then
//               the epilogue: TMEM -> registers (+ bias) -> logits rows
// The CTAs of the first column tile also compute the shared-expert gate column
// (x . g over K in stage order) on the split warps, which touch every x value.
// Batches too small to cover the SMs split K over up to 8 CTA layers (grid z);
// each layer writes its partial logits and router_reduce_kernel adds the
// layers in order, then the bias (deterministic for a given batch size).
// Every mbarrier wait is bounded; a CTA that gives up records an error code and
// drains its issued MMAs before freeing TMEM.
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.h"
#include "internal.h"
#include "tc_common.cuh"

namespace aero {
namespace {

constexpr int kRtM = 128;
constexpr int kRtK = 32;  // f32 values per stage row (128 bytes)
constexpr int kRtStages = 3;
constexpr int kRtThreads = 192;
constexpr uint32_t kRtXBytes = kRtM * kRtK * 4;          // 16 KiB
constexpr uint32_t kRtWBytes = kRtNMax * kRtK * 4;       // 16 KiB
constexpr uint32_t kRtStageBytes = 2 * kRtXBytes + 2 * kRtWBytes;  // x (hi in place), x lo, W hi, W lo
constexpr uint32_t kRtTmemCols = 512;  // accumulators at columns 0 (even hi x hi), 128 (odd), 256 (corrections)
constexpr size_t kRtSmem = (size_t)kRtStages * kRtStageBytes + 1024 + 256;

enum : int { kRtErrFull = 11, kRtErrSplit = 12, kRtErrEmpty = 13, kRtErrAcc = 14 };

struct RouterTcParams {
    int T, K;          // tokens, reduction length of one K split (dp / splits)
    int n_rows, N;     // router rows on the tensor cores; rows per CTA tile
    const float* bias;
    int n_bias;
    const float* gate_row;  // shared-gate input (K) or null; its logit goes to column n_rows
    float* logits;
    int ld;
    int32_t* err;
    int32_t* err_host; // host-mapped copy of the first code (read by the host without synchronising), or null
    float* partial;    // split K: per-split logits [split][T][ld] (no bias), summed by router_reduce_kernel
};

__device__ __forceinline__ float tf32_hi(float v) {
    return __uint_as_float((__float_as_uint(v) + 0x1000u) & 0xFFFFE000u);
}

__global__ void __launch_bounds__(kRtThreads, 1) router_tc_kernel(const __grid_constant__ CUtensorMap tx,
                                                                  const __grid_constant__ CUtensorMap twh,
                                                                  const __grid_constant__ CUtensorMap twl,
                                                                  RouterTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRtStages * kRtStageBytes);
    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto split = [&](int s) { return bar0 + 8u * (kRtStages + s); };
    auto empty = [&](int s) { return bar0 + 8u * (2 * kRtStages + s); };
    const uint32_t acc_full = bar0 + 8u * (3 * kRtStages), drain_bar = bar0 + 8u * (3 * kRtStages + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * kRtStages + 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kRtStages + 3);
    auto xh = [&](int s) { return smem + s * kRtStageBytes; };
    auto xl = [&](int s) { return smem + s * kRtStageBytes + kRtXBytes; };
    auto wh = [&](int s) { return smem + s * kRtStageBytes + 2 * kRtXBytes; };
    auto wl = [&](int s) { return smem + s * kRtStageBytes + 2 * kRtXBytes + kRtWBytes; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * kRtM, n0 = blockIdx.y * p.N;
    const int nk = p.K / kRtK;
    const int kbase = (int)blockIdx.z * p.K;  // this CTA's K split
    const uint32_t tmem_cols = kRtTmemCols;
    auto fail = [&](int code) {
        *abort_flag = 1;
        if (atomicCAS(p.err, 0, code) == 0 && p.err_host) {
            *reinterpret_cast<volatile int32_t*>(p.err_host) = code;
            __threadfence_system();
        }
    };
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRtStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(split(s), 4);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------- TMA producer
            const uint32_t bytes = kRtXBytes + 2u * (uint32_t)p.N * kRtK * 4u;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kRtStages;
                if (kb >= kRtStages && !mbar_wait(empty(s), ((kb / kRtStages) - 1) & 1, abort_flag)) {
                    fail(kRtErrEmpty);
                    break;
                }
                mbar_expect_tx(full(s), bytes);
                tma_load_2d(smem_u32(xh(s)), &tx, kbase + kb * kRtK, m0, full(s));
                tma_load_2d(smem_u32(wh(s)), &twh, kbase + kb * kRtK, n0, full(s));
                tma_load_2d(smem_u32(wl(s)), &twl, kbase + kb * kRtK, n0, full(s));
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------- MMA issuer
            const uint32_t idesc = idesc_tf32(kRtM, p.N);
            bool issued = false, ok = true;
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % kRtStages;
                if (!mbar_wait(split(s), (kb / kRtStages) & 1, abort_flag)) {
                    fail(kRtErrSplit);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ah = smem_u32(xh(s)), al = smem_u32(xl(s)), bh = smem_u32(wh(s)), bl = smem_u32(wl(s));
                const uint32_t d_main = tmem + (uint32_t)(kb & 1) * 128u, d_corr = tmem + 256u;
#pragma unroll
                for (int kk = 0; kk < kRtK / 8; ++kk) {
                    const uint32_t acc_main = (kb > 1 || kk > 0) ? 1u : 0u;
                    const uint32_t acc_corr = (kb > 0 || kk > 0) ? 1u : 0u;
                    umma_tf32_ss(d_main, sw128_desc(ah + kk * 32), sw128_desc(bh + kk * 32), idesc, acc_main);
                    umma_tf32_ss(d_corr, sw128_desc(ah + kk * 32), sw128_desc(bl + kk * 32), idesc, acc_corr);
                    umma_tf32_ss(d_corr, sw128_desc(al + kk * 32), sw128_desc(bh + kk * 32), idesc, 1u);
                }
                issued = true;
                umma_commit(empty(s));
            }
            if (ok) {
                umma_commit(acc_full);
            } else if (issued) {
                umma_commit(drain_bar);  // MMAs in flight must finish before TMEM is freed
                mbar_wait_timed(drain_bar, 0);
            }
        }
    } else {
        // -------------------------------------------- split, then epilogue
        const int q = warp & 3;
        const int r = q * 32 + lane;  // tile row = TMEM lane
        const bool do_gate = p.gate_row != nullptr && blockIdx.y == 0;
        float g_acc = 0.f;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % kRtStages;
            const bool got = __all_sync(0xffffffffu, mbar_wait(full(s), (kb / kRtStages) & 1, abort_flag));
            if (!got) {
                if (lane == 0) fail(kRtErrFull);
                ok = false;
                break;
            }
            uint8_t* hrow = xh(s) + r * 128;
            uint8_t* lrow = xl(s) + r * 128;
            const float* g = do_gate ? p.gate_row + kbase + kb * kRtK : nullptr;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int off = (c ^ (r & 7)) << 4;  // 128B swizzle: logical chunk c of row r
                float4 v = *reinterpret_cast<float4*>(hrow + off);
                if (do_gate) {
                    const float4 gv = __ldg(reinterpret_cast<const float4*>(g + 4 * c));
                    g_acc = fmaf(v.x, gv.x, g_acc);
                    g_acc = fmaf(v.y, gv.y, g_acc);
                    g_acc = fmaf(v.z, gv.z, g_acc);
                    g_acc = fmaf(v.w, gv.w, g_acc);
                }
                const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
                *reinterpret_cast<float4*>(lrow + off) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
                *reinterpret_cast<float4*>(hrow + off) = h;
            }
            fence_proxy_async();
            __syncwarp();
            if (lane == 0) mbar_arrive(split(s));
        }
        const int row = m0 + r;
        if (ok) {
            const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full, 0, abort_flag));
            if (!got) {
                if (lane == 0) fail(kRtErrAcc);
            } else {
                tc_fence_after();
                const uint32_t lane_base = (uint32_t)(q * 32) << 16;
                // split K: this split's partial sums, reduced (with the bias) by a second kernel
                const bool part = p.partial != nullptr;
                float* dst = part ? p.partial + (size_t)blockIdx.z * p.T * p.ld : p.logits;
                const float* bias = part ? nullptr : p.bias;
                float* out = dst + (int64_t)row * p.ld + n0;
                for (int c0 = 0; c0 < p.N; c0 += 16) {
                    uint32_t v0[16], v1[16], vc[16];
                    tmem_ld16(tmem + lane_base + (uint32_t)c0, v0);
                    tmem_ld16(tmem + lane_base + 128u + (uint32_t)c0, v1);
                    tmem_ld16(tmem + lane_base + 256u + (uint32_t)c0, vc);
                    tmem_wait_ld();
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        v[j] = (__uint_as_float(v0[j]) + (nk > 1 ? __uint_as_float(v1[j]) : 0.f)) + __uint_as_float(vc[j]);
                    if (row < p.T) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const int e = n0 + c0 + j;
                            float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                            if (bias) {
                                if (e < p.n_bias) o.x += bias[e];
                                if (e + 1 < p.n_bias) o.y += bias[e + 1];
                                if (e + 2 < p.n_bias) o.z += bias[e + 2];
                                if (e + 3 < p.n_bias) o.w += bias[e + 3];
                            }
                            *reinterpret_cast<float4*>(out + c0 + j) = o;
                        }
                    }
                }
                if (do_gate && row < p.T) dst[(int64_t)row * p.ld + p.n_rows] = g_acc;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols));
    }
}

// logits[t][c] = sum over splits (in order) of partial[s][t][c] (+ bias[c] for c < n_bias),
// for c < cols (the router rows and, when present, the shared-gate column).
__global__ void router_reduce_kernel(const float* __restrict__ partial, int splits, int T, int ld, int cols,
                                     const float* __restrict__ bias, int n_bias, float* __restrict__ logits) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (c >= cols) return;
    float v = 0.f;
    for (int sp = 0; sp < splits; ++sp) v += partial[((size_t)sp * T + t) * ld + c];
    if (bias && c < n_bias) v += bias[c];
    logits[(int64_t)t * ld + c] = v;
}

__global__ void split_tf32_kernel(const float* __restrict__ in, int64_t n, float* __restrict__ hi,
                                  float* __restrict__ lo) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = in[i], h = tf32_hi(v);
    hi[i] = h;
    lo[i] = v - h;
}

}  // namespace

int router_tc_tile_rows(int n_rows) {
    if (n_rows <= 0 || n_rows % 16 != 0) return 0;
    if (n_rows <= kRtNMax) return n_rows;
    // equal tiles of at most kRtNMax rows, a multiple of 16 each
    const int tiles = (n_rows + kRtNMax - 1) / kRtNMax;
    const int N = (n_rows / 16 + tiles - 1) / tiles * 16;
    return n_rows % N == 0 ? N : 0;
}

cudaError_t router_tc_prepare(const float* W, int n_rows, int dp, float* w_hi, float* w_lo, RouterTcMaps* maps,
                              cudaStream_t s) {
    const int N = router_tc_tile_rows(n_rows);
    if (N == 0 || dp % kRtK != 0) return cudaErrorInvalidValue;
    const int64_t n = (int64_t)n_rows * dp;
    split_tf32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(W, n, w_hi, w_lo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    maps->N = N;
    maps->n_rows = n_rows;
    maps->dp = dp;
    const bool ok = encode_tmap_2d(&maps->hi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, w_hi, (uint64_t)n_rows, (uint64_t)dp,
                                   (uint64_t)dp, (uint32_t)N, kRtK, CU_TENSOR_MAP_SWIZZLE_128B) &&
                    encode_tmap_2d(&maps->lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, w_lo, (uint64_t)n_rows, (uint64_t)dp,
                                   (uint64_t)dp, (uint32_t)N, kRtK, CU_TENSOR_MAP_SWIZZLE_128B);
    return ok ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_router_tc(const RouterTcMaps& maps, const float* x, int T, const float* bias, int n_bias,
                             const float* gate_row, float* logits, int ld, int32_t* err, int32_t* err_host,
                             float* partial, int partial_rows, int n_sm, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if ((ld & 3) || ((uintptr_t)logits & 15)) return cudaErrorInvalidValue;
    CUtensorMap tx;
    if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, (uint64_t)T, (uint64_t)maps.dp, (uint64_t)maps.dp,
                        kRtM, kRtK, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        const cudaError_t e =
            cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRtSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    // small batches: split K over up to 8 CTA layers (one CTA per SM), taking
    // the split count with the fewest K blocks per SM, fewer splits on ties
    // (each split writes partial logits; a second kernel adds them in order)
    const int tiles = ((T + kRtM - 1) / kRtM) * (maps.n_rows / maps.N);
    int splits = 1;
    auto work = [&](int sp) { return (int64_t)((tiles * sp + n_sm - 1) / n_sm) * (maps.dp / sp); };
    // (a split keeps at least two K blocks: the two main accumulators alternate per block)
    for (int sp = 2; partial && sp <= 8; sp *= 2)
        if (maps.dp % (sp * kRtK) == 0 && maps.dp / sp >= 2 * kRtK && (int64_t)sp * T <= partial_rows &&
            work(sp) < work(splits))
            splits = sp;
    RouterTcParams p{};
    p.T = T;
    p.K = maps.dp / splits;
    p.partial = splits > 1 ? partial : nullptr;
    p.n_rows = maps.n_rows;
    p.N = maps.N;
    p.bias = bias;
    p.n_bias = n_bias;
    p.gate_row = gate_row;
    p.logits = logits;
    p.ld = ld;
    p.err = err;
    p.err_host = err_host;
    dim3 grid((T + kRtM - 1) / kRtM, maps.n_rows / maps.N, splits);
    router_tc_kernel<<<grid, kRtThreads, kRtSmem, s>>>(tx, maps.hi, maps.lo, p);
    if (splits > 1) {
        const int cols = maps.n_rows + (gate_row ? 1 : 0);
        router_reduce_kernel<<<dim3((cols + 127) / 128, T), 128, 0, s>>>(partial, splits, T, ld, cols, bias, n_bias,
                                                                         logits);
    }
    return cudaGetLastError();
}

}  // namespace aero
