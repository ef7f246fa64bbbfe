// Prefill: grouped expert GEMMs on the 5th-generation tensor cores.
//
// Per routed expert segment (token rows sorted by expert) and for the shared
// expert (all tokens), two grouped GEMMs in "weights x tokens" orientation, so
// the 128-row MMA M extent runs over weight rows and the ragged token count is
// the N extent (16..256 in steps of 16; nothing is padded to 128 tokens):
//   gate/up:  D_g = Wg[m0:m0+128, :] . X^T,  D_u = Wu[...] . X^T  (K = d)
//             epilogue: act = silu(D_g) * D_u  -> f16 act rows
//   down:     D = Wd[n0:n0+128, :] . act^T (K = F)  -> f16 y rows
// Operands are f16 (kind::f16, fp32 accumulate). bf16 operands were measured
// (and reproduced by a numpy model of the same roundings) at 2.6% of the output
// RMS in max-abs error on Q4_K layers, above the 1% bar; f16 rounds 8x finer at
// the same tensor-core rate and measures 0.26%.
// One CTA computes one (tile, 128-row block). Warp roles, 10 warps:
//   warp 0     TMA producer of the token operand (cp.async.bulk.tensor, 128B
//              swizzle, no multicast) and owner of the TMEM allocation
//   warp 1     one elected thread issues tcgen05.mma (kind::f16, f16 inputs,
//              fp32 accumulators in TMEM) and tcgen05.commit
//   warps 2-9  stream the expert's Q4_K / Q8_0 blocks with 16-byte loads,
//              dequantise in registers (f32 w = s*q - m, then f16) and store
//              the tile in the canonical K-major SWIZZLE_128B layout; warps 4-7
//              then run the epilogue from TMEM (tcgen05.ld 32x32b)
// Stages are double/triple buffered through mbarriers. Every wait is bounded by
// %globaltimer (2 s); on expiry the CTA records an error code, drains its own
// copies and MMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <cub/block/block_scan.cuh>
#include <string>

#include "gemm.h"
#include "internal.h"

namespace aero {
namespace {

constexpr int kBK = 64;                        // K per stage: 64 f16 = one 128-byte swizzle row
constexpr int kTileM = 128;
constexpr int kThreads = 320;
constexpr int kDeqThreads = 256;
constexpr uint32_t kABytes = kTileM * kBK * 2;  // 16 KiB per weight operand per stage
constexpr uint32_t kBBytes = kGemmNT * kBK * 2; // 32 KiB token operand per stage
constexpr uint64_t kWaitNs = 2000000000ull;

enum : int { kErrFullA = 1, kErrFullB = 2, kErrEmpty = 3, kErrAcc = 4 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait that ignores the abort flag (used to drain this thread's own copies).
__device__ bool mbar_wait_timed(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = gtimer();
    while (!mbar_try(bar, parity))
        if (gtimer() - t0 > kWaitNs) return false;
    return true;
}
// Bounded wait: false on timeout or when another role of this CTA gave up.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
        if (gtimer() - t0 > kWaitNs) return false;
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// K-major operand, SWIZZLE_128B: 8-row groups 1024 bytes apart (SBO), leading
// offset unused, descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: f32 accumulate, f16 A and B (format 0), both
// K-major.
__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// byte offset of 16-byte chunk c (0..7) of row r inside a SWIZZLE_128B tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
}

struct GemmParams {
    QMat A0, A1;          // routed: gate, up (gate/up GEMM) or down
    QMat S0, S1;          // shared expert
    const GemmTile* tiles;
    const int32_t* n_tiles;
    int K, Ks;            // reduction length for routed / shared tiles
    int MT, MTs, MTmax;   // 128-row blocks for routed / shared
    __half* out;
    int out_ld;
    int32_t* err;
};

// Raw quant data one dequant thread needs for one stage and one matrix.
struct Raw {
    uint4 q0, q1;   // Q4_K: q0; Q8_0: q0, q1 (32 int8)
    uint4 meta;     // Q4_K: 16-byte header; Q8_0: .x = fp16 scale
};

template <int DT>
__device__ __forceinline__ void raw_load(const QMat& m, int e, int row, int kb, int h, Raw& r) {
    const uint8_t* qrow = qm_row_qs(m, e, row);
    const uint8_t* mrow = qm_row_meta(m, e, row);
    const int k0 = kb * kBK;
    if (DT == AERO_DT_Q4_K) {
        const int sb = k0 >> 8, g = (k0 >> 6) & 3;
        r.q0 = ld_stream16(qrow + sb * 128 + g * 32 + h * 16);
        r.meta = __ldg(reinterpret_cast<const uint4*>(mrow + sb * 16));
    } else {
        const int blk = (k0 >> 5) + h;
        r.q0 = ld_stream16(qrow + blk * 32);
        r.q1 = ld_stream16(qrow + blk * 32 + 16);
        r.meta.x = (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(mrow) + blk);
    }
}

// Dequantise and store one thread's share (row r, half h) of a 128 x 64 tile.
template <int DT>
__device__ __forceinline__ void raw_store(const Raw& raw, int kb, int r, int h, uint8_t* tile) {
    if (DT == AERO_DT_Q4_K) {
        const uint8_t* mb = reinterpret_cast<const uint8_t*>(&raw.meta);
        const float d = __half2float(__ushort_as_half((unsigned short)(mb[0] | (mb[1] << 8))));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(mb[2] | (mb[3] << 8))));
        const int g = (kb & 3);
        int sc0, m0, sc1, m1;
        q4k_sc_m(mb + 4, 2 * g, sc0, m0);
        q4k_sc_m(mb + 4, 2 * g + 1, sc1, m1);
        const float s0 = d * (float)sc0, n0 = -(dmin * (float)m0);
        const float s1 = d * (float)sc1, n1 = -(dmin * (float)m1);
        const uint32_t w[4] = {raw.q0.x, raw.q0.y, raw.q0.z, raw.q0.w};
        uint32_t lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t l = w[i] & 0x0F0F0F0Fu, u = (w[i] >> 4) & 0x0F0F0F0Fu;
            lo[2 * i] = pack_h2(fmaf(ubyte_to_f(l, 0), s0, n0), fmaf(ubyte_to_f(l, 1), s0, n0));
            lo[2 * i + 1] = pack_h2(fmaf(ubyte_to_f(l, 2), s0, n0), fmaf(ubyte_to_f(l, 3), s0, n0));
            hi[2 * i] = pack_h2(fmaf(ubyte_to_f(u, 0), s1, n1), fmaf(ubyte_to_f(u, 1), s1, n1));
            hi[2 * i + 1] = pack_h2(fmaf(ubyte_to_f(u, 2), s1, n1), fmaf(ubyte_to_f(u, 3), s1, n1));
        }
        // lo values are k = 16h .. 16h+15 (chunks 2h, 2h+1); hi are 32 + 16h .. (chunks 4+2h, 5+2h)
        *reinterpret_cast<uint4*>(tile + sw128_off(r, 2 * h)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(tile + sw128_off(r, 2 * h + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
        *reinterpret_cast<uint4*>(tile + sw128_off(r, 4 + 2 * h)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(tile + sw128_off(r, 5 + 2 * h)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
    } else {
        const float d = __half2float(__ushort_as_half((unsigned short)raw.meta.x));
        const uint32_t w[8] = {raw.q0.x, raw.q0.y, raw.q0.z, raw.q0.w, raw.q1.x, raw.q1.y, raw.q1.z, raw.q1.w};
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t wb = w[i] ^ 0x80808080u;
            o[2 * i] = pack_h2(d * sbyte_biased_to_f(wb, 0), d * sbyte_biased_to_f(wb, 1));
            o[2 * i + 1] = pack_h2(d * sbyte_biased_to_f(wb, 2), d * sbyte_biased_to_f(wb, 3));
        }
        // values k = 32h .. 32h+31: chunks 4h .. 4h+3
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(tile + sw128_off(r, 4 * h + c)) =
                make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
    }
}

template <int DT, bool GATEUP>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_b, GemmParams p) {
    constexpr int kStages = GATEUP ? 3 : 4;
    constexpr uint32_t kStage = (GATEUP ? 2 : 1) * kABytes + kBBytes;
    constexpr uint32_t kTmemCols = GATEUP ? 512 : 256;

    const int tile_i = blockIdx.x / p.MTmax, mt = blockIdx.x % p.MTmax;
    if (tile_i >= *p.n_tiles) return;
    const GemmTile t = p.tiles[tile_i];
    const bool shared = t.expert < 0;
    if (mt >= (shared ? p.MTs : p.MT)) return;
    const QMat& A0 = shared ? p.S0 : p.A0;
    const QMat& A1 = shared ? p.S1 : p.A1;
    const int e = shared ? 0 : t.expert;
    const int nkb = (shared ? p.Ks : p.K) / kBK;
    const int N = (t.nvalid + 15) & ~15;
    const int m0 = mt * kTileM;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStage);
    // full_a[s], full_b[s], empty[s], acc, drain
    const uint32_t bar0 = smem_u32(bars);
    auto full_a = [&](int s) { return bar0 + 8u * s; };
    auto full_b = [&](int s) { return bar0 + 8u * (kStages + s); };
    auto empty = [&](int s) { return bar0 + 8u * (2 * kStages + s); };
    const uint32_t acc_bar = bar0 + 8u * (3 * kStages), drain_bar = acc_bar + 8u;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 3 * kStages + 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kStages + 3);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_a(s), kDeqThreads);
            mbar_init(full_b(s), 1);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_bar, 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto fail = [&](int code) {
        *abort_flag = 1;
        atomicCAS(p.err, 0, code);
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---- token operand producer
            int last_kb[kStages];
            for (int s = 0; s < kStages; ++s) last_kb[s] = -1;
            bool ok = true;
            for (int kb = 0; kb < nkb && ok; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = (kb / kStages) & 1;
                if (!mbar_wait(empty(s), ph ^ 1, abort_flag)) {
                    fail(kErrEmpty);
                    ok = false;
                    break;
                }
                const uint32_t b_dst = smem_u32(smem + s * kStage + (GATEUP ? 2 : 1) * kABytes);
                mbar_expect_tx(full_b(s), (uint32_t)N * kBK * 2);
                for (int r = 0; r < N; r += 16) tma_load_2d(b_dst + (uint32_t)r * 128, &tmap_b, kb * kBK, t.pos0 + r, full_b(s));
                last_kb[s] = kb;
            }
            if (!ok || *abort_flag) {
                // let every copy this thread issued land before the CTA exits
                for (int s = 0; s < kStages; ++s)
                    if (last_kb[s] >= 0) mbar_wait_timed(full_b(s), (last_kb[s] / kStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            const uint32_t idesc = idesc_f16(kTileM, N);
            bool issued = false, ok = true;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kStages;
                const uint32_t ph = (kb / kStages) & 1;
                if (!mbar_wait(full_a(s), ph, abort_flag)) {
                    fail(kErrFullA);
                    ok = false;
                    break;
                }
                if (!mbar_wait(full_b(s), ph, abort_flag)) {
                    fail(kErrFullB);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = smem_u32(smem + s * kStage);
                const uint32_t b = a0 + (GATEUP ? 2 : 1) * kABytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                    umma_f16(tmem, sw128_desc(a0 + kk * 32), sw128_desc(b + kk * 32), idesc, acc);
                    if (GATEUP) umma_f16(tmem + 256, sw128_desc(a0 + kABytes + kk * 32), sw128_desc(b + kk * 32), idesc, acc);
                }
                issued = true;
                umma_commit(empty(s));
            }
            if (ok) {
                umma_commit(acc_bar);
            } else if (issued) {
                umma_commit(drain_bar);  // MMAs in flight must finish before TMEM is freed
                mbar_wait_timed(drain_bar, 0);
            }
        }
    } else {
        // ---- dequant producers (warps 2-9), then epilogue (warps 4-7)
        const int dt = threadIdx.x - 64;
        const int r = dt >> 1, h = dt & 1;
        const int row = m0 + r;
        Raw cur0, cur1, nxt0, nxt1;
        raw_load<DT>(A0, e, row, 0, h, cur0);
        if (GATEUP) raw_load<DT>(A1, e, row, 0, h, cur1);
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            if (kb + 1 < nkb) {
                raw_load<DT>(A0, e, row, kb + 1, h, nxt0);
                if (GATEUP) raw_load<DT>(A1, e, row, kb + 1, h, nxt1);
            }
            const int s = kb % kStages;
            const uint32_t ph = (kb / kStages) & 1;
            if (!mbar_wait(empty(s), ph ^ 1, abort_flag)) {
                fail(kErrEmpty);
                ok = false;
                break;
            }
            uint8_t* a0 = smem + s * kStage;
            raw_store<DT>(cur0, kb, r, h, a0);
            if (GATEUP) raw_store<DT>(cur1, kb, r, h, a0 + kABytes);
            fence_proxy_async();
            mbar_arrive(full_a(s));
            cur0 = nxt0;
            if (GATEUP) cur1 = nxt1;
        }
        // tcgen05.ld is warp-collective: keep the epilogue decision warp-uniform
        ok = __all_sync(0xffffffffu, ok);
        if (ok && warp >= 4 && warp < 8) {
            const int q = warp & 3;
            const bool got = __all_sync(0xffffffffu, mbar_wait(acc_bar, 0, abort_flag));
            if (!got) {
                fail(kErrAcc);
            } else {
                tc_fence_after();
                const uint32_t lane_base = (uint32_t)(q * 32) << 16;
                const int f = m0 + q * 32 + lane;
                for (int c0 = 0; c0 < N; c0 += 16) {
                    uint32_t g[16], u[16];
                    tmem_ld16(tmem + lane_base + c0, g);
                    if (GATEUP) tmem_ld16(tmem + lane_base + 256 + c0, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int col = c0 + j;
                        if (col < t.nvalid) {
                            float v = __uint_as_float(g[j]);
                            if (GATEUP) v = silu_f(v) * __uint_as_float(u[j]);
                            p.out[(int64_t)(t.pos0 + col) * p.out_ld + f] = __float2half_rn(v);
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ------------------------------------------------------------------ helpers
__global__ void gather_kernel(const float* __restrict__ x, const int32_t* __restrict__ perm, int k, int P, int rows,
                              int dp, __half* __restrict__ xp) {
    const int per_row = dp / 8;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * per_row) return;
    const int row = (int)(i / per_row), c = (int)(i % per_row) * 8;
    const int tok = row < P ? perm[row] / k : row - P;
    const float* src = x + (int64_t)tok * dp + c;
    const float4 a = ld_f4(src), b = ld_f4(src + 4);
    *reinterpret_cast<uint4*>(xp + (int64_t)row * dp + c) =
        make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(b.x, b.y), pack_h2(b.z, b.w));
}

__global__ void __launch_bounds__(1024) build_tiles_kernel(const int32_t* __restrict__ act_e,
                                                           const int32_t* __restrict__ act_off,
                                                           const int32_t* __restrict__ n_active, int P, int T,
                                                           int has_shared, GemmTile* __restrict__ tiles,
                                                           int32_t* __restrict__ n_tiles) {
    using Scan = cub::BlockScan<int, 1024>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int na = *n_active;
    for (int base = 0; base < na; base += 1024) {
        const int u = base + threadIdx.x;
        int cnt = 0, n = 0;
        if (u < na) {
            n = act_off[u + 1] - act_off[u];
            cnt = (n + kGemmNT - 1) / kGemmNT;
        }
        int ex, tot;
        Scan(tmp).ExclusiveSum(cnt, ex, tot);
        const int c0 = carry;
        for (int j = 0; j < cnt; ++j)
            tiles[c0 + ex + j] = GemmTile{act_e[u], act_off[u] + j * kGemmNT, min(kGemmNT, n - j * kGemmNT), 0};
        __syncthreads();
        if (threadIdx.x == 0) carry = c0 + tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        int c = carry;
        if (has_shared)
            for (int j = 0; j * kGemmNT < T; ++j) tiles[c++] = GemmTile{-1, P + j * kGemmNT, min(kGemmNT, T - j * kGemmNT), 0};
        *n_tiles = c;
    }
}

__global__ void combine_h_kernel(const __half* __restrict__ y, const int32_t* __restrict__ inv,
                                    const float* __restrict__ w, const float* __restrict__ sgate, int T, int k, int d,
                                    int has_shared, float* __restrict__ out) {
    const int d4 = d >> 2;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * d4) return;
    const int t = (int)(i / d4), c = (int)(i % d4) * 4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int s = 0; s < k; ++s) {
        const float wt = w[(int64_t)t * k + s];
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(y + (int64_t)inv[(int64_t)t * k + s] * d + c));
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        a0 += wt * lo.x;
        a1 += wt * lo.y;
        a2 += wt * hi.x;
        a3 += wt * hi.y;
    }
    if (has_shared) {
        const float g = sgate[t];
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(y + ((int64_t)T * k + t) * d + c));
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        a0 += g * lo.x;
        a1 += g * lo.y;
        a2 += g * hi.x;
        a3 += g * hi.y;
    }
    *reinterpret_cast<float4*>(out + (int64_t)t * d + c) = make_float4(a0, a1, a2, a3);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// 2-D f16 tensor (rows x cols, row stride ld elements), box 16 rows x 64 cols, 128B swizzle.
bool make_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, 16u};
    cuuint32_t es[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int DT, bool GATEUP>
cudaError_t launch_gemm(const CUtensorMap& tmap, const GemmParams& p, int max_tiles, cudaStream_t s) {
    constexpr int kStages = GATEUP ? 3 : 4;
    constexpr size_t smem = (size_t)kStages * ((GATEUP ? 2 : 1) * kABytes + kBBytes) + 1024 + 256;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(grouped_gemm_kernel<DT, GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const int grid = max_tiles * p.MTmax;
    if (grid <= 0) return cudaSuccess;
    grouped_gemm_kernel<DT, GATEUP><<<grid, kThreads, smem, s>>>(tmap, p);
    return cudaGetLastError();
}

}  // namespace

size_t gemm_workspace_bytes(int dp, int act_ld, int P, int T, int max_tiles) {
    auto al = [](size_t v) { return (v + 1023) & ~(size_t)1023; };
    const size_t rows = (size_t)P + T;
    return al(rows * dp * 2) + al(rows * act_ld * 2) + al(rows * dp * 2) + al((size_t)max_tiles * sizeof(GemmTile)) + 1024;
}

bool gemm_setup(void* ws, size_t ws_bytes, int dp, int act_ld, int P_cap, int T_cap, int max_tiles, GemmBuffers* b,
                std::string* why) {
    auto al = [](size_t v) { return (v + 1023) & ~(size_t)1023; };
    const size_t rows = (size_t)P_cap + T_cap;
    if (ws_bytes < gemm_workspace_bytes(dp, act_ld, P_cap, T_cap, max_tiles)) {
        *why = "prefill workspace too small";
        return false;
    }
    char* c = static_cast<char*>(ws);
    b->xperm = reinterpret_cast<__half*>(c);
    c += al(rows * dp * 2);
    b->act = reinterpret_cast<__half*>(c);
    c += al(rows * act_ld * 2);
    b->y = reinterpret_cast<__half*>(c);
    c += al(rows * dp * 2);
    b->tiles = reinterpret_cast<GemmTile*>(c);
    c += al((size_t)max_tiles * sizeof(GemmTile));
    b->n_tiles = reinterpret_cast<int32_t*>(c);
    b->err = b->n_tiles + 1;
    b->rows_cap = (int)rows;
    if (!make_tmap(&b->tmap_x, b->xperm, rows, (uint64_t)dp, (uint64_t)dp) ||
        !make_tmap(&b->tmap_act, b->act, rows, (uint64_t)act_ld, (uint64_t)act_ld)) {
        *why = "cuTensorMapEncodeTiled failed (driver entry point unavailable or bad layout)";
        return false;
    }
    return true;
}

cudaError_t launch_prefill(const PrefillArgs& a, GemmBuffers& b, cudaStream_t s, int* launches) {
    const int P = a.T * a.k;
    const int rows = P + (a.has_shared ? a.T : 0);
    const int max_tiles = gemm_max_tiles(P, a.T, a.E, a.has_shared);
    {
        const int64_t n = (int64_t)rows * (a.dp / 8);
        gather_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(a.x, a.perm, a.k, P, rows, a.dp, b.xperm);
    }
    build_tiles_kernel<<<1, 1024, 0, s>>>(a.act_e, a.act_off, a.n_active, P, a.T, a.has_shared, b.tiles, b.n_tiles);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    GemmParams g{};
    g.tiles = b.tiles;
    g.n_tiles = b.n_tiles;
    g.err = b.err;
    // gate/up
    g.A0 = a.gate;
    g.A1 = a.up;
    g.S0 = a.sg;
    g.S1 = a.su;
    g.K = a.dp;
    g.Ks = a.dp;
    g.MT = a.F / kTileM;
    g.MTs = a.has_shared ? a.Fs / kTileM : 0;
    g.MTmax = g.MT > g.MTs ? g.MT : g.MTs;
    g.out = b.act;
    g.out_ld = a.act_ld;
    e = a.gate.dtype == AERO_DT_Q4_K ? launch_gemm<AERO_DT_Q4_K, true>(b.tmap_x, g, max_tiles, s)
                                     : launch_gemm<AERO_DT_Q8_0, true>(b.tmap_x, g, max_tiles, s);
    if (e != cudaSuccess) return e;
    // down
    g.A0 = a.down;
    g.A1 = a.down;
    g.S0 = a.sd;
    g.S1 = a.sd;
    g.K = a.F;
    g.Ks = a.Fs;
    g.MT = a.dp / kTileM;
    g.MTs = a.has_shared ? a.dp / kTileM : 0;
    g.MTmax = g.MT;
    g.out = b.y;
    g.out_ld = a.dp;
    e = a.down.dtype == AERO_DT_Q4_K ? launch_gemm<AERO_DT_Q4_K, false>(b.tmap_act, g, max_tiles, s)
                                     : launch_gemm<AERO_DT_Q8_0, false>(b.tmap_act, g, max_tiles, s);
    if (launches) *launches += 4;
    return e;
}

cudaError_t launch_combine_h(const __half* y, const int32_t* inv, const float* w, const float* sgate, int T,
                                int k, int d, int has_shared, float* out, cudaStream_t s) {
    const int64_t n = (int64_t)T * (d / 4);
    if (n == 0) return cudaSuccess;
    combine_h_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, inv, w, sgate, T, k, d, has_shared, out);
    return cudaGetLastError();
}

}  // namespace aero
