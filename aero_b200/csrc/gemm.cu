// Prefill: grouped expert GEMMs on the 5th-generation tensor cores.
//
// Per routed expert segment (token rows sorted by expert) and for the shared
// expert (all tokens), two grouped GEMMs in "weights x tokens" orientation: the
// 128-row MMA M extent runs over weight rows and the ragged token count is the
// N extent (16..192 in steps of 16), so nothing is padded to 128 tokens.
//   gate/up:  D_g = Wg[m0:m0+128, :] . X^T,  D_u = Wu[...] . X^T   (K = d)
//             epilogue: act = silu(D_g) * D_u  -> f16 act rows
//   down:     D = Wd[n0:n0+128, :] . act^T                        (K = F)
//             epilogue: f16 y rows
// Operands are f16 (kind::f16, fp32 accumulate). bf16 operands were measured
// (and reproduced by a numpy model of the same roundings) at 2.6% of the output
// RMS in max-abs error on Q4_K layers, above the 1% bar; f16 rounds 8x finer at
// the same tensor-core rate.
//
// Persistent kernel: one CTA per SM walks work items (tile, 128-row block)
// blockIdx.x, blockIdx.x + gridDim.x, ... Warp roles (23 warps):
//   warp 0      TMA producer of the raw quant blocks of the item's 128 weight
//               rows (2-D tensor maps over the expert-major qs and header
//               planes, 128 values per stage, a deep ring)
//   warp 22     TMA producer of the token operand (f16 rows, 128B swizzle,
//               K-major, one box of the tile's height per K step; no multicast
//               anywhere)
//   warp 1      one thread issues tcgen05.mma with the weight operand A in TMEM
//               and the token operand B in shared memory, fp32 accumulators in
//               TMEM, tcgen05.commit to the ring barriers
//   warps 2-17  dequantise from shared memory with packed half2 arithmetic
//               (Q4_K: s*q - m per 32-value sub-block; Q8_0: d*q) and write A
//               into TMEM with tcgen05.st (row m of A = TMEM lane m, two f16 per
//               column); the block headers ride in the same TMA stages
//   warps 18-21 epilogue: tcgen05.ld of the accumulators 16 columns at a time,
//               SwiGLU, f16 results staged in shared memory for 16-byte stores
// The weight tile never passes through shared memory, which halves the shared
// memory traffic per K step. The down GEMM double-buffers its accumulators so
// its epilogue overlaps the next item's main loop.
// Every wait is bounded by %globaltimer (2 s): on expiry the CTA records an
// error code (read by the host at its next synchronisation), drains its own
// copies and MMAs, frees TMEM and exits.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cub/block/block_scan.cuh>
#include <string>

#include "gemm.h"
#include "internal.h"
#include "tc_common.cuh"

namespace aero {
namespace {

constexpr int kBK = 64;          // K per MMA stage (A and B)
constexpr int kRawK = 128;       // K per raw (quant) stage
constexpr int kTileM = 128;
constexpr int kThreads = 736;    // 23 warps
constexpr int kDeqWarps = 16;
constexpr int kEpiWarp0 = 2 + kDeqWarps;   // warps 18-21
constexpr int kTokWarp = kEpiWarp0 + 4;    // warp 22
constexpr int kBMaps = kGemmNT / 16;  // token-operand maps, box heights 16, 32, ..., 192
constexpr int kBStages = 4;
constexpr uint32_t kBStageBytes = kGemmNT * kBK * 2;  // 24 KiB: up to 192 token rows x 128 B
constexpr uint32_t kRawRing = 96 * 1024;
// TMEM columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccStride = kGemmNT;     // 192 columns per accumulator
constexpr uint32_t kAColBase = 2 * kGemmNT;  // 384: two A stages of 64 columns (gate/up) or 32 (down)

enum : int { kErrRawFull = 1, kErrBFull = 2, kErrEmpty = 3, kErrAcc = 4, kErrAFull = 5, kErrAEmpty = 6 };

struct GemmParams {
    QMat A0, A1;          // routed: gate, up (gate/up GEMM) or down
    QMat S0, S1;          // shared expert
    const GemmTile* tiles;
    const int32_t* n_tiles;
    int K, Ks;            // reduction length for routed / shared items
    int MT, MTs, MTmax;   // 128-row blocks for routed / shared
    int e_begin;          // first expert held by the planes (expert parallelism)
    __half* out;
    int out_ld;
    int32_t* err;
};

struct Item {
    GemmTile t;
    int mt, nkb, N;
    bool shared;
};

// The next work item of this CTA at or after w (skipping blocks a shared tile lacks).
__device__ __forceinline__ bool item_at(const GemmParams& p, int n_tiles, int& w, Item& it) {
    const int total = n_tiles * p.MTmax;
    while (w < total) {
        const int ti = w / p.MTmax, mt = w % p.MTmax;
        const GemmTile t = p.tiles[ti];
        const bool sh = t.expert < 0;
        if (mt < (sh ? p.MTs : p.MT)) {
            it.t = t;
            it.mt = mt;
            it.shared = sh;
            it.nkb = (sh ? p.Ks : p.K) / kBK;
            it.N = (t.nvalid + 15) & ~15;
            return true;
        }
        w += gridDim.x;
    }
    return false;
}

// Kernel tensor maps: the token operand with box heights 16, 32, ..., 192 rows
// (one copy per K step covers a whole tile), then per weight family the qs
// plane and the header plane, routed (w) and shared (s), matrix 0 and 1.
struct GemmMaps {
    CUtensorMap b[kBMaps];
    CUtensorMap w0, w1, s0, s1, mw0, mw1, ms0, ms1;
};

template <int DT, bool GATEUP>
struct Cfg {
    static constexpr int kRawRowBytes = DT == AERO_DT_Q4_K ? kRawK / 2 : kRawK;  // 64 or 128
    static constexpr int kMats = GATEUP ? 2 : 1;
    static constexpr uint32_t kQsBytes = (uint32_t)kMats * kTileM * kRawRowBytes;
    static constexpr uint32_t kMetaBytes = (uint32_t)kMats * kTileM * 16;  // a 16-byte header slice per row
    static constexpr uint32_t kRawStageBytes = kQsBytes + kMetaBytes;
    static constexpr int kRawStages = (int)(kRawRing / kRawStageBytes);
    static constexpr int kAcc = GATEUP ? 1 : 2;  // accumulator buffers
    static constexpr size_t kSmem = kRawRing + (size_t)kBStages * kBStageBytes + 1024 + 512 + 4 * 1024;
};

template <int DT, bool GATEUP>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_kernel(const __grid_constant__ GemmMaps tm, GemmParams p) {
    using C = Cfg<DT, GATEUP>;
    constexpr int kRS = C::kRawStages;
    const int n_tiles = *p.n_tiles;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* raw_ring = smem;           // kRS x kRawStageBytes
    uint8_t* b_ring = smem + kRawRing;  // kBStages x kBStageBytes (1024-aligned)
    uint64_t* bars = reinterpret_cast<uint64_t*>(b_ring + kBStages * kBStageBytes);
    const uint32_t bar0 = smem_u32(bars);
    // barrier table: raw_full[kRS], raw_empty[kRS], b_full[4], b_empty[4], a_full[2], a_empty[2],
    // acc_full[2], acc_empty[2], drain
    auto raw_full = [&](int s) { return bar0 + 8u * s; };
    auto raw_empty = [&](int s) { return bar0 + 8u * (kRS + s); };
    auto b_full = [&](int s) { return bar0 + 8u * (2 * kRS + s); };
    auto b_empty = [&](int s) { return bar0 + 8u * (2 * kRS + kBStages + s); };
    auto a_full = [&](int s) { return bar0 + 8u * (2 * kRS + 2 * kBStages + s); };
    auto a_empty = [&](int s) { return bar0 + 8u * (2 * kRS + 2 * kBStages + 2 + s); };
    auto acc_full = [&](int s) { return bar0 + 8u * (2 * kRS + 2 * kBStages + 4 + s); };
    auto acc_empty = [&](int s) { return bar0 + 8u * (2 * kRS + 2 * kBStages + 6 + s); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kRS + 2 * kBStages + 8);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kRS + 2 * kBStages + 9);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kRS + 2 * kBStages + 10);
    uint8_t* epi_smem = b_ring + kBStages * kBStageBytes + 512;  // 4 warps x 1 KiB output staging

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRS; ++s) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), kDeqWarps);
        }
        for (int s = 0; s < kBStages; ++s) {
            mbar_init(b_full(s), 1);
            mbar_init(b_empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(a_full(s), kDeqWarps);
            mbar_init(a_empty(s), 1);
            mbar_init(acc_full(s), 1);
            mbar_init(acc_empty(s), 4);
        }
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
            // ---------------------------------------------------------- producer
            int raw_n = 0, b_n = 0;  // running stage counters
            bool ok = true;
            Item it;
            for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x) {
                const CUtensorMap* w0 = it.shared ? &tm.s0 : &tm.w0;
                const CUtensorMap* w1 = it.shared ? &tm.s1 : &tm.w1;
                const CUtensorMap* m0 = it.shared ? &tm.ms0 : &tm.mw0;
                const CUtensorMap* m1 = it.shared ? &tm.ms1 : &tm.mw1;
                const QMat& A = it.shared ? p.S0 : p.A0;
                const int y0 = (it.shared ? 0 : (it.t.expert - p.e_begin)) * A.rows + it.mt * kTileM;
                for (int kb = 0; kb < it.nkb && ok; kb += 2) {
                    {
                        const int s = raw_n % kRS;
                        if (!mbar_wait(raw_empty(s), ((raw_n / kRS) & 1) ^ 1, abort_flag)) {
                            fail(kErrEmpty);
                            ok = false;
                            break;
                        }
                        const uint32_t dst = smem_u32(raw_ring + s * C::kRawStageBytes);
                        mbar_expect_tx(raw_full(s), C::kRawStageBytes);
                        // qs of values [64 kb, 64 kb + 128), and the 16-byte header slice
                        // covering the 256 values around them
                        const int x = (kb / 2) * C::kRawRowBytes;
                        const int xm = (kb / 4) * 16;
                        tma_load_2d(dst, w0, x, y0, raw_full(s));
                        tma_load_2d(dst + C::kQsBytes, m0, xm, y0, raw_full(s));
                        if (GATEUP) {
                            tma_load_2d(dst + kTileM * C::kRawRowBytes, w1, x, y0, raw_full(s));
                            tma_load_2d(dst + C::kQsBytes + kTileM * 16, m1, xm, y0, raw_full(s));
                        }
                        ++raw_n;
                    }
                }
            }
            if (!ok) {
                // let every copy this thread issued land before the CTA exits
                for (int i = 0; i < kRS && i < raw_n; ++i) {
                    const int n = raw_n - 1 - i;
                    mbar_wait_timed(raw_full(n % kRS), (n / kRS) & 1);
                }
            }
        }
    } else if (warp == kTokWarp) {
        if (lane == 0) {
            // ---------------------------------------------------- token producer
            int b_n = 0;
            bool ok = true;
            Item it;
            for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x) {
                const CUtensorMap* bm = &tm.b[it.N / 16 - 1];
                for (int kb = 0; kb < it.nkb; ++kb) {
                    const int sb = b_n % kBStages;
                    if (!mbar_wait(b_empty(sb), ((b_n / kBStages) & 1) ^ 1, abort_flag)) {
                        fail(kErrEmpty);
                        ok = false;
                        break;
                    }
                    const uint32_t dst = smem_u32(b_ring + sb * kBStageBytes);
                    mbar_expect_tx(b_full(sb), (uint32_t)it.N * kBK * 2);
                    tma_load_2d(dst, bm, kb * kBK, it.t.pos0, b_full(sb));
                    ++b_n;
                }
            }
            if (!ok) {
                for (int i = 0; i < kBStages && i < b_n; ++i) {
                    const int n = b_n - 1 - i;
                    mbar_wait_timed(b_full(n % kBStages), (n / kBStages) & 1);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------- MMA issuer
            int a_n = 0, b_n = 0, item_n = 0;
            bool ok = true, issued = false;
            Item it;
            for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x, ++item_n) {
                const int ab = item_n % C::kAcc;
                if (!mbar_wait(acc_empty(ab), ((item_n / C::kAcc) & 1) ^ 1, abort_flag)) {
                    fail(kErrAcc);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t idesc = idesc_f16(kTileM, it.N);
                const uint32_t d0 = tmem + (GATEUP ? 0u : (uint32_t)ab * kAccStride);
                for (int kb = 0; kb < it.nkb; ++kb) {
                    const int sa = a_n & 1, sb = b_n % kBStages;
                    if (!mbar_wait(a_full(sa), (a_n >> 1) & 1, abort_flag)) {
                        fail(kErrAFull);
                        ok = false;
                        break;
                    }
                    if (!mbar_wait(b_full(sb), (b_n / kBStages) & 1, abort_flag)) {
                        fail(kErrBFull);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t b = smem_u32(b_ring + sb * kBStageBytes);
                    const uint32_t a0 = tmem + kAColBase + (uint32_t)sa * (GATEUP ? 64u : 32u);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        umma_ts(d0, a0 + kk * 8, sw128_desc(b + kk * 32), idesc, acc);
                        if (GATEUP) umma_ts(d0 + kAccStride, a0 + 32 + kk * 8, sw128_desc(b + kk * 32), idesc, acc);
                    }
                    issued = true;
                    umma_commit(a_empty(sa));
                    umma_commit(b_empty(sb));
                    ++a_n;
                    ++b_n;
                }
                if (ok) umma_commit(acc_full(ab));
            }
            if (!ok && issued) {
                umma_commit(drain_bar);  // MMAs in flight must finish before TMEM is freed
                mbar_wait_timed(drain_bar, 0);
            }
        }
    } else if (warp < kEpiWarp0) {
        // -------------------------------------------------------------- dequant
        // 16 warps: warp (warp & 3) may write TMEM lane quarter q; its combo
        // c = (warp - 2) / 4 picks its share of each 64-value K-block:
        //   gate/up: matrix c / 2, values [32 (c % 2), +32)   (16 TMEM columns)
        //   down:    values [16 c, 16 c + 16)                 (8 TMEM columns)
        const int cmb = (warp - 2) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;  // weight row within the 128-row block
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        const int mat = GATEUP ? (cmb >> 1) : 0;
        const int half = GATEUP ? (cmb & 1) : 0;
        int raw_n = 0, a_n = 0;
        bool ok = true;
        Item it;
        for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x) {
            for (int kb = 0; kb < it.nkb; ++kb) {
                const int s = raw_n % kRS;
                if ((kb & 1) == 0) {
                    const bool got = __all_sync(0xffffffffu, mbar_wait(raw_full(s), (raw_n / kRS) & 1, abort_flag));
                    if (!got) {
                        if (lane == 0) fail(kErrRawFull);
                        ok = false;
                        break;
                    }
                }
                const int sa = a_n & 1;
                const bool got = __all_sync(0xffffffffu, mbar_wait(a_empty(sa), ((a_n >> 1) & 1) ^ 1, abort_flag));
                if (!got) {
                    if (lane == 0) fail(kErrAEmpty);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint8_t* stage = raw_ring + s * C::kRawStageBytes;
                // this row's qs for the stage (TMA-swizzled: 64B for Q4_K rows of 64 bytes,
                // 128B for Q8_0 rows of 128 bytes: logical 16-byte chunk c sits at c ^ f(r))
                const uint8_t* qrow = stage + mat * kTileM * C::kRawRowBytes + r * C::kRawRowBytes;
                const int swz = DT == AERO_DT_Q4_K ? ((r >> 1) & 3) : (r & 7);
                auto qchunk = [&](int c) { return *reinterpret_cast<const uint4*>(qrow + ((c ^ swz) << 4)); };
                const uint4 meta = *reinterpret_cast<const uint4*>(stage + C::kQsBytes + mat * kTileM * 16 + r * 16);
                const uint32_t abase = tmem + lane_base + kAColBase + (uint32_t)sa * (GATEUP ? 64u : 32u);
                if (DT == AERO_DT_Q4_K) {
                    // values: low nibbles of the K-block's 32 bytes are values 0-31 (sub-block 2g),
                    // high nibbles 32-63 (sub-block 2g+1); column j holds values 2j, 2j+1
                    const bool hi = GATEUP ? half : (cmb >> 1);
                    const uint8_t* mb = reinterpret_cast<const uint8_t*>(&meta);
                    const float d = __half2float(__ushort_as_half((unsigned short)(mb[0] | (mb[1] << 8))));
                    const float dmin = __half2float(__ushort_as_half((unsigned short)(mb[2] | (mb[3] << 8))));
                    int sc, mn;
                    q4k_sc_m(mb + 4, 2 * (kb & 3) + (hi ? 1 : 0), sc, mn);
                    const __half2 sh = __float2half2_rn(d * (float)sc), nh = __float2half2_rn(-(dmin * (float)mn));
                    const int shift = hi ? 4 : 0;
                    if (GATEUP) {
                        const uint4 v0 = qchunk(2 * (kb & 1)), v1 = qchunk(2 * (kb & 1) + 1);
                        const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                        uint32_t cols[16];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t a2 = __byte_perm(wv[i], 0, 0x4140) >> shift;
                            const uint32_t b2 = __byte_perm(wv[i], 0, 0x4342) >> shift;
                            cols[2 * i] = h2u(__hfma2(nib2_to_h2(a2), sh, nh));
                            cols[2 * i + 1] = h2u(__hfma2(nib2_to_h2(b2), sh, nh));
                        }
                        tmem_st16(abase + (uint32_t)mat * 32u + (uint32_t)half * 16u, cols);
                    } else {
                        // combo c: bytes [16 (c & 1), +16), low (c < 2) or high nibbles -> columns 8c .. 8c+7
                        const uint4 v = qchunk(2 * (kb & 1) + (cmb & 1));
                        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
                        uint32_t cols[8];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            cols[2 * i] = h2u(__hfma2(nib2_to_h2(__byte_perm(wv[i], 0, 0x4140) >> shift), sh, nh));
                            cols[2 * i + 1] = h2u(__hfma2(nib2_to_h2(__byte_perm(wv[i], 0, 0x4342) >> shift), sh, nh));
                        }
                        tmem_st8(abase + (uint32_t)cmb * 8u, cols);
                    }
                } else {
                    // the 16-byte slice holds 8 fp16 scales for 256 values; this K-block uses two
                    // (values 0-31 and 32-63); column j holds values 2j, 2j+1
                    const uint32_t mw[4] = {meta.x, meta.y, meta.z, meta.w};
                    const uint32_t sc8 = mw[kb & 3];
                    const int blk = GATEUP ? half : (cmb >> 1);
                    const __half2 dd = __half2half2(__ushort_as_half((unsigned short)(blk ? (sc8 >> 16) : (sc8 & 0xFFFFu))));
                    if (GATEUP) {
                        const uint4 v0 = qchunk(4 * (kb & 1) + 2 * blk), v1 = qchunk(4 * (kb & 1) + 2 * blk + 1);
                        const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
                        uint32_t cols[16];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const uint32_t wb = wv[i] ^ 0x80808080u;
                            cols[2 * i] = h2u(__hmul2(byte2_to_h2(__byte_perm(wb, 0, 0x4140)), dd));
                            cols[2 * i + 1] = h2u(__hmul2(byte2_to_h2(__byte_perm(wb, 0, 0x4342)), dd));
                        }
                        tmem_st16(abase + (uint32_t)mat * 32u + (uint32_t)half * 16u, cols);
                    } else {
                        const uint4 v = qchunk(4 * (kb & 1) + cmb);
                        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
                        uint32_t cols[8];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t wb = wv[i] ^ 0x80808080u;
                            cols[2 * i] = h2u(__hmul2(byte2_to_h2(__byte_perm(wb, 0, 0x4140)), dd));
                            cols[2 * i + 1] = h2u(__hmul2(byte2_to_h2(__byte_perm(wb, 0, 0x4342)), dd));
                        }
                        tmem_st8(abase + (uint32_t)cmb * 8u, cols);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(a_full(sa));
                ++a_n;
                if ((kb & 1) || kb + 1 == it.nkb) {
                    if (lane == 0) mbar_arrive(raw_empty(s));
                    ++raw_n;
                }
            }
        }
    } else if (warp < kTokWarp) {
        // -------------------------------------------------------------- epilogue
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        __half* stage = reinterpret_cast<__half*>(epi_smem + (warp - kEpiWarp0) * 1024);
        int item_n = 0;
        Item it;
        for (int w = blockIdx.x; item_at(p, n_tiles, w, it); w += gridDim.x, ++item_n) {
            const int ab = item_n % C::kAcc;
            const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full(ab), (item_n / C::kAcc) & 1, abort_flag));
            if (!got) {
                if (lane == 0) fail(kErrAcc);
                break;
            }
            tc_fence_after();
            const uint32_t d0 = tmem + lane_base + (GATEUP ? 0u : (uint32_t)ab * kAccStride);
            // 16 columns (tokens) at a time: one TMEM round trip, then the f16 results
            // go through this warp's 16 x 32 staging tile so each lane stores 16 bytes
            __half* const out_row0 = p.out + (int64_t)it.t.pos0 * p.out_ld + it.mt * kTileM + q * 32 + (lane & 3) * 8;
            for (int c0 = 0; c0 < it.N; c0 += 16) {
                uint32_t g[16];
                tmem_ld16(d0 + c0, g);
                if (GATEUP) {
                    uint32_t u[16];
                    tmem_ld16(d0 + kAccStride + c0, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float v = __uint_as_float(g[j]);
                        // silu(v) * u; fast exp / divide suffice for an f16 result
                        stage[j * 32 + lane] = __float2half_rn(__fdividef(v, 1.0f + __expf(-v)) * __uint_as_float(u[j]));
                    }
                } else {
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) stage[j * 32 + lane] = __float2half_rn(__uint_as_float(g[j]));
                }
                __syncwarp();
#pragma unroll
                for (int r8 = 0; r8 < 2; ++r8) {
                    const int j = r8 * 8 + (lane >> 2);
                    const uint4 v = *reinterpret_cast<const uint4*>(stage + j * 32 + (lane & 3) * 8);
                    if (c0 + j < it.t.nvalid) *reinterpret_cast<uint4*>(out_row0 + (int64_t)(c0 + j) * p.out_ld) = v;
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty(ab));
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
// xperm rows: [0, P_real) the routed pairs in sorted order, [P, P + Tsh) the
// first Tsh input rows for the shared expert. P_real (= offsets[E]) is read on
// the device: sorted positions [P_real, P) hold skipped slots and are not
// gathered. Grid-stride over 8-value chunks.
template <typename XT>
__global__ void gather_kernel(const XT* __restrict__ x, const int32_t* __restrict__ perm,
                              const int32_t* __restrict__ p_real, int k, int P, int Tsh, int dp,
                              __half* __restrict__ xp) {
    const int per_row = dp / 8;
    const int pr = *p_real;
    const int64_t n = (int64_t)(pr + Tsh) * per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int v = (int)(i / per_row), c = (int)(i % per_row) * 8;
        const int row = v < pr ? v : P + (v - pr);
        const int tok = v < pr ? perm[v] / k : v - pr;
        uint4 o;
        if constexpr (sizeof(XT) == 2) {
            o = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)tok * dp + c));
        } else {
            const float* src = reinterpret_cast<const float*>(x) + (int64_t)tok * dp + c;
            const float4 a = ld_f4(src), b = ld_f4(src + 4);
            o = make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(b.x, b.y), pack_h2(b.z, b.w));
        }
        *reinterpret_cast<uint4*>(xp + (int64_t)row * dp + c) = o;
    }
}

__global__ void __launch_bounds__(1024) build_tiles_kernel(const int32_t* __restrict__ act_e,
                                                           const int32_t* __restrict__ act_off,
                                                           const int32_t* __restrict__ n_active, int P, int Tsh,
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
            for (int j = 0; j * kGemmNT < Tsh; ++j)
                tiles[c++] = GemmTile{-1, P + j * kGemmNT, min(kGemmNT, Tsh - j * kGemmNT), 0};
        *n_tiles = c;
    }
}

// out[t] = sum over slots s of w[t][s] * y[inv[t*k+s]] (+ sgate[t] * y[P + t]
// for t < Tsh). With idx given, slots whose bucket is >= E_real were skipped.
__global__ void combine_h_kernel(const __half* __restrict__ y, const int32_t* __restrict__ inv,
                                 const float* __restrict__ w, const float* __restrict__ sgate,
                                 const int32_t* __restrict__ idx, int E_real, int T, int Tsh, int k, int d,
                                 int has_shared, float* __restrict__ out) {
    const int d4 = d >> 2;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * d4) return;
    const int t = (int)(i / d4), c = (int)(i % d4) * 4;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    for (int s = 0; s < k; ++s) {
        if (idx && idx[(int64_t)t * k + s] >= E_real) continue;
        const float wt = w[(int64_t)t * k + s];
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(y + (int64_t)inv[(int64_t)t * k + s] * d + c));
        const float2 lo = __half22float2(u2h(v.x));
        const float2 hi = __half22float2(u2h(v.y));
        a0 += wt * lo.x;
        a1 += wt * lo.y;
        a2 += wt * hi.x;
        a3 += wt * hi.y;
    }
    if (has_shared && t < Tsh) {
        const float g = sgate[t];
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(y + ((int64_t)T * k + t) * d + c));
        const float2 lo = __half22float2(u2h(v.x));
        const float2 hi = __half22float2(u2h(v.y));
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

}  // namespace

bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t rows,
                    uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn || !base) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t es[2] = {1u, 1u};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

// 2-D f16 activations (rows x cols, row stride ld elements): box box_rows x 64 cols, 128B swizzle.
bool make_tmap_act(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
    cuuint32_t es[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A weight plane as 2-D bytes [n_expert * rows][row bytes] (experts must be
// contiguous): box = 128 rows x box_bytes.
bool make_tmap_plane(CUtensorMap* m, const uint8_t* base, uint64_t row_bytes, int rows, int64_t estride,
                     int n_local_experts, int box_bytes, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn || !base) return false;
    if ((uint64_t)estride != row_bytes * (uint64_t)rows || row_bytes % 16) return false;
    cuuint64_t dims[2] = {row_bytes, (cuuint64_t)rows * (cuuint64_t)n_local_experts};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)kTileM};
    cuuint32_t es[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// qs plane: the raw bytes of 128 values per box row (Q4_K 64 B, 64B swizzle;
// Q8_0 128 B, 128B swizzle). Header plane: 16-byte slices, no swizzle.
bool make_tmap_qs(CUtensorMap* m, const QMat& q, int n_local) {
    const bool q4 = q.dtype == AERO_DT_Q4_K;
    return make_tmap_plane(m, q.qs, (uint64_t)qm_row_qs_bytes(q.dtype, q.cols), q.rows, q.qs_estride, n_local,
                           q4 ? kRawK / 2 : kRawK, q4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
}
bool make_tmap_meta(CUtensorMap* m, const QMat& q, int n_local) {
    return make_tmap_plane(m, q.meta, (uint64_t)qm_row_meta_bytes(q.dtype, q.cols), q.rows, q.meta_estride, n_local, 16,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
}

template <int DT, bool GATEUP>
cudaError_t launch_gemm(const GemmMaps& maps, const GemmParams& p, int n_sm, cudaStream_t s) {
    using C = Cfg<DT, GATEUP>;
    static_assert(C::kRawStages >= 2, "raw ring too small");
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(grouped_gemm_kernel<DT, GATEUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)C::kSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    grouped_gemm_kernel<DT, GATEUP><<<n_sm, kThreads, C::kSmem, s>>>(maps, p);
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
    for (int i = 0; i < kBMaps; ++i)
        if (!make_tmap_act(&b->tmap_x[i], b->xperm, rows, (uint64_t)dp, (uint64_t)dp, 16u * (i + 1)) ||
            !make_tmap_act(&b->tmap_act[i], b->act, rows, (uint64_t)act_ld, (uint64_t)act_ld, 16u * (i + 1))) {
            *why = "cuTensorMapEncodeTiled failed for the activation buffers";
            return false;
        }
    return true;
}

bool gemm_weight_maps(const QMat& gate, const QMat& up, const QMat& down, const QMat& sg, const QMat& su, const QMat& sd,
                      int n_local, int has_shared, GemmWeightMaps* m, std::string* why) {
    // the planes' base pointers here are the allocations (expert e_begin first)
    bool ok = make_tmap_qs(&m->q[0], gate, n_local) && make_tmap_qs(&m->q[1], up, n_local) &&
              make_tmap_qs(&m->q[2], down, n_local) && make_tmap_meta(&m->m[0], gate, n_local) &&
              make_tmap_meta(&m->m[1], up, n_local) && make_tmap_meta(&m->m[2], down, n_local);
    if (ok && has_shared)
        ok = make_tmap_qs(&m->q[3], sg, 1) && make_tmap_qs(&m->q[4], su, 1) && make_tmap_qs(&m->q[5], sd, 1) &&
             make_tmap_meta(&m->m[3], sg, 1) && make_tmap_meta(&m->m[4], su, 1) && make_tmap_meta(&m->m[5], sd, 1);
    if (ok && !has_shared)
        for (int i = 0; i < 3; ++i) {
            m->q[3 + i] = m->q[i];
            m->m[3 + i] = m->m[i];
        }
    if (!ok) *why = "cuTensorMapEncodeTiled failed for an expert weight plane";
    return ok;
}

cudaError_t launch_prefill_prep(const PrefillArgs& a, GemmBuffers& b, cudaStream_t s) {
    const int P = a.T * a.k;
    const int Tsh = a.has_shared ? a.Tsh : 0;
    {
        const int64_t n = (int64_t)(P + Tsh) * (a.dp / 8);
        const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)a.n_sm * 16));
        if (a.x_f16)
            gather_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(a.x), a.perm, a.p_real, a.k, P, Tsh,
                                                        a.dp, b.xperm);
        else
            gather_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(a.x), a.perm, a.p_real, a.k, P, Tsh,
                                                       a.dp, b.xperm);
    }
    build_tiles_kernel<<<1, 1024, 0, s>>>(a.act_e, a.act_off, a.n_active, P, Tsh, a.has_shared, b.tiles, b.n_tiles);
    return cudaGetLastError();
}

cudaError_t launch_prefill_gemm(const PrefillArgs& a, GemmBuffers& b, const GemmWeightMaps& wm, bool gateup,
                                cudaStream_t s) {
    GemmParams g{};
    g.tiles = b.tiles;
    g.n_tiles = b.n_tiles;
    g.err = b.err;
    g.e_begin = a.e_begin;
    GemmMaps maps;
    if (gateup) {
        g.A0 = a.gate;
        g.A1 = a.up;
        g.S0 = a.has_shared ? a.sg : a.gate;
        g.S1 = a.has_shared ? a.su : a.up;
        g.K = a.dp;
        g.Ks = a.dp;
        g.MT = a.F / kTileM;
        g.MTs = a.has_shared ? a.Fs / kTileM : 0;
        g.MTmax = g.MT > g.MTs ? g.MT : g.MTs;
        g.out = b.act;
        g.out_ld = a.act_ld;
        for (int i = 0; i < kBMaps; ++i) maps.b[i] = b.tmap_x[i];
        maps.w0 = wm.q[0];
        maps.w1 = wm.q[1];
        maps.s0 = wm.q[3];
        maps.s1 = wm.q[4];
        maps.mw0 = wm.m[0];
        maps.mw1 = wm.m[1];
        maps.ms0 = wm.m[3];
        maps.ms1 = wm.m[4];
        return a.gate.dtype == AERO_DT_Q4_K ? launch_gemm<AERO_DT_Q4_K, true>(maps, g, a.n_sm, s)
                                            : launch_gemm<AERO_DT_Q8_0, true>(maps, g, a.n_sm, s);
    }
    g.A0 = a.down;
    g.A1 = a.down;
    g.S0 = a.has_shared ? a.sd : a.down;
    g.S1 = g.S0;
    g.K = a.F;
    g.Ks = a.has_shared ? a.Fs : a.F;
    g.MT = a.dp / kTileM;
    g.MTs = a.has_shared ? a.dp / kTileM : 0;
    g.MTmax = g.MT;
    g.out = b.y;
    g.out_ld = a.dp;
    for (int i = 0; i < kBMaps; ++i) maps.b[i] = b.tmap_act[i];
    maps.w0 = maps.w1 = wm.q[2];
    maps.s0 = maps.s1 = wm.q[5];
    maps.mw0 = maps.mw1 = wm.m[2];
    maps.ms0 = maps.ms1 = wm.m[5];
    return a.down.dtype == AERO_DT_Q4_K ? launch_gemm<AERO_DT_Q4_K, false>(maps, g, a.n_sm, s)
                                        : launch_gemm<AERO_DT_Q8_0, false>(maps, g, a.n_sm, s);
}

cudaError_t launch_combine_h(const __half* y, const int32_t* inv, const float* w, const float* sgate,
                             const int32_t* idx, int E_real, int T, int Tsh, int k, int d, int has_shared, float* out,
                             cudaStream_t s) {
    const int64_t n = (int64_t)T * (d / 4);
    if (n == 0) return cudaSuccess;
    combine_h_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, inv, w, sgate, idx, E_real, T, Tsh, k, d,
                                                                 has_shared, out);
    return cudaGetLastError();
}

}  // namespace aero
