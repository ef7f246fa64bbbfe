// Prefill: grouped expert GEMMs on the 5th-generation tensor cores.
//
// Per routed expert segment (token rows sorted by expert) and for the shared
// expert (all tokens), two grouped GEMMs in "weights x tokens" orientation: the
// 128-row MMA M extent runs over weight rows and the ragged token count is the
// N extent (16..192 in steps of 16), so nothing is padded to 128 tokens.
//   gate/up:  an item is 64 rows of gate and the same 64 rows of up, interleaved
//             by half-warps (M rows 32q + i = gate row 16q + i, 32q + 16 + i = up row
//             16q + i, i < 16): D = [Wg; Wu] . X^T (K = d)
//             epilogue: act = silu(D_g) * D_u, the partner rows meeting by a lane
//             shuffle -> f16 act rows
//   down:     D = Wd[n0:n0+128, :] . act^T                        (K = F)
//             epilogue: f16 y rows
// Operands are f16 (kind::f16, fp32 accumulate). bf16 operands were measured
// (and reproduced by a numpy model of the same roundings) at 2.6% of the output
// RMS in max-abs error on Q4_K layers, above the 1% bar; f16 rounds 8x finer at
// the same tensor-core rate.
//
// Persistent kernel: one CTA per SM walks work items (tile, row block)
// blockIdx.x, blockIdx.x + gridDim.x, ... Warp roles (23 warps):
//   warp 0      TMA producer of the raw quant blocks of the item's 128 weight
//               rows (2-D tensor maps over the expert-major qs and header
//               planes, 128 values per stage, a deep ring)
//   warp 22     TMA producer of the token operand (f16 rows, 128B swizzle,
//               K-major, one box of the tile's height per K step; no multicast
//               anywhere)
//   warp 1      one thread issues tcgen05.mma with the weight operand A in TMEM
//               and the token operand B in shared memory, fp32 accumulators in
//               TMEM (two, so an item's epilogue overlaps the next main loop),
//               tcgen05.commit to the ring barriers
//   warps 2-17  dequantise from shared memory with packed half2 arithmetic
//               (Q4_K: s*q - m per 32-value sub-block; Q8_0: d*q) and write A
//               into TMEM with tcgen05.st (row m of A = TMEM lane m, two f16 per
//               column; four A stages of one 64-value K step); the block headers
//               ride in the same TMA stages
//   warps 18-21 epilogue: tcgen05.ld of the accumulators 16 columns at a time,
//               f16 results staged in shared memory for 16-byte stores
// The weight tile never passes through shared memory as f16, which halves the
// shared memory traffic per K step.
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
constexpr int kStages = 4;                            // K-step stages (A in TMEM, B in shared memory)
constexpr int kBStages = kStages;
constexpr uint32_t kBStageBytes = kGemmNT * kBK * 2;  // 24 KiB: up to 192 token rows x 128 B
constexpr uint32_t kRawRing = 96 * 1024;
// TMEM columns
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccStride = kGemmNT;     // 192 columns per accumulator, two accumulators
// A stages (kStages, one 64-value K step each): 128 rows x 64 f16 = 32 columns each
constexpr uint32_t kAStageCols = 32;
constexpr uint32_t kAColBase = 2 * kGemmNT;  // 384: the A stages fill columns 384-511

enum : int { kErrRawFull = 1, kErrBFull = 2, kErrEmpty = 3, kErrAcc = 4, kErrAFull = 5, kErrAEmpty = 6 };

struct GemmParams {
    QMat A0, A1;          // routed: gate, up (gate/up GEMM) or down
    QMat S0, S1;          // shared expert
    const GemmTile* tiles;
    const int32_t* n_tiles;
    int K, Ks;            // reduction length for routed / shared items
    int MT, MTs, MTmax;   // row blocks (items) per tile for routed / shared
    int e_begin;          // first expert held by the planes (expert parallelism)
    __half* out;
    int out_ld;
    int32_t* err;
    int32_t* err_host;    // host-mapped copy of the first code, or null
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
    CUtensorMap b[kBMaps];  // token operand tiles: xperm (gate/up) or act (down) rows
    CUtensorMap w0, w1, s0, s1, mw0, mw1, ms0, ms1;
};

template <int DT, bool GATEUP>
struct Cfg {
    static constexpr int kRawRowBytes = DT == AERO_DT_Q4_K ? kRawK / 2 : kRawK;  // 64 or 128
    // 128 weight rows per raw stage either way: gate/up items take 64 rows of
    // each matrix, down items 128 rows
    static constexpr uint32_t kQsBytes = (uint32_t)kTileM * kRawRowBytes;
    static constexpr uint32_t kMetaBytes = (uint32_t)kTileM * 16;  // a 16-byte header slice per row
    static constexpr uint32_t kRawStageBytes = kQsBytes + kMetaBytes;
    static constexpr int kRawStages = (int)(kRawRing / kRawStageBytes);
    static constexpr int kRowsPerMat = GATEUP ? kTileM / 2 : kTileM;  // weight rows of one matrix per item
    static constexpr size_t kSmem = kRawRing + (size_t)kBStages * kBStageBytes + 1024 + 512 + 4 * 1024;
};

// Values of a K step are written to TMEM in the order 0, 2, 1, 3, 4, 6, 5, 7,
// ... (the middle two of every four swapped): a 32-bit word of 4 quant bytes
// then becomes two f16 pairs (bytes 0, 2) and (bytes 1, 3) with one shift and
// two masks. The token operand is stored with the same order (x16_kernel,
// and the gate/up epilogue for the down GEMM's operand), so the products are
// unchanged.
__device__ __forceinline__ int kperm(int k) { return (k & ~3) | ((k & 1) << 1) | ((k >> 1) & 1); }

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
    // barrier table: raw_full[kRS], raw_empty[kRS], full[kStages], empty[kStages], acc_full[2],
    // acc_empty[2], drain. A K step's A stage (TMEM) and B stage (shared memory) share one
    // index and one pair of barriers: full completes when the 16 dequant warps have
    // arrived and the token copy has landed, empty when the step's MMAs have finished.
    auto raw_full = [&](int s) { return bar0 + 8u * s; };
    auto raw_empty = [&](int s) { return bar0 + 8u * (kRS + s); };
    auto full = [&](int s) { return bar0 + 8u * (2 * kRS + s); };
    auto empty = [&](int s) { return bar0 + 8u * (2 * kRS + kStages + s); };
    auto acc_full = [&](int s) { return bar0 + 8u * (2 * kRS + 2 * kStages + s); };
    auto acc_empty = [&](int s) { return bar0 + 8u * (2 * kRS + 2 * kStages + 2 + s); };
    const uint32_t drain_bar = bar0 + 8u * (2 * kRS + 2 * kStages + 4);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kRS + 2 * kStages + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kRS + 2 * kStages + 6);
    uint8_t* epi_smem = b_ring + kBStages * kBStageBytes + 512;  // 4 warps x 1 KiB output staging

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRS; ++s) {
            mbar_init(raw_full(s), 1);
            mbar_init(raw_empty(s), kDeqWarps);
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full(s), kDeqWarps + 1);  // + the token producer's expect_tx arrival
            mbar_init(empty(s), 1);
        }
        for (int s = 0; s < 2; ++s) {
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
        if (atomicCAS(p.err, 0, code) == 0 && p.err_host) {
            *reinterpret_cast<volatile int32_t*>(p.err_host) = code;
            __threadfence_system();
        }
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------------------------------------------------- producer
            int raw_n = 0;
            bool ok = true;
            Item it;
            for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x) {
                const CUtensorMap* w0 = it.shared ? &tm.s0 : &tm.w0;
                const CUtensorMap* w1 = it.shared ? &tm.s1 : &tm.w1;
                const CUtensorMap* m0 = it.shared ? &tm.ms0 : &tm.mw0;
                const CUtensorMap* m1 = it.shared ? &tm.ms1 : &tm.mw1;
                const QMat& A = it.shared ? p.S0 : p.A0;
                const int y0 = (it.shared ? 0 : (it.t.expert - p.e_begin)) * A.rows + it.mt * C::kRowsPerMat;
                for (int kb = 0; kb < it.nkb && ok; kb += 2) {
                    const int s = raw_n % kRS;
                    if (!mbar_wait(raw_empty(s), ((raw_n / kRS) & 1) ^ 1, abort_flag)) {
                        fail(kErrEmpty);
                        ok = false;
                        break;
                    }
                    const uint32_t dst = smem_u32(raw_ring + s * C::kRawStageBytes);
                    mbar_expect_tx(raw_full(s), C::kRawStageBytes);
                    // qs of values [64 kb, 64 kb + 128), and the 16-byte header slice
                    // covering the 256 values around them; gate/up: gate rows then up rows
                    const int x = (kb / 2) * C::kRawRowBytes;
                    const int xm = (kb / 4) * 16;
                    tma_load_2d(dst, w0, x, y0, raw_full(s));
                    tma_load_2d(dst + C::kQsBytes, m0, xm, y0, raw_full(s));
                    if (GATEUP) {
                        tma_load_2d(dst + C::kRowsPerMat * C::kRawRowBytes, w1, x, y0, raw_full(s));
                        tma_load_2d(dst + C::kQsBytes + C::kRowsPerMat * 16, m1, xm, y0, raw_full(s));
                    }
                    ++raw_n;
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
                    const int sb = b_n % kStages;
                    if (!mbar_wait(empty(sb), ((b_n / kStages) & 1) ^ 1, abort_flag)) {
                        fail(kErrEmpty);
                        ok = false;
                        break;
                    }
                    const uint32_t dst = smem_u32(b_ring + sb * kBStageBytes);
                    mbar_expect_tx(full(sb), (uint32_t)it.N * kBK * 2);
                    tma_load_2d(dst, bm, kb * kBK, it.t.pos0, full(sb));
                    ++b_n;
                }
            }
            if (!ok) {
                // the copies in flight land whatever the dequant warps do: wait for
                // their bytes with a timed wait on the stage's transaction count
                for (int i = 0; i < kStages && i < b_n; ++i) {
                    const int n = b_n - 1 - i;
                    mbar_wait_timed(full(n % kStages), (n / kStages) & 1);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------------------------------------------------- MMA issuer
            int a_n = 0, item_n = 0;
            bool ok = true, issued = false;
            Item it;
            for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x, ++item_n) {
                const int ab = item_n & 1;
                if (!mbar_wait(acc_empty(ab), ((item_n >> 1) & 1) ^ 1, abort_flag)) {
                    fail(kErrAcc);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t idesc = idesc_f16(kTileM, it.N);
                const uint32_t d0 = tmem + (uint32_t)ab * kAccStride;
                for (int kb = 0; kb < it.nkb; ++kb) {
                    const int sa = a_n % kStages;
                    if (!mbar_wait(full(sa), (a_n / kStages) & 1, abort_flag)) {
                        fail(kErrAFull);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t b = smem_u32(b_ring + sa * kBStageBytes);
                    const uint32_t a0 = tmem + kAColBase + (uint32_t)sa * kAStageCols;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_ts(d0, a0 + kk * 8, sw128_desc(b + kk * 32), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
                    issued = true;
                    umma_commit(empty(sa));
                    ++a_n;
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
        // c = (warp - 2) / 4 takes one 32-value quant sub-block (Q4_K) or block
        // (Q8_0) per raw stage of two 64-value K steps: K step kb + c / 2, values
        // [32 (c & 1), 32 (c & 1) + 32) (16 TMEM columns), so each thread decodes
        // one scale per stage. TMEM lane r is weight row r of the item; gate/up items
        // interleave the matrices by half-warps: in lane quarter q, lanes 0-15 hold
        // gate rows 16 q + (0..15) and lanes 16-31 the same rows of up (so the
        // raw-stage rows an 8-lane phase reads are consecutive: no bank conflicts).
        const int cmb = (warp - 2) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const int srow = GATEUP ? (lane >> 4) * (kTileM / 2) + q * 16 + (lane & 15) : r;  // row in the raw stage
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        const int swz = DT == AERO_DT_Q4_K ? ((srow >> 1) & 3) : (srow & 7);
        const int step = cmb >> 1, half = cmb & 1;
        // this thread's 32 values of K step ks: the 32 raw bytes (two 16-byte chunks
        // of its stage row, TMA-swizzled: 64B for Q4_K rows of 64 bytes, 128B for Q8_0
        // rows of 128 bytes, logical chunk c at c ^ f(row)) and the row's header slice
        uint4 meta, v0, v1;
        auto load = [&](int rn, int ks) {
            const uint8_t* stage = raw_ring + (rn % kRS) * C::kRawStageBytes;
            const uint8_t* qrow = stage + srow * C::kRawRowBytes;
            meta = *reinterpret_cast<const uint4*>(stage + C::kQsBytes + srow * 16);
            const int c = DT == AERO_DT_Q4_K ? 2 * (ks & 1) : 4 * (ks & 1) + 2 * half;
            v0 = *reinterpret_cast<const uint4*>(qrow + ((c ^ swz) << 4));
            v1 = *reinterpret_cast<const uint4*>(qrow + (((c + 1) ^ swz) << 4));
        };
        // -> 16 TMEM columns (f16 pairs in the kperm order)
        auto convert = [&](int ks, uint32_t (&cols)[16]) {
            const uint32_t wv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
            if (DT == AERO_DT_Q4_K) {
                // the K step's 32 bytes: low nibbles are its values 0-31 (sub-block 2g),
                // high nibbles 32-63 (sub-block 2g+1)
                int sc, mn;
                q4k_sc_m_words(meta.y, meta.z, meta.w, 2 * (ks & 3) + half, sc, mn);
                // (d sc, dmin m) in f16: the 6-bit sc and m are exact as 1024 + v - 1024,
                // and one rounding of the exact products equals the f32 route's
                const __half2 k1024 = u2h(0x64006400u);
                const __half2 scm = __hsub2(u2h((uint32_t)sc | ((uint32_t)mn << 16) | 0x64006400u), k1024);
                const __half2 prod = __hmul2(u2h(meta.x), scm);  // meta.x = (d, dmin)
                const __half2 sh = __low2half2(prod), nh = __hneg2(__high2half2(prod));
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t w0 = half ? wv[i] >> 4 : wv[i];
                    const uint32_t w1 = wv[i] >> (half ? 12 : 8);
                    // (bytes 0, 2) and (bytes 1, 3): 1024 + q exactly, then s q - m
                    const __half2 q02 = __hsub2(u2h((w0 & 0x000F000Fu) | 0x64006400u), k1024);
                    const __half2 q13 = __hsub2(u2h((w1 & 0x000F000Fu) | 0x64006400u), k1024);
                    cols[2 * i] = h2u(__hfma2(q02, sh, nh));
                    cols[2 * i + 1] = h2u(__hfma2(q13, sh, nh));
                }
            } else {
                // the 16-byte slice holds 8 fp16 scales for 256 values; this thread's
                // 32 values are block 2 (ks & 3) + half
                const int kq = ks & 3;
                const uint32_t sc8 = kq == 0 ? meta.x : kq == 1 ? meta.y : kq == 2 ? meta.z : meta.w;
                const __half2 dd = __half2half2(__ushort_as_half((unsigned short)(half ? (sc8 >> 16) : (sc8 & 0xFFFFu))));
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint32_t wb = wv[i] ^ 0x80808080u;
                    cols[2 * i] = h2u(__hmul2(byte2_to_h2(__byte_perm(wb, 0, 0x4240)), dd));
                    cols[2 * i + 1] = h2u(__hmul2(byte2_to_h2(__byte_perm(wb, 0, 0x4341)), dd));
                }
            }
        };
        // Passes over the CTA's items, both K steps of a raw stage per pass (item K
        // lengths are multiples of 128): one raw wait, one header load, one
        // tcgen05.wait::st for two stages. (Issuing the next pass's raw wait and
        // loads before this pass's arrivals measured slower.)
        int raw_n = 0, a_n = 0;
        bool ok = true;
        Item it;
        for (int w = blockIdx.x; ok && item_at(p, n_tiles, w, it); w += gridDim.x) {
            for (int kb = 0; kb < it.nkb; kb += 2) {
                const int s = raw_n % kRS;
                const int sa0 = a_n % kStages, sa1 = (a_n + 1) % kStages;
                // one lane polls the barriers; __syncwarp orders the rest of the warp
                // after its acquire
                bool got = true;
                if (lane == 0) {
                    got = mbar_wait(raw_full(s), (raw_n / kRS) & 1, abort_flag) &&
                          mbar_wait(empty(sa0), ((a_n / kStages) & 1) ^ 1, abort_flag) &&
                          mbar_wait(empty(sa1), (((a_n + 1) / kStages) & 1) ^ 1, abort_flag);
                    if (!got) fail(kErrAEmpty);
                }
                if (!__shfl_sync(0xffffffffu, got, 0)) {
                    ok = false;
                    break;
                }
                __syncwarp();
                tc_fence_after();
                load(raw_n, kb + step);
                uint32_t cc[16];
                convert(kb + step, cc);
                tmem_st16(tmem + lane_base + kAColBase + (uint32_t)(step ? sa1 : sa0) * kAStageCols +
                              (uint32_t)half * 16u,
                          cc);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    // every dequant warp arrives on both stages of the pass
                    mbar_arrive(full(sa0));
                    mbar_arrive(full(sa1));
                    mbar_arrive(raw_empty(s));
                }
                a_n += 2;
                ++raw_n;
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
            const int ab = item_n & 1;
            const bool got = __shfl_sync(0xffffffffu, lane == 0 ? mbar_wait(acc_full(ab), (item_n >> 1) & 1, abort_flag) : false, 0);
            if (!got) {
                if (lane == 0) fail(kErrAcc);
                break;
            }
            __syncwarp();
            tc_fence_after();
            const uint32_t d0 = tmem + lane_base + (uint32_t)ab * kAccStride;
            if (GATEUP) {
                // lanes i / i + 16 hold gate / up row 16 q + i of the item's 64 rows.
                // Per 16 token columns: swap with the partner lane, the gate lane forms
                // act for tokens 0-7, the up lane for tokens 8-15; stage [16 tok][16 f]
                // (f in the permuted K order of the down GEMM) and store 32-byte rows.
                const int fl = lane & 15, upl = lane >> 4;
                const int fcol = kperm(16 * q + fl) - 16 * q;  // within this warp's 16 f columns
                __half* const out0 = p.out + (int64_t)it.t.pos0 * p.out_ld + it.mt * (kTileM / 2) + 16 * q;
                for (int c0 = 0; c0 < it.N; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(d0 + c0, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        // gate lane: tokens j, own gate with the partner's up; up lane: tokens 8 + j
                        const uint32_t send = upl ? v[j] : v[8 + j];
                        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 16);
                        const float g = __uint_as_float(upl ? recv : v[j]);
                        const float u = __uint_as_float(upl ? v[8 + j] : recv);
                        stage[(8 * upl + j) * 16 + fcol] = __float2half_rn(__fdividef(g, 1.0f + __expf(-g)) * u);
                    }
                    __syncwarp();
                    {
                        // lane -> (token row, half) of the staged tile: one 16-byte store each
                        const int tok = lane >> 1, hf = lane & 1;
                        const uint4 o = *reinterpret_cast<const uint4*>(stage + tok * 16 + 8 * hf);
                        if (c0 + tok < it.t.nvalid)
                            *reinterpret_cast<uint4*>(out0 + (int64_t)(c0 + tok) * p.out_ld + 8 * hf) = o;
                    }
                    __syncwarp();
                }
            } else {
                // 16 columns (tokens) at a time: one TMEM round trip, then the f16 results
                // go through this warp's 16 x 32 staging tile so each lane stores 16 bytes
                __half* const out_row0 = p.out + (int64_t)it.t.pos0 * p.out_ld + it.mt * kTileM + q * 32 + (lane & 3) * 8;
                for (int c0 = 0; c0 < it.N; c0 += 16) {
                    uint32_t g[16];
                    tmem_ld16(d0 + c0, g);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) stage[j * 32 + lane] = __float2half_rn(__uint_as_float(g[j]));
                    __syncwarp();
#pragma unroll
                    for (int r8 = 0; r8 < 2; ++r8) {
                        const int j = r8 * 8 + (lane >> 2);
                        const uint4 v = *reinterpret_cast<const uint4*>(stage + j * 32 + (lane & 3) * 8);
                        if (c0 + j < it.t.nvalid) *reinterpret_cast<uint4*>(out_row0 + (int64_t)(c0 + j) * p.out_ld) = v;
                    }
                    __syncwarp();
                }
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
// x16 row r = input row r as f16 with its values in the GEMM's K order (0, 2,
// 1, 3 within every four: kperm). One warp per row, 8 values (one 16-byte
// store) per lane per chunk.
template <typename XT>
__global__ void x16_kernel(const XT* __restrict__ x, int rows, int dp, __half* __restrict__ x16) {
    const int lane = threadIdx.x & 31;
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    for (int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r < rows; r += nw) {
        __half* dst = x16 + (int64_t)r * dp;
#pragma unroll 4
        for (int c = lane * 8; c < dp; c += 256) {
            uint4 o;
            if constexpr (sizeof(XT) == 2) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(x + (int64_t)r * dp + c));
                o = make_uint4(__byte_perm(u.x, u.y, 0x5410), __byte_perm(u.x, u.y, 0x7632),
                               __byte_perm(u.z, u.w, 0x5410), __byte_perm(u.z, u.w, 0x7632));
            } else {
                const float* src = reinterpret_cast<const float*>(x) + (int64_t)r * dp + c;
                const float4 a = ld_f4(src), b = ld_f4(src + 4);
                o = make_uint4(pack_h2(a.x, a.z), pack_h2(a.y, a.w), pack_h2(b.x, b.z), pack_h2(b.y, b.w));
            }
            *reinterpret_cast<uint4*>(dst + c) = o;
        }
    }
}

// xperm rows: [0, P_real) the routed pairs in sorted order, [P, P + Tsh) the
// first Tsh input rows for the shared expert, copied from x16 (which the 34 MB
// of a config-5 call keep in L2). P_real (= offsets[E]) is read on the device:
// sorted positions [P_real, P) hold skipped slots and are not gathered. One
// warp per row, 16-byte copies.
__global__ void gather_kernel(const __half* __restrict__ x16, const int32_t* __restrict__ perm,
                              const int32_t* __restrict__ p_real, int k, int P, int Tsh, int dp,
                              __half* __restrict__ xp) {
    const int pr = *p_real;
    const int rows = pr + Tsh;
    const int lane = threadIdx.x & 31;
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    for (int v = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); v < rows; v += nw) {
        const int row = v < pr ? v : P + (v - pr);
        const int tok = v < pr ? perm[v] / k : v - pr;
        const uint4* src = reinterpret_cast<const uint4*>(x16 + (int64_t)tok * dp);
        uint4* dst = reinterpret_cast<uint4*>(xp + (int64_t)row * dp);
#pragma unroll 4
        for (int c = lane; c < dp / 8; c += 32) dst[c] = __ldg(src + c);
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
// Each thread owns 8 columns (one 16-byte load of f16 per row it reads). The
// result rows are f32, or f16 when OUT_F16 (partial rows of an expert-parallel
// step that cross the network).
template <bool OUT_F16>
__global__ void combine_h_kernel(const __half* __restrict__ y, const int32_t* __restrict__ inv,
                                 const float* __restrict__ w, const float* __restrict__ sgate,
                                 const int32_t* __restrict__ idx, int E_real, int T, int Tsh, int k, int d,
                                 int has_shared, void* __restrict__ out_v) {
    const int d8 = d >> 3;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)T * d8) return;
    const int t = (int)(i / d8), c = (int)(i % d8) * 8;
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    auto add = [&](float wt, const __half* row) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(row + c));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(u2h(u[j]));
            a[2 * j] += wt * f.x;
            a[2 * j + 1] += wt * f.y;
        }
    };
    for (int s = 0; s < k; ++s) {
        if (idx && idx[(int64_t)t * k + s] >= E_real) continue;
        add(w[(int64_t)t * k + s], y + (int64_t)inv[(int64_t)t * k + s] * d);
    }
    if (has_shared && t < Tsh) add(sgate[t], y + ((int64_t)T * k + t) * d);
    if constexpr (OUT_F16) {
        *reinterpret_cast<uint4*>(static_cast<__half*>(out_v) + (int64_t)t * d + c) =
            make_uint4(pack_h2(a[0], a[1]), pack_h2(a[2], a[3]), pack_h2(a[4], a[5]), pack_h2(a[6], a[7]));
    } else {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(out_v) + (int64_t)t * d + c);
        o[0] = make_float4(a[0], a[1], a[2], a[3]);
        o[1] = make_float4(a[4], a[5], a[6], a[7]);
    }
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
                     int n_local_experts, int box_bytes, CUtensorMapSwizzle swz, int box_rows) {
    auto fn = encode_fn();
    if (!fn || !base) return false;
    if ((uint64_t)estride != row_bytes * (uint64_t)rows || row_bytes % 16) return false;
    cuuint64_t dims[2] = {row_bytes, (cuuint64_t)rows * (cuuint64_t)n_local_experts};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
    cuuint32_t es[2] = {1u, 1u};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// qs plane: the raw bytes of 128 values per box row (Q4_K 64 B, 64B swizzle;
// Q8_0 128 B, 128B swizzle). Header plane: 16-byte slices, no swizzle.
// box_rows: 64 for the gate/up families (an item takes 64 rows of each), 128 for down.
bool make_tmap_qs(CUtensorMap* m, const QMat& q, int n_local, int box_rows) {
    const bool q4 = q.dtype == AERO_DT_Q4_K;
    return make_tmap_plane(m, q.qs, (uint64_t)qm_row_qs_bytes(q.dtype, q.cols), q.rows, q.qs_estride, n_local,
                           q4 ? kRawK / 2 : kRawK, q4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, box_rows);
}
bool make_tmap_meta(CUtensorMap* m, const QMat& q, int n_local, int box_rows) {
    return make_tmap_plane(m, q.meta, (uint64_t)qm_row_meta_bytes(q.dtype, q.cols), q.rows, q.meta_estride, n_local, 16,
                           CU_TENSOR_MAP_SWIZZLE_NONE, box_rows);
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
    return al((size_t)T * dp * 2) + al(rows * dp * 2) + al(rows * act_ld * 2) + al(rows * dp * 2) +
           al((size_t)max_tiles * sizeof(GemmTile)) + 1024;
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
    b->x16 = reinterpret_cast<__half*>(c);
    c += al((size_t)T_cap * dp * 2);
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
    const int h = kTileM / 2;
    bool ok = make_tmap_qs(&m->q[0], gate, n_local, h) && make_tmap_qs(&m->q[1], up, n_local, h) &&
              make_tmap_qs(&m->q[2], down, n_local, kTileM) && make_tmap_meta(&m->m[0], gate, n_local, h) &&
              make_tmap_meta(&m->m[1], up, n_local, h) && make_tmap_meta(&m->m[2], down, n_local, kTileM);
    if (ok && has_shared)
        ok = make_tmap_qs(&m->q[3], sg, 1, h) && make_tmap_qs(&m->q[4], su, 1, h) && make_tmap_qs(&m->q[5], sd, 1, kTileM) &&
             make_tmap_meta(&m->m[3], sg, 1, h) && make_tmap_meta(&m->m[4], su, 1, h) &&
             make_tmap_meta(&m->m[5], sd, 1, kTileM);
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
        const int64_t warps = a.T;  // a warp per input row
        const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, (int64_t)a.n_sm * 16));
        if (a.x_f16)
            x16_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(a.x), a.T, a.dp, b.x16);
        else
            x16_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(a.x), a.T, a.dp, b.x16);
    }
    {
        const int64_t warps = (int64_t)(P + Tsh);  // a warp per row
        const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((warps + 7) / 8, (int64_t)a.n_sm * 16));
        gather_kernel<<<grid, 256, 0, s>>>(b.x16, a.perm, a.p_real, a.k, P, Tsh, a.dp, b.xperm);
    }
    build_tiles_kernel<<<1, 1024, 0, s>>>(a.act_e, a.act_off, a.n_active, P, Tsh, a.has_shared, b.tiles, b.n_tiles);
    return cudaGetLastError();
}

cudaError_t launch_prefill_gemm(const PrefillArgs& a, GemmBuffers& b, const GemmWeightMaps& wm, bool gateup,
                                cudaStream_t s) {
    // the kernel's stages pair up K steps: every reduction length is a multiple of 128
    if (a.dp % kRawK || a.F % kRawK || (a.has_shared && a.Fs % kRawK)) return cudaErrorInvalidValue;
    GemmParams g{};
    g.tiles = b.tiles;
    g.n_tiles = b.n_tiles;
    g.err = b.err;
    g.err_host = b.err_host;
    g.e_begin = a.e_begin;
    GemmMaps maps{};
    if (gateup) {
        g.A0 = a.gate;
        g.A1 = a.up;
        g.S0 = a.has_shared ? a.sg : a.gate;
        g.S1 = a.has_shared ? a.su : a.up;
        g.K = a.dp;
        g.Ks = a.dp;
        g.MT = a.F / (kTileM / 2);  // 64 rows of gate and of up per item
        g.MTs = a.has_shared ? a.Fs / (kTileM / 2) : 0;
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
                             const int32_t* idx, int E_real, int T, int Tsh, int k, int d, int has_shared, void* out,
                             int out_f16, cudaStream_t s) {
    const int64_t n = (int64_t)T * (d / 8);
    if (n == 0) return cudaSuccess;
    if (out_f16)
        combine_h_kernel<true><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, inv, w, sgate, idx, E_real, T, Tsh, k, d,
                                                                           has_shared, out);
    else
        combine_h_kernel<false><<<(unsigned)((n + 255) / 256), 256, 0, s>>>(y, inv, w, sgate, idx, E_real, T, Tsh, k,
                                                                            d, has_shared, out);
    return cudaGetLastError();
}

}  // namespace aero
