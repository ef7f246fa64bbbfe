// Expert-parallel exchange over peer memory: one process per GPU, each rank's
// exchange window mapped into every other rank's address space (CUDA IPC over
// NVLink / NVSwitch), so the rows and the partial outputs cross as stores from
// the kernels that produce them (rows staged in shared memory and sent with
// bulk copies), with no collective library in the step.
//
// Window of rank q (same layout on every rank; slab s holds the rows of rank
// (q + s) mod n, so slab 0 is q's own tokens):
//   rows [n][slab][dp]      token rows (f16 or f32) written by their owner
//   meta [n][slab][meta_ld] metadata rows (k ids owned by q or -1, k weights,
//                           shared gate, padding)
//   back [n][slab][dp]      partial outputs of q's rows computed by rank
//                           (q + s) mod n, in q's row order for that rank
//   cnt  [n]                rows in each slab this step
//   flag_rows [n], flag_back [n]   step number of the last completed write
//   done_pack, done_ret     CTA counters of the two writing kernels
//   err                     first wait that gave up (0: none)
// A step (epoch e):
//   pack    one warp per token: rows + metadata into the destination windows
//           (rows in arrival order within a slab); the last CTA then writes
//           cnt and flag_rows = e into every peer's window
//   prep    waits for flag_rows = e from every peer, then metadata -> buckets
//   (this rank's experts over its window rows)
//   return  each row's partial output into its owner's back slab (slab 0:
//           this rank's y); on the GEMM path this is the expert block's
//           combine itself. The last CTA sets flag_back = e in every peer's
//           window
//   combine waits for flag_back = e, then self part + remote parts in rank
//           order (the same sum, in the same order, as the all-to-all path)
// One buffer per direction suffices: a rank writes step e+1 rows into a peer
// only after its own step-e combine, which waited for that peer's step-e
// returns, which the peer sent after it had finished reading its step-e rows;
// and a peer returns step e+1 partials only after reading step e+1 rows, which
// this rank writes after its step-e combine has read the step-e partials.
// Every wait is bounded (wait_ns of %globaltimer, a handle option, 5 s by
// default): on expiry the CTA records an error code in the window (and in the
// handle's host-mapped error word), later waits of the rank return at once, and
// the host reads the code (aero_cuda_ep_peer_status, or the next call).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "internal.h"

namespace aero {
namespace {

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Row stores through the bulk-copy engine: a warp stages a row in shared
// memory and one lane copies it to the (local or peer) destination with
// cp.async.bulk (plain bulk copies shared -> global, no multicast); 16-byte
// aligned addresses and sizes.
__device__ __forceinline__ uint32_t sh_u32(const void* q) { return (uint32_t)__cvta_generic_to_shared(q); }
__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the staged rows may be overwritten
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// the copies are complete, ordered before this thread's later generic stores
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
// this thread's shared-memory writes, visible to the bulk-copy engine
__device__ __forceinline__ void fence_to_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

constexpr int kRowWarps = 8;  // warps (staging rows) per CTA of the row-moving kernels

template <typename T>
__device__ __forceinline__ T* wptr(const EpPeerTable& p, int rank, int64_t off) {
    return reinterpret_cast<T*>(p.base[rank] + off);
}

// Thread 0 waits until flags[1..n-1] of this rank's window reach `epoch`; the
// CTA gets the result. A wait that runs out records `code` in the window.
__device__ bool peer_wait(const EpPeerTable& p, int64_t flag_off, uint32_t epoch, int code) {
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        volatile int32_t* err = wptr<int32_t>(p, p.me, p.off_err);
        const uint32_t* flags = wptr<const uint32_t>(p, p.me, flag_off);
        int ok = *err == 0;
        const uint64_t t0 = gtimer();
        for (int s = 1; s < p.n && ok; ++s) {
            while ((int32_t)(ld_acquire_sys(flags + s) - epoch) < 0) {
                if (*err != 0) {
                    ok = 0;
                    break;
                }
                if (gtimer() - t0 > p.wait_ns) {
                    if (atomicCAS(const_cast<int32_t*>(err), 0, code) == 0 && p.err_host) {
                        *reinterpret_cast<volatile int32_t*>(p.err_host) = code;
                        __threadfence_system();
                    }
                    ok = 0;
                    break;
                }
                __nanosleep(128);
            }
        }
        __threadfence();
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// Called by every thread of every CTA after its stores: the last CTA to get
// here runs `last(tid)` for tid in [0, blockDim) after all CTAs' stores are
// visible system-wide. (The barrier orders the CTA's stores before thread 0's
// system-scope fence, which is cumulative over them.)
template <typename F>
__device__ __forceinline__ void after_all_ctas(uint32_t* done, F last) {
    __shared__ int is_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        is_last = atomicAdd(done, 1u) == gridDim.x - 1;
        if (is_last) {
            *done = 0;  // ready for the next launch
            __threadfence_system();
        }
    }
    __syncthreads();
    if (is_last) last((int)threadIdx.x);
}

__device__ __forceinline__ uint32_t pack_h2f(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Rows and metadata of this rank's tokens into every destination window, one
// warp per token: the token's k experts name its destination ranks; its row
// is read and converted once, then stored to each destination (slab 0 of this
// rank's own window at row t; for rank r != me, slab (me - r) mod n of r's
// window at the next free row j, taken from slot_ctr[r]). pos[t*n + r] is where
// the token's partial for r comes back in this rank's window
// (((r - me) mod n) * slab + j, or t for r = me, -1 where r holds none of its
// experts). Rows sit in arrival order within a slab: a row's result does not
// depend on its position. The last CTA publishes the counts and raises
// flag_rows in every peer's window, then clears slot_ctr for the next step.
template <typename RT>
__global__ void ep_peer_pack_kernel(EpPeerTable p, const float* __restrict__ x, int T,
                                    const int32_t* __restrict__ idx, const float* __restrict__ w,
                                    const float* __restrict__ sgate, int has_shared, EpRankTable rt,
                                    int32_t* __restrict__ slot_ctr, int32_t* __restrict__ counts,
                                    int32_t* __restrict__ pos, uint32_t epoch) {
    constexpr int kMaxChunks = 8;  // dp <= 2048: 8 chunks of 8 values per lane
    const int n = p.n, me = p.me, slab = p.slab, dp = p.dp, k = p.k;
    const int lane = threadIdx.x & 31;
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    const int nch = dp / 256;
    extern __shared__ __align__(16) uint8_t row_stage[];
    RT* srow = reinterpret_cast<RT*>(row_stage + (size_t)(threadIdx.x >> 5) * dp * sizeof(RT));
    const uint32_t row_bytes = (uint32_t)(dp * sizeof(RT));
    for (int t = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); t < T; t += nw) {
        // destination ranks of this token's slots
        int e = -1, owner = -1;
        if (lane < k) {
            e = idx[(int64_t)t * k + lane];
            owner = 0;
            while (owner + 1 < n && e >= rt.begin[owner + 1]) ++owner;
        }
        uint32_t lo_bits = owner >= 0 && owner < 32 ? 1u << owner : 0u;
        uint32_t hi_bits = owner >= 32 ? 1u << (owner - 32) : 0u;
        lo_bits = __reduce_or_sync(0xffffffffu, lo_bits);
        hi_bits = __reduce_or_sync(0xffffffffu, hi_bits);
        const uint64_t dests = ((uint64_t)hi_bits << 32 | lo_bits) | (1ull << me);
        const float wt = lane < k ? w[(int64_t)t * k + lane] : 0.f;
        const float sg = has_shared ? sgate[t] : 0.f;
        // the row, converted once into this warp's staging row (after the bulk
        // copies of the previous token have read it)
        float4 fa[kMaxChunks], fb[kMaxChunks];
        const float* src = x + (int64_t)t * dp;
#pragma unroll
        for (int i = 0; i < kMaxChunks; ++i)
            if (i < nch) {
                fa[i] = ld_f4(src + i * 256 + lane * 8);
                fb[i] = ld_f4(src + i * 256 + lane * 8 + 4);
            }
        if (lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int i = 0; i < kMaxChunks; ++i)
            if (i < nch) {
                const float4 a = fa[i], b = fb[i];
                if constexpr (sizeof(RT) == 2) {
                    *reinterpret_cast<uint4*>(srow + i * 256 + lane * 8) =
                        make_uint4(pack_h2f(a.x, a.y), pack_h2f(a.z, a.w), pack_h2f(b.x, b.y), pack_h2f(b.z, b.w));
                } else {
                    float* o = reinterpret_cast<float*>(srow) + i * 256 + lane * 8;
                    *reinterpret_cast<float4*>(o) = a;
                    *reinterpret_cast<float4*>(o + 4) = b;
                }
            }
        fence_to_async_shared();
        __syncwarp();
        int my_pos = -1;  // lane r < n: pos[t*n + r]
        for (uint64_t rest = dests; rest; rest &= rest - 1) {
            const int r = __ffsll((long long)rest) - 1;
            int j = t;
            if (r != me) {
                if (lane == 0) j = atomicAdd(slot_ctr + r, 1);
                j = __shfl_sync(0xffffffffu, j, 0);
            }
            const int s = (r - me + n) % n;                          // r's slab in this rank's window
            const int64_t drow = (int64_t)((n - s) % n) * slab + j;  // the row in r's window
            if (lane == r) my_pos = s * slab + j;
            if (lane == 0) bulk_store(wptr<RT>(p, r, p.off_rows) + drow * dp, sh_u32(srow), row_bytes);
            int32_t* m = wptr<int32_t>(p, r, p.off_meta) + drow * p.meta_ld;
            if (lane < k) {
                m[lane] = owner == r ? e : -1;
                m[k + lane] = __float_as_int(wt);
            }
            if (lane < p.meta_ld - 2 * k) m[2 * k + lane] = lane == 0 ? __float_as_int(r == me ? sg : 0.f) : 0;
        }
        if (lane < n) pos[(int64_t)t * n + lane] = my_pos;
        if (lane == 0) bulk_commit();
    }
    if (lane == 0) bulk_wait_all();
    after_all_ctas(wptr<uint32_t>(p, me, p.off_done_pack), [&](int tid) {
        if (tid == me) {
            counts[me] = T;
            wptr<int32_t>(p, me, p.off_cnt)[0] = T;
        } else if (tid < n) {
            const int r = tid, slot = (me - r + n) % n;
            const int c = slot_ctr[r];
            counts[r] = c;
            slot_ctr[r] = 0;  // for the next step
            wptr<int32_t>(p, r, p.off_cnt)[slot] = c;
            st_release_sys(wptr<uint32_t>(p, r, p.off_flag_rows) + slot, epoch);
        }
    });
}

// Waits for every peer's rows, then metadata rows of the window -> buckets
// (E for slots owned elsewhere and for unused slab rows), weights, shared gates
// (slab 0 rows only). Ids that are neither -1 nor owned here count in *bad.
__global__ void ep_peer_prep_kernel(EpPeerTable p, int T, int e_begin, int e_end, int E, uint32_t epoch,
                                    int32_t* __restrict__ idx, float* __restrict__ w, float* __restrict__ sgate,
                                    int32_t* __restrict__ bad) {
    peer_wait(p, p.off_flag_rows, epoch, kEpErrRowsWait);
    const int k = p.k, R = p.n * p.slab;
    const volatile int32_t* cnt = wptr<int32_t>(p, p.me, p.off_cnt);
    const int32_t* meta = wptr<const int32_t>(p, p.me, p.off_meta);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)R * k;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / k), q = (int)(i % k);
        const int s = r / p.slab, j = r % p.slab;
        const bool valid = j < (s == 0 ? T : cnt[s]);
        const int32_t* m = meta + (int64_t)r * p.meta_ld;
        const int e = valid ? m[q] : -1;
        const bool own = e >= e_begin && e < e_end;
        if (!own && e != -1) atomicAdd(bad, 1);
        idx[i] = own ? e : E;
        w[i] = valid ? __int_as_float(m[k + q]) : 0.f;
        if (q == 0) sgate[r] = r < T ? __int_as_float(m[2 * k]) : 0.f;
    }
}

// y rows of slabs 1..n-1 into the owners' back slabs (one warp per row,
// 16-byte units), then the last CTA raises flag_back in every peer's window.
template <typename PT>
__global__ void ep_peer_return_kernel(EpPeerTable p, const PT* __restrict__ y, uint32_t epoch,
                                      int32_t* __restrict__ recv_out) {
    const int n = p.n, me = p.me, slab = p.slab;
    const int lane = threadIdx.x & 31;
    const int units = p.dp * (int)sizeof(PT) / 16;
    const int rows = (n - 1) * slab;
    const volatile int32_t* cnt = wptr<int32_t>(p, me, p.off_cnt);
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    for (int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); row < rows; row += nw) {
        const int s = 1 + row / slab, j = row - (s - 1) * slab;
        if (j >= cnt[s]) continue;  // whole warp
        const int owner = (me + s) % n;
        const uint4* src = reinterpret_cast<const uint4*>(y + ((int64_t)s * slab + j) * p.dp);
        uint4* dst = reinterpret_cast<uint4*>(wptr<PT>(p, owner, p.off_back) + ((int64_t)(n - s) * slab + j) * p.dp);
#pragma unroll 4
        for (int u = lane; u < units; u += 32) dst[u] = src[u];
    }
    after_all_ctas(wptr<uint32_t>(p, me, p.off_done_ret), [&](int tid) {
        // this step's received counts, kept before the peers may write the next step's
        if (tid < n) recv_out[tid] = cnt[tid];
        if (tid >= 1 && tid < n) {
            const int owner = (me + tid) % n;
            st_release_sys(wptr<uint32_t>(p, owner, p.off_flag_back) + (n - tid), epoch);
        }
    });
}

// The expert block's last step fused with the return: window row r gets
// sum over its slots of w * ye[inv] (+ sgate * ye[R*k + r] for the self rows)
// from the f16 per-expert GEMM outputs ye, written as PT straight to its
// destination: this rank's y for slab 0, the owner's back slab otherwise
// (padding rows are skipped). One warp per row, 8 values per lane per chunk.
// Then the last CTA raises flag_back in every peer's window.
template <typename PT>
__global__ void ep_peer_combine_return_kernel(EpPeerTable p, const __half* __restrict__ ye,
                                              const int32_t* __restrict__ inv, const float* __restrict__ w,
                                              const float* __restrict__ sgate, const int32_t* __restrict__ idx,
                                              int E_real, int T, int has_shared, PT* __restrict__ yself,
                                              uint32_t epoch, int32_t* __restrict__ recv_out) {
    const int n = p.n, me = p.me, slab = p.slab, dp = p.dp, k = p.k;
    const int lane = threadIdx.x & 31;
    const int R = n * slab;
    const volatile int32_t* cnt = wptr<int32_t>(p, me, p.off_cnt);
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    extern __shared__ __align__(16) uint8_t row_stage[];
    PT* srow = reinterpret_cast<PT*>(row_stage + (size_t)(threadIdx.x >> 5) * dp * sizeof(PT));
    for (int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r < R; r += nw) {
        const int s = r / slab, j = r - s * slab;
        if (j >= (s == 0 ? T : cnt[s])) continue;  // whole warp
        if (lane == 0) bulk_wait_read();  // the previous row's copy has read the staging row
        __syncwarp();
        PT* dst = s == 0 ? yself + (int64_t)j * dp
                         : wptr<PT>(p, (me + s) % n, p.off_back) + ((int64_t)(n - s) * slab + j) * dp;
        // this row's slots, lane q holding slot q (k <= 32)
        int my_row = -1;
        float my_w = 0.f;
        if (lane < k && idx[(int64_t)r * k + lane] < E_real) {
            my_row = inv[(int64_t)r * k + lane];
            my_w = w[(int64_t)r * k + lane];
        }
        const bool sh = has_shared && s == 0;
        const float sw = sh ? sgate[j] : 0.f;
        for (int c = lane * 8; c < dp; c += 256) {
            float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            auto add = [&](float wt, const __half* row) {
                const uint4 v = *reinterpret_cast<const uint4*>(row + c);
                const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const __half2 h2 = *reinterpret_cast<const __half2*>(&u[q]);
                    const float2 f = __half22float2(h2);
                    a[2 * q] += wt * f.x;
                    a[2 * q + 1] += wt * f.y;
                }
            };
            for (int q = 0; q < k; ++q) {
                const int row = __shfl_sync(0xffffffffu, my_row, q);
                const float wt = __shfl_sync(0xffffffffu, my_w, q);
                if (row >= 0) add(wt, ye + (int64_t)row * dp);
            }
            if (sh) add(sw, ye + ((int64_t)R * k + j) * dp);
            if constexpr (sizeof(PT) == 2) {
                *reinterpret_cast<uint4*>(srow + c) =
                    make_uint4(pack_h2f(a[0], a[1]), pack_h2f(a[2], a[3]), pack_h2f(a[4], a[5]), pack_h2f(a[6], a[7]));
            } else {
                float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(srow) + c);
                o[0] = make_float4(a[0], a[1], a[2], a[3]);
                o[1] = make_float4(a[4], a[5], a[6], a[7]);
            }
        }
        fence_to_async_shared();
        __syncwarp();
        if (lane == 0) {
            bulk_store(dst, sh_u32(srow), (uint32_t)(dp * sizeof(PT)));
            bulk_commit();
        }
    }
    if (lane == 0) bulk_wait_all();
    after_all_ctas(wptr<uint32_t>(p, me, p.off_done_ret), [&](int tid) {
        // this step's received counts, kept before the peers may write the next step's
        if (tid < n) recv_out[tid] = cnt[tid];
        if (tid >= 1 && tid < n) {
            const int owner = (me + tid) % n;
            st_release_sys(wptr<uint32_t>(p, owner, p.off_flag_back) + (n - tid), epoch);
        }
    });
}

// 8 values of a partial row (f16 or f32) added to acc.
template <typename PT>
__device__ __forceinline__ void add8(const PT* q, float (&acc)[8]) {
    if constexpr (sizeof(PT) == 2) {
        const uint4 v = *reinterpret_cast<const uint4*>(q);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(q), b = *reinterpret_cast<const float4*>(q + 4);
        acc[0] += a.x, acc[1] += a.y, acc[2] += a.z, acc[3] += a.w;
        acc[4] += b.x, acc[5] += b.y, acc[6] += b.z, acc[7] += b.w;
    }
}

// Waits for every peer's returns, then out[t] = y[t] + the remote parts in
// ascending rank order. One warp per (token, 256-value chunk): lane r holds
// pos[t][r], each lane adds 8 values of every part.
template <typename PT>
__global__ void ep_peer_combine_kernel(EpPeerTable p, const PT* __restrict__ y, const int32_t* __restrict__ pos, int T,
                                       uint32_t epoch, float* __restrict__ out) {
    peer_wait(p, p.off_flag_back, epoch, kEpErrBackWait);
    const int n = p.n, dp = p.dp, nch = dp / 256;
    const int lane = threadIdx.x & 31;
    const PT* back = wptr<const PT>(p, p.me, p.off_back);
    const int nw = (int)((gridDim.x * blockDim.x) >> 5);
    for (int u = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); u < T * nch; u += nw) {
        const int t = u / nch, c = (u - t * nch) * 256 + lane * 8;
        const int my_pos = lane < n && lane != p.me ? pos[(int64_t)t * n + lane] : -1;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        add8(y + (int64_t)t * dp + c, acc);
        for (int r = 0; r < n; ++r) {
            const int q = __shfl_sync(0xffffffffu, my_pos, r);
            if (q >= 0) add8(back + (int64_t)q * dp + c, acc);
        }
        float4* o = reinterpret_cast<float4*>(out + (int64_t)t * dp + c);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

unsigned grid_for(int64_t items, int n_sm, int per_sm) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, (int64_t)n_sm * per_sm));
}

}  // namespace

EpPeerTable ep_peer_layout(int n, int me, int slab, int dp, int k, int rows_f16, size_t* bytes) {
    EpPeerTable p{};
    p.n = n;
    p.me = me;
    p.slab = slab;
    p.dp = dp;
    p.k = k;
    p.meta_ld = 2 * k + 2;
    p.rows_f16 = rows_f16;
    const int64_t R = (int64_t)n * slab;
    const int64_t esz = rows_f16 ? 2 : 4;
    int64_t off = 0;
    auto take = [&](int64_t b) {
        const int64_t o = off;
        off += (b + 255) & ~(int64_t)255;
        return o;
    };
    p.off_rows = take(R * dp * esz);
    p.off_meta = take(R * p.meta_ld * 4);
    p.off_back = take(R * dp * esz);
    p.off_cnt = take((int64_t)n * 4);
    p.off_flag_rows = take((int64_t)n * 4);
    p.off_flag_back = take((int64_t)n * 4);
    p.off_done_pack = take(4);
    p.off_done_ret = take(4);
    p.off_err = take(4);
    *bytes = (size_t)off;
    return p;
}

cudaError_t launch_ep_peer_pack(const EpPeerTable& p, const float* x, int T, const int32_t* idx, const float* w,
                                const float* sgate, int has_shared, const EpRankTable& rt, int32_t* slot_ctr,
                                int32_t* counts, int32_t* pos, uint32_t epoch, int n_sm, cudaStream_t s) {
    if (p.dp % 256 || p.dp > 2048 || p.k > 32 || p.n > 32) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kRowWarps * p.dp * (p.rows_f16 ? 2 : 4);
    const unsigned grid = grid_for((int64_t)std::max(T, 1) * 32, n_sm, 4);  // a warp per token
    cudaError_t e;
    if (p.rows_f16) {
        e = cudaFuncSetAttribute(ep_peer_pack_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        ep_peer_pack_kernel<__half><<<grid, kRowWarps * 32, smem, s>>>(p, x, T, idx, w, sgate, has_shared, rt, slot_ctr,
                                                                      counts, pos, epoch);
    } else {
        e = cudaFuncSetAttribute(ep_peer_pack_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        ep_peer_pack_kernel<float><<<grid, kRowWarps * 32, smem, s>>>(p, x, T, idx, w, sgate, has_shared, rt, slot_ctr,
                                                                     counts, pos, epoch);
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_peer_prep(const EpPeerTable& p, int T, int e_begin, int e_end, int E, uint32_t epoch,
                                int32_t* idx, float* w, float* sgate, int32_t* bad, int n_sm, cudaStream_t s) {
    const unsigned grid = grid_for((int64_t)p.n * p.slab * p.k, n_sm, 4);
    ep_peer_prep_kernel<<<grid, 256, 0, s>>>(p, T, e_begin, e_end, E, epoch, idx, w, sgate, bad);
    return cudaGetLastError();
}

cudaError_t launch_ep_peer_return(const EpPeerTable& p, const void* y, uint32_t epoch, int32_t* recv_out, int n_sm,
                                  cudaStream_t s) {
    const unsigned grid = grid_for((int64_t)(p.n - 1) * p.slab * 32, n_sm, 8);  // a warp per row
    if (p.rows_f16)
        ep_peer_return_kernel<__half><<<grid, 256, 0, s>>>(p, static_cast<const __half*>(y), epoch, recv_out);
    else
        ep_peer_return_kernel<float><<<grid, 256, 0, s>>>(p, static_cast<const float*>(y), epoch, recv_out);
    return cudaGetLastError();
}

cudaError_t launch_ep_peer_combine_return(const EpPeerTable& p, const __half* ye, const int32_t* inv, const float* w,
                                          const float* sgate, const int32_t* idx, int E_real, int T, int has_shared,
                                          void* yself, uint32_t epoch, int32_t* recv_out, int n_sm,
                                          cudaStream_t s) {
    if (p.dp % 256) return cudaErrorInvalidValue;
    const size_t smem = (size_t)kRowWarps * p.dp * (p.rows_f16 ? 2 : 4);
    const unsigned grid = grid_for((int64_t)p.n * p.slab * 32, n_sm, 4);  // a warp per row
    cudaError_t e;
    if (p.rows_f16) {
        e = cudaFuncSetAttribute(ep_peer_combine_return_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
        ep_peer_combine_return_kernel<__half><<<grid, kRowWarps * 32, smem, s>>>(
            p, ye, inv, w, sgate, idx, E_real, T, has_shared, static_cast<__half*>(yself), epoch, recv_out);
    } else {
        e = cudaFuncSetAttribute(ep_peer_combine_return_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
        if (e != cudaSuccess) return e;
        ep_peer_combine_return_kernel<float><<<grid, kRowWarps * 32, smem, s>>>(
            p, ye, inv, w, sgate, idx, E_real, T, has_shared, static_cast<float*>(yself), epoch, recv_out);
    }
    return cudaGetLastError();
}

cudaError_t launch_ep_peer_combine(const EpPeerTable& p, const void* y, const int32_t* pos, int T, uint32_t epoch,
                                   float* out, int n_sm, cudaStream_t s) {
    if (p.dp % 256) return cudaErrorInvalidValue;
    const unsigned grid = grid_for((int64_t)std::max(T, 1) * (p.dp / 256) * 32, n_sm, 8);  // a warp per chunk
    if (p.rows_f16)
        ep_peer_combine_kernel<__half><<<grid, 256, 0, s>>>(p, static_cast<const __half*>(y), pos, T, epoch, out);
    else
        ep_peer_combine_kernel<float><<<grid, 256, 0, s>>>(p, static_cast<const float*>(y), pos, T, epoch, out);
    return cudaGetLastError();
}

}  // namespace aero
