// Host-side declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "common.cuh"

namespace aero {

// ---------------------------------------------------------------- kernels
// Router projection: logits[t][r] = x_t . W[r] (+ bias[r] for r < n_bias), for
// rows r in [row_begin, row_end) of the (n_rows, d) f32 matrix W; logits has row
// stride ld. Chooses a GEMV form for small T and a tiled SIMT GEMM for large T.
cudaError_t launch_router(const float* x, int T, int d, const float* W, int row_begin, int row_end,
                          const float* bias, int n_bias, float* logits, int ld, cudaStream_t s);

// Input rows of the decode GEMVs in integer form: per 32-value block b of a row,
// x ~= sx[b] * (128 * q1 + q0) with q1 in [-128, 127] and q0 in [0, 127] (a
// 15-bit code split into two int8 planes, so quant codes meet it in dp4a), plus
// the exact f32 sums of every 16 values (the Q4_K min term). Rows of K values:
// q1, q0 K bytes each, sx K/32 and s16 K/16 floats.
struct QInput {
    int8_t* q1;
    int8_t* q0;
    float* sx;
    float* s16;
    int K;  // values per row
};
inline size_t qinput_bytes(int rows, int K) {
    return (size_t)rows * ((size_t)2 * K + (size_t)K / 32 * 4 + (size_t)K / 16 * 4);
}
// Carves a QInput for `rows` rows of K values out of `base` (qinput_bytes long, 16-byte aligned).
inline QInput qinput_at(void* base, int rows, int K) {
    char* b = static_cast<char*>(base);
    QInput q;
    q.q1 = reinterpret_cast<int8_t*>(b);
    q.q0 = reinterpret_cast<int8_t*>(b + (size_t)rows * K);
    q.sx = reinterpret_cast<float*>(b + (size_t)2 * rows * K);
    q.s16 = reinterpret_cast<float*>(b + (size_t)2 * rows * K + (size_t)rows * (K / 32) * 4);
    q.K = K;
    return q;
}
// Quantises R rows of x (row stride ld floats) into q (K = q.K values per row).
cudaError_t launch_qinput(const float* x, int R, int ld, QInput q, cudaStream_t s);

// The dispatch of a single-token call, written by the top-k pass: its k pairs
// are k distinct experts, each pair its own segment in slot order (perm, inv
// identity; act_e = the selected experts, act_off[i] = i, n_active = k,
// *p_real = k). Pairs computed independently and combined in slot order give
// the same result as the expert-sorted dispatch.
struct SingleDispatch {
    int32_t *perm = nullptr, *inv = nullptr, *act_e = nullptr, *act_off = nullptr, *n_active = nullptr,
            *p_real = nullptr;
};
// Top-k over logits[t][0..E) (row stride ld): idx/w (T, k), sgate[t] =
// sigmoid(logits[t][E]) when has_shared. With xq.q1 non-null, also writes token
// t's row of x (T, xq.K) as integer input. With T == 1 and one.perm non-null,
// also writes that call's dispatch (SingleDispatch).
cudaError_t launch_topk(const float* logits, int ld, int T, int E, int k, int norm, int has_shared, int32_t* idx,
                        float* w, float* sgate, const float* x, QInput xq, cudaStream_t s,
                        SingleDispatch one = SingleDispatch{});

// Resident-subset layers: idx[0..n) global expert ids -> slot[id] (the
// expert's position in the layer's planes). An id whose slot is -1 records
// kErrNotResident in *err (and *err_host when non-null) and maps to slot 0.
constexpr int kErrNotResident = 41;
cudaError_t launch_resident_remap(int32_t* idx, int n, const int32_t* slot, int32_t* err, int32_t* err_host,
                                  cudaStream_t s);

// Dispatch: expert-contiguous permutation of the T*k pairs. Writes offsets[E+1],
// perm[P] (sorted position -> pair), inv[P] (pair -> sorted position), the active
// list act_e[n_active] / act_off[n_active+1] (segment starts, in sorted
// positions) and n_active. `work` is scratch of dispatch_work_bytes(P, E).
// Buckets e >= n_real (default: none) are sorted but left out of the active
// list; act_off[n_active] is then offsets[n_real], the end of the real pairs.
size_t dispatch_work_bytes(int P, int E);
cudaError_t launch_dispatch(const int32_t* idx, int P, int E, int32_t* offsets, int32_t* perm,
                            int32_t* inv, int32_t* act_e, int32_t* act_off, int32_t* n_active,
                            void* work, cudaStream_t s, int n_real = -1);

struct GemvArgs {
    QMat gate, up, down;     // routed experts
    QMat sg, su, sd;         // shared expert (n_expert 1), valid when has_shared
    const float* x;          // (T, d)
    QInput xq;               // x rows as integer input (T rows, K = d), for quantised experts
    QInput aq;               // act rows as integer input (P + T rows, K = act_ld), written by gate/up
    const int32_t* perm;
    const int32_t* act_e;
    const int32_t* act_off;
    const int32_t* n_active;
    int T, k, d, F, Fs, has_shared, max_active;
    int max_pairs;           // upper bound on the pairs of one routed expert (min(T, ...))
    int Tsh;                 // the shared expert runs on tokens [0, Tsh)
    int act_ld;              // row stride of act (>= max(F, Fs))
    float* act;              // (P + T, act_ld)
    float* y;                // (P + T, d)
};
cudaError_t launch_gemv_gateup(const GemvArgs& a, cudaStream_t s);
cudaError_t launch_gemv_down(const GemvArgs& a, cudaStream_t s);

// out[t] = sum_s w[t][s] * y[inv[t*k+s]] (+ sgate[t] * y[P + t] for t < Tsh); with
// idx non-null, slots whose bucket idx[t*k+s] >= E_real are skipped.
cudaError_t launch_combine(const float* y, const int32_t* inv, const float* w, const float* sgate,
                           const int32_t* idx, int E_real, int T, int Tsh, int k, int d, int has_shared,
                           float* out, cudaStream_t s);

// Decode (decode.cu): the whole layer of a call of up to kDecodeMaxTokens tokens
// in one cooperative launch (router, top-k, dispatch, gate/up, down, combine),
// for Q8_0 / Q4_K experts.
constexpr int kDecodeMaxTokens = 32;
struct DecodeArgs {
    const float* x;           // (T, dp) f32
    const float* logits_in;   // caller logits (T, ld_in), or null: the router runs
    int ld_in;
    const float* router;      // (E + 1, dp) f32, row E = the shared-gate input
    const float* bias;        // (E) or null
    QMat gate, up, down, sg, su, sd;
    int T, E, k, norm, has_shared, dp, F, Fs;
    int act_ld;               // row length of the coded act rows (>= max(F, Fs), multiple of 64)
    float* logits;            // (T, lg_ld) scratch (column E: the shared-gate logit)
    int lg_ld;
    uint8_t* xq;              // T coded x rows (decode_qx_row_bytes(dp) each)
    float* act;               // (T * k + T, act_ld) f32 act rows by sorted position (shared expert: T * k + t)
    int32_t* idx_out;         // (T * k) selected experts (also the exchange of a call whose top-k is spread)
    float* w_out;             // (T * k)
    float* sgate_out;         // (T) shared-expert gates (exchange of a spread top-k)
    int32_t* n_active_out;    // active experts of the call
    int32_t* p_real_out;      // T * k
    float* y;                 // (T * k + T, dp) f32: each pair's expert output (shared expert: rows T * k + t)
    float* out;               // (T, dp) f32
    uint32_t* bar;            // [0] grid-barrier counter, [2] exit counter: both zero at every launch's
                              // start (the kernel's last CTA resets them; the host after an abort)
    int32_t* err;
    int32_t* err_host;
    uint64_t wait_ns;
    uint64_t* stamps;         // null, or 6 %globaltimer stamps of CTA 0: start, ends of phases A..E (profiling)
};
bool decode_supported(int dtype, int T, int E, int k, int dp, int F, int Fs, int has_shared);
int64_t decode_qx_row_bytes(int K);
// Grid barriers a launch of T tokens passes (each CTA adds one arrival per barrier).
int decode_barriers(int T);
// Launches the kernel on *grid_out CTAs.
cudaError_t launch_decode(const DecodeArgs& a, int n_sm, cudaStream_t s, int* grid_out);

// Expert-parallel exchange (ep.cu). Rank r owns experts [begin[r], begin[r+1]).
constexpr int kEpMaxRanks = 64;
struct EpRankTable {
    int n;
    int begin[kEpMaxRanks + 1];
};
// Send plan for T local tokens with top-k ids idx (T, k): send_tok/send_rank
// (S rows, remote ranks in order, tokens in order), counts[r] rows per rank and
// counts[n] = S, pos (T, n): the row of each (token, rank) in the slab layout of
// the send buffer (rank r's rows at [r * slab, r * slab + counts[r])) or -1.
cudaError_t launch_ep_plan(const int32_t* idx, int T, int k, const EpRankTable& rt, int me, int slab,
                           int32_t* send_tok, int32_t* send_rank, int32_t* counts, int32_t* pos, cudaStream_t s);
// Writes the self rows (T) and the n send slabs of `slab` rows (real rows, then
// padding whose metadata ids are all -1) with metadata rows of meta_ld int32:
// k ids (-1 where the destination does not own the slot's expert), k weights,
// the shared gate (self rows only), zero padding.
cudaError_t launch_ep_pack(const float* x, int T, int dp, int k, const int32_t* idx, const float* w,
                           const float* sgate, int has_shared, const EpRankTable& rt, int me, int slab,
                           const int32_t* send_tok, const int32_t* counts, int rows_f16, void* self_rows,
                           int32_t* self_meta, void* send_rows, int32_t* send_meta, int meta_ld, int n_sm,
                           cudaStream_t s);
// Receiver side: metadata -> idx (bucket E for slots owned elsewhere), w, sgate.
cudaError_t launch_ep_prep(const int32_t* meta, int meta_ld, int R, int k, int Tsh, int e_begin, int e_end, int E,
                           int32_t* idx, float* w, float* sgate, int32_t* bad, cudaStream_t s);
// out[t] = self_out[t] + sum over remote ranks (ascending) of back[pos[t][r]];
// the partial rows are f32, or f16 with parts_f16.
cudaError_t launch_ep_combine(const void* self_out, const void* back, int parts_f16, const int32_t* pos, int T, int n,
                              int me, int dp, float* out, cudaStream_t s);

// Expert-parallel exchange over peer memory (ep_peer.cu): every rank's window,
// mapped into this process, and the byte offsets of its regions (the same on
// every rank).
struct EpPeerTable {
    int n, me, slab, dp, k, meta_ld, rows_f16;
    uint64_t wait_ns;    // limit of every flag wait
    int32_t* err_host;   // host-mapped copy of the first expired wait's code, or null
    int64_t off_rows, off_meta, off_back, off_cnt, off_flag_rows, off_flag_back, off_done_pack, off_done_ret, off_err;
    char* base[kEpMaxRanks];
};
enum : int { kEpErrRowsWait = 21, kEpErrBackWait = 22 };
// Region offsets for n ranks, slabs of `slab` rows of dp values (f16 or f32);
// *bytes = window size.
EpPeerTable ep_peer_layout(int n, int me, int slab, int dp, int k, int rows_f16, size_t* bytes);
// Rows and metadata of the T local tokens into the destination windows (one warp
// per token; row slots taken from slot_ctr, zero between steps), pos (T, n): the
// row in this rank's window where the partial for (t, r) returns, or -1;
// counts[r] rows sent to r (counts[me] = T); then cnt and flag_rows = epoch in
// every peer. dp a multiple of 256 up to 2048.
cudaError_t launch_ep_peer_pack(const EpPeerTable& p, const float* x, int T, const int32_t* idx, const float* w,
                                const float* sgate, int has_shared, const EpRankTable& rt, int32_t* slot_ctr,
                                int32_t* counts, int32_t* pos, uint32_t epoch, int n_sm, cudaStream_t s);
// Waits for every peer's rows of this epoch, then window metadata -> idx / w / sgate (R = n * slab rows).
cudaError_t launch_ep_peer_prep(const EpPeerTable& p, int T, int e_begin, int e_end, int E, uint32_t epoch,
                                int32_t* idx, float* w, float* sgate, int32_t* bad, int n_sm, cudaStream_t s);
// y rows of the peers' slabs back into their windows, then flag_back = epoch in every peer.
// (both return launches copy the window's received counts to recv_out (n) first)
cudaError_t launch_ep_peer_return(const EpPeerTable& p, const void* y, uint32_t epoch, int32_t* recv_out, int n_sm,
                                  cudaStream_t s);
// GEMM path: the expert block's combine over the window rows (f16 per-expert
// outputs ye, slots from inv / w / idx, shared rows at ye[R*k + t]) written
// straight to y (slab 0) and the owners' back slabs, then flag_back = epoch.
cudaError_t launch_ep_peer_combine_return(const EpPeerTable& p, const __half* ye, const int32_t* inv, const float* w,
                                          const float* sgate, const int32_t* idx, int E_real, int T, int has_shared,
                                          void* yself, uint32_t epoch, int32_t* recv_out, int n_sm,
                                          cudaStream_t s);
// Waits for every peer's returns, then out[t] = y[t] + remote parts in rank order.
cudaError_t launch_ep_peer_combine(const EpPeerTable& p, const void* y, const int32_t* pos, int T, uint32_t epoch,
                                   float* out, int n_sm, cudaStream_t s);

// Quant helpers.
cudaError_t launch_repack(int dtype, const uint8_t* gguf, int64_t n_rows_total, int cols,
                          int rows_per_expert, int64_t expert0, uint8_t* qs, uint8_t* meta,
                          int64_t qs_estride, int64_t meta_estride, cudaStream_t s);
cudaError_t launch_dequant_gguf(int dtype, const uint8_t* gguf, int64_t n_values, float* out,
                                cudaStream_t s);
cudaError_t launch_quantize(int dtype, const float* x, int64_t n_values, uint8_t* out,
                            cudaStream_t s);
cudaError_t launch_f16_to_f32(const uint16_t* in, int64_t n, float* out, cudaStream_t s);

// ---------------------------------------------------------------- guard
enum MemClass { kWeightsResident = 0, kWeightsCache, kKVCache, kScratch, kRuntime, kMemClassCount };
bool guard_try_reserve(size_t bytes, int cls);
void guard_release(size_t bytes, int cls);
// cudaMalloc charged to the guard; returns cudaErrorMemoryAllocation when refused.
cudaError_t guarded_malloc(void** p, size_t bytes, int cls);
// Device (or managed) memory, as cudaPointerGetAttributes reports it.
bool is_device_ptr(const void* p);
void guarded_free(void* p, size_t bytes, int cls);

std::string fmt_bytes(size_t b);

// Sets the message aero_cuda_moe_last_error(NULL) returns on this thread.
void set_free_error(const std::string& msg);

}  // namespace aero
