// Prefill grouped GEMM (tcgen05 / TMEM) entry points.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "common.cuh"

namespace aero {

// One tile of token rows for one expert segment: rows [pos0, pos0 + nvalid) of
// the permuted activation buffers. expert < 0 marks the shared expert.
struct GemmTile {
    int32_t expert, pos0, nvalid, pad;
};

constexpr int kGemmNT = 192;  // token rows per tile (the MMA N extent)

// Upper bound on the number of tiles for P routed pairs and T tokens.
inline int gemm_max_tiles(int P, int T, int E, int has_shared) {
    const int act = P < E ? P : E;
    return act + (P + kGemmNT - 1) / kGemmNT + (has_shared ? (T + kGemmNT - 1) / kGemmNT : 0);
}

// Device workspace the prefill path needs (tile list + f16 operand buffers).
size_t gemm_workspace_bytes(int dp, int act_ld, int P, int T, int max_tiles);

struct GemmBuffers {
    __half* x16;     // (T_cap, dp)       the call's input rows as f16, in the GEMM's K order
    __half* xperm;   // (rows_cap, dp)    x16 rows by sorted position (shared expert: P + token)
    __half* act;     // (rows_cap, act_ld) act rows by sorted position (shared expert: P + token)
    __half* y;       // (rows_cap, dp)
    GemmTile* tiles;        // (max tiles)
    int32_t* n_tiles;
    int32_t* err;           // pipeline timeout code (0 = none)
    int32_t* err_host = nullptr;  // host-mapped copy of the first code, or null
    int rows_cap;
    CUtensorMap tmap_x[kGemmNT / 16], tmap_act[kGemmNT / 16];  // box heights 16, 32, ..., kGemmNT
};

// A 2-D tiled TMA descriptor over a row-major matrix (rows x cols elements of
// elem_bytes, row stride ld elements): box box_rows x box_cols, no OOB fill.
bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* base, uint64_t rows,
                    uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz);

// Carve the workspace and encode the TMA descriptors for it.
bool gemm_setup(void* ws, size_t ws_bytes, int dp, int act_ld, int P_cap, int T_cap, int max_tiles, GemmBuffers* b,
                std::string* why);

// TMA descriptors of the expert weight planes: q[] the qs planes, m[] the
// header planes, in the order gate, up, down, shared gate, shared up, shared down.
struct GemmWeightMaps {
    CUtensorMap q[6], m[6];
};
// Encode them for planes whose qs/meta pointers are the allocation bases.
bool gemm_weight_maps(const QMat& gate, const QMat& up, const QMat& down, const QMat& sg, const QMat& su, const QMat& sd,
                      int n_local, int has_shared, GemmWeightMaps* m, std::string* why);

struct PrefillArgs {
    QMat gate, up, down, sg, su, sd;
    const void* x;            // (T, dp) f32, or f16 when x_f16
    int x_f16;
    int Tsh;                  // the shared expert runs on rows [0, Tsh)
    const int32_t* p_real;    // device: number of sorted positions that hold real pairs
    const int32_t* perm;      // sorted position -> pair
    const int32_t* act_e;
    const int32_t* act_off;
    const int32_t* n_active;
    int T, k, dp, F, Fs, has_shared, E;
    int act_ld;
    int e_begin;   // first expert held by the planes
    int n_sm;      // persistent grid size
};

// The prefill path: launch_prefill_prep (the f16 copy of the input rows, its
// rows gathered into sorted-pair order, the tile list: 3 kernels), then
// launch_prefill_gemm with gateup=true (gate/up GEMM + SwiGLU into act) and
// gateup=false (down GEMM into y, f16, rows [0, P + Tsh)); the combine reads y
// with launch_combine_h.
cudaError_t launch_prefill_prep(const PrefillArgs& a, GemmBuffers& b, cudaStream_t s);
cudaError_t launch_prefill_gemm(const PrefillArgs& a, GemmBuffers& b, const GemmWeightMaps& wm, bool gateup,
                                cudaStream_t s);
// out[t] = sum_s w[t][s] * y[inv[t*k+s]] (+ sgate[t] * y[P + t] for t < Tsh); with
// idx non-null, slots whose bucket idx[t*k+s] >= E_real are skipped. out rows
// are f32, or f16 with out_f16.
cudaError_t launch_combine_h(const __half* y, const int32_t* inv, const float* w, const float* sgate,
                             const int32_t* idx, int E_real, int T, int Tsh, int k, int d, int has_shared,
                             void* out, int out_f16, cudaStream_t s);

// Router projection on the tensor cores (router_tc.cu): f32-accurate logits
// from three TF32 products of split operands, for prefill batches.
constexpr int kRtNMax = 128;
struct RouterTcMaps {
    CUtensorMap hi, lo;  // W_hi / W_lo tiles of N (<= kRtNMax) rows x 32 values
    int N, n_rows, dp;
};
// Rows per CTA column tile for n_rows router rows; 0 when the shape is not supported.
int router_tc_tile_rows(int n_rows);
// Split W (n_rows, dp) f32 into w_hi / w_lo (same shape, device) and encode their maps.
cudaError_t router_tc_prepare(const float* W, int n_rows, int dp, float* w_hi, float* w_lo, RouterTcMaps* maps,
                              cudaStream_t s);
// logits[t][e] = x_t . W[e] (+ bias[e] for e < n_bias) for t < T, e < n_rows;
// with gate_row, logits[t][n_rows] = x_t . gate_row (f32, K in order). ld % 4 == 0.
// partial (partial_rows x ld floats, may be null) lets small batches split K
// over more CTAs; the splits are summed in a fixed order.
cudaError_t launch_router_tc(const RouterTcMaps& maps, const float* x, int T, const float* bias, int n_bias,
                             const float* gate_row, float* logits, int ld, int32_t* err, int32_t* err_host,
                             float* partial, int partial_rows, int n_sm, cudaStream_t s);

}  // namespace aero
