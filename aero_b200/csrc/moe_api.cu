// The C ABI of the library: layer handles, upload, and per-call orchestration.
//
// A call runs: router projection -> top-k -> dispatch -> expert products ->
// combine, all on the handle's stream with no host synchronisation in between
// (the number of active experts lives on the device; grids are sized for the
// maximum and surplus CTAs exit). Semantics follow engine/moe.py:117-177 and
// src/moe.cpp:122-161.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/aero_cuda_moe.h"
#include "gemm.h"
#include "gguf_loader.h"
#include "internal.h"

namespace aero {
bool is_device_ptr(const void* p) {
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

namespace {

thread_local std::string g_free_error;

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

struct Alloc {
    void* p;
    size_t bytes;
    int cls;
};

// rows of split-K partial logits kept for the tensor-core router (splits x tokens)
constexpr int kRouterPartRows = 8192;

struct Scratch {
    int cap_T = 0;
    void* base = nullptr;
    size_t bytes = 0;
    float *x_stage, *out_stage, *lg_stage, *logits, *w, *sgate, *act, *y;
    float* lg_part = nullptr;  // router split-K partials (lg_part_rows x lg_ld)
    int lg_part_rows = 0;
    int32_t *idx, *offsets, *perm, *inv, *act_e, *act_off, *n_active, *ep_bad, *tc_err;
    void* dwork;
    QInput xq{}, aq{};  // GEMV inputs in integer form (null planes for F32 experts)
    void* gemm_ws;
    size_t gemm_ws_bytes = 0;
    int gemv_cap = 0;
    // fused decode path: coded x and act rows, grid-barrier counter and error word
    uint8_t* dxq = nullptr;
    float *dact = nullptr, *dy = nullptr;
    uint32_t* dbar = nullptr;
    int32_t* derr = nullptr;
    uint64_t* dstamps = nullptr;  // phase stamps of the fused decode kernel (profiling)
};

// Expert-parallel exchange over peer memory: this rank's window (IPC-exported),
// the peers' windows mapped here, and the step's local buffers.
struct PeerCtx {
    bool open = false, connected = false;
    EpPeerTable tab{};
    EpRankTable rt{};
    char* window = nullptr;
    size_t window_bytes = 0;
    void* y = nullptr;  // expert-block output for the window's rows (row type)
    size_t y_bytes = 0;
    int32_t* aux = nullptr;  // slot counters (n), counts (n + 1), pos (slab * n), received (n)
    size_t aux_bytes = 0;
    std::vector<char*> mapped;  // peers' windows opened here
    uint32_t epoch = 0;
    // first code of a peer wait that gave up, once the host has seen it: the
    // exchange's waits return at once from then on, so later steps are refused
    int32_t failed = 0;
    // phase timing (profiling): route, plan, pack, rows wait + unpack, experts, return, combine
    static constexpr int kPhases = 7;
    bool prof = false;
    cudaEvent_t ev[kPhases + 1] = {};
    double ms[kPhases] = {};
    long n_prof = 0;
};

constexpr int kAsyncSlots = 4;

struct Handle {
    int device = 0;
    cudaStream_t stream = nullptr, own_stream = nullptr;
    std::mutex mu;
    int d = 0, dp = 0, E = 0, k = 0, F = 0, Fp = 0, Fs = 0, Fsp = 0, norm = 1, has_shared = 0;
    int e_begin = 0, e_end = 0, has_router = 0, act_ld = 0;
    // resident subset: the planes hold the experts listed at open; slot[E] maps
    // a global id to its plane position (-1: not resident). Routed ids are
    // remapped after top-k, so dispatch and the expert products see slots.
    bool subset = false;
    int32_t* slot = nullptr;
    std::vector<int32_t> slot_owner;  // expert held by each plane slot (host mirror of `slot`)
    int dtype = 0, sh_dtype = 0;
    QMat gate{}, up{}, down{}, sg{}, su{}, sd{};
    float* router_ext = nullptr;  // (E + 1, dp): row E = shared gate input (or zeros)
    float* router_bias = nullptr;
    // tensor-core router for prefill batches: W split into TF32 hi / lo parts
    RouterTcMaps rtc{};
    bool rtc_ok = false;          // the layer's shape allows it
    bool rtc_enabled = true;      // AERO_CUDA_OPT_ROUTER_TC
    int lg_ld = 0;                // row stride of the logits scratch: E + 1 rounded up to 4
    std::vector<Alloc> allocs;
    Scratch sc;
    std::string err;
    long calls = 0, tokens = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.f;
    bool timing = false;
    // per-stage device time (profiling mode): stages are router, top-k,
    // dispatch, gate/up, down, combine
    static constexpr int kStages = 6;
    bool profiling = false;
    cudaEvent_t sev[kStages + 1] = {};
    double stage_ms[kStages] = {};
    long stage_n[kStages] = {};
    long launches = 0;        // kernels launched by this handle
    // host-mapped word where the kernels copy the first code of a bounded wait
    // that gave up: the host reads it at the next call without synchronising
    int32_t* err_host = nullptr;
    uint64_t peer_wait_ns = 5000000000ull;  // AERO_CUDA_OPT_PEER_WAIT_MS
    bool decode_enabled = true;             // AERO_CUDA_OPT_DECODE_FUSED
    // prefill (tcgen05 grouped GEMM) path
    bool gemm_ok = false;     // layer shape/type supports it
    int gemm_min_tokens = 64; // calls with at least this many tokens use it
    GemmBuffers gb{};
    bool gb_ready = false;
    GemmWeightMaps wmaps{};
    int n_sm = 148;
    int last_active = -1;     // active experts of the last profiled call
    int last_pairs = -1;      // its routed (token, expert) pairs computed here
    int last_shared_rows = 0; // its rows through the shared expert
    bool last_gemm = false;   // whether it took the GEMM path
    bool last_decode = false; // whether it took the fused decode kernel
    PeerCtx peer;
    // asynchronous host-buffer calls (aero_cuda_moe_submit / _wait): kAsyncSlots slots,
    // each with its device input / output rows; copies in and out run on their
    // own streams so one call's copies overlap another's block
    struct AsyncSlot {
        float *x = nullptr, *out = nullptr;  // (cap, dp) each, one allocation
        size_t bytes = 0;
        int cap = 0, T = 0;
        bool pending = false;
        cudaEvent_t in = nullptr, done = nullptr, copied = nullptr;
    } aslot[kAsyncSlots];
    cudaStream_t s_in = nullptr, s_out = nullptr;

    void peer_release() {
        for (char* m : peer.mapped)
            if (m) cudaIpcCloseMemHandle(m);
        peer.mapped.clear();
        if (peer.window) guarded_free(peer.window, peer.window_bytes, kScratch);
        if (peer.y) guarded_free(peer.y, peer.y_bytes, kScratch);
        if (peer.aux) guarded_free(peer.aux, peer.aux_bytes, kScratch);
        for (auto& e : peer.ev)
            if (e) cudaEventDestroy(e);
        peer = PeerCtx{};
    }

    ~Handle() {
        if (device >= 0) cudaSetDevice(device);
        if (own_stream) cudaStreamSynchronize(own_stream);
        if (peer.open) {
            cudaStreamSynchronize(stream);
            peer_release();
        }
        for (auto& q : aslot) {
            if (q.copied) cudaEventSynchronize(q.copied);
            if (q.x) guarded_free(q.x, q.bytes, kScratch);
            for (cudaEvent_t e : {q.in, q.done, q.copied})
                if (e) cudaEventDestroy(e);
        }
        if (s_in) cudaStreamDestroy(s_in);
        if (s_out) cudaStreamDestroy(s_out);
        for (auto& a : allocs) guarded_free(a.p, a.bytes, a.cls);
        if (sc.base) guarded_free(sc.base, sc.bytes, kScratch);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        for (auto& e : sev)
            if (e) cudaEventDestroy(e);
        if (own_stream) cudaStreamDestroy(own_stream);
        if (err_host) cudaFreeHost(err_host);
    }
    bool fail(const char* fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        err = buf;
        return false;
    }
    void mark(int i) {
        if (profiling) cudaEventRecord(sev[i], stream);
    }
    bool cuda_ok(cudaError_t e, const char* what) {
        if (e == cudaSuccess) return true;
        cudaGetLastError();
        return fail("%s: %s", what, cudaGetErrorString(e));
    }
    void* dalloc(size_t bytes, int cls, const char* what) {
        void* p = nullptr;
        const cudaError_t e = guarded_malloc(&p, bytes, cls);
        if (e != cudaSuccess) {
            cudaGetLastError();
            fail("device allocation of %s for %s refused: %s", fmt_bytes(bytes).c_str(), what,
                 e == cudaErrorMemoryAllocation ? "over the memory guard budget or out of device memory"
                                                : cudaGetErrorString(e));
            return nullptr;
        }
        allocs.push_back({p, bytes, cls});
        return p;
    }
};

int64_t dtype_block_values(int dt) { return dt == AERO_DT_Q8_0 ? 32 : dt == AERO_DT_Q4_K ? 256 : dt == AERO_DT_F32 ? 1 : 0; }
int64_t dtype_block_bytes(int dt) { return dt == AERO_DT_Q8_0 ? 34 : dt == AERO_DT_Q4_K ? 144 : dt == AERO_DT_F32 ? 4 : 0; }
int64_t gguf_bytes(int dt, int64_t n) {
    const int64_t bv = dtype_block_values(dt);
    return bv ? n / bv * dtype_block_bytes(dt) : -1;
}

// Upload one expert-tensor family (n_experts x rows x cols, GGUF bytes at src,
// host or device) into planes. F32 tensors are zero-padded to prow x pcol.
bool upload_family(Handle& h, const aero_cuda_tensor& t, int total_experts, int e0, int e1, int rows, int cols,
                   int prow, int pcol, QMat& m, const char* what) {
    const int dt = t.dtype;
    if (dt != AERO_DT_Q8_0 && dt != AERO_DT_Q4_K && dt != AERO_DT_F32)
        return h.fail("%s: unsupported ggml type %d (this library reads F32, Q8_0, Q4_K)", what, dt);
    const int64_t bv = dtype_block_values(dt);
    if (cols % bv) return h.fail("%s: row width %d is not a multiple of the %lld-value block", what, cols, (long long)bv);
    const int64_t per_expert = gguf_bytes(dt, (int64_t)rows * cols);
    if (!t.data || t.nbytes < per_expert * total_experts)
        return h.fail("%s: %lld bytes given, %lld needed", what, (long long)t.nbytes, (long long)(per_expert * total_experts));
    const int ne = e1 - e0;
    m.dtype = dt;
    m.rows = dt == AERO_DT_F32 ? prow : rows;
    m.cols = dt == AERO_DT_F32 ? pcol : cols;
    m.n_expert = ne;
    m.qs_estride = align128((int64_t)m.rows * qm_row_qs_bytes(dt, m.cols));
    m.meta_estride = align128((int64_t)m.rows * qm_row_meta_bytes(dt, m.cols));
    uint8_t* qs = (uint8_t*)h.dalloc((size_t)(m.qs_estride * ne), kWeightsResident, what);
    if (!qs) return false;
    uint8_t* meta = nullptr;
    if (m.meta_estride > 0) {
        meta = (uint8_t*)h.dalloc((size_t)(m.meta_estride * ne), kWeightsResident, what);
        if (!meta) return false;
    }
    m.qs = qs;
    m.meta = meta;
    const uint8_t* src = static_cast<const uint8_t*>(t.data) + (int64_t)e0 * per_expert;
    const bool src_dev = is_device_ptr(t.data);
    if (dt == AERO_DT_F32) {
        if (!h.cuda_ok(cudaMemsetAsync(qs, 0, (size_t)(m.qs_estride * ne), h.stream), what)) return false;
        for (int e = 0; e < ne; ++e)
            if (!h.cuda_ok(cudaMemcpy2DAsync(qs + (int64_t)e * m.qs_estride, (size_t)pcol * 4, src + (int64_t)e * per_expert,
                                             (size_t)cols * 4, (size_t)cols * 4, (size_t)rows,
                                             src_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, h.stream),
                           what))
                return false;
        return h.cuda_ok(cudaStreamSynchronize(h.stream), what);
    }
    // Quant families: host bytes stream through a bounded staging buffer (at
    // most 256 MiB of experts at a time), repacked on the device chunk by chunk.
    // The planes themselves were admitted as one plan at open and are charged
    // to the guard by their allocations.
    const int64_t chunk_experts = std::max<int64_t>(1, std::min<int64_t>(ne, (256ll << 20) / std::max<int64_t>(1, per_expert)));
    const int64_t stage_bytes = chunk_experts * per_expert;
    uint8_t* stage = nullptr;
    if (!src_dev) {
        void* p = nullptr;
        const cudaError_t e = guarded_malloc(&p, (size_t)stage_bytes, kScratch);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return h.fail("%s: staging buffer of %s refused", what, fmt_bytes((size_t)stage_bytes).c_str());
        }
        stage = (uint8_t*)p;
    }
    bool ok = true;
    for (int64_t c0 = 0; c0 < ne && ok; c0 += chunk_experts) {
        const int64_t cn = std::min<int64_t>(chunk_experts, ne - c0);
        const uint8_t* s = src + c0 * per_expert;
        if (!src_dev) {
            ok = h.cuda_ok(cudaMemcpyAsync(stage, s, (size_t)(cn * per_expert), cudaMemcpyHostToDevice, h.stream), what);
            s = stage;
        } else if (dt == AERO_DT_Q4_K && ((uintptr_t)s & 15) != 0) {
            ok = h.fail("%s: device source is not 16-byte aligned", what);
        }
        if (ok)
            ok = h.cuda_ok(launch_repack(dt, s, cn * rows, cols, rows, c0, qs, meta, m.qs_estride, m.meta_estride, h.stream),
                           what);
        if (ok && !src_dev) ok = h.cuda_ok(cudaStreamSynchronize(h.stream), what);  // staging reuse
    }
    if (ok) ok = h.cuda_ok(cudaStreamSynchronize(h.stream), what);
    if (stage) guarded_free(stage, (size_t)stage_bytes, kScratch);
    return ok;
}

bool ensure_scratch(Handle& h, int T) {
    if (T <= h.sc.cap_T && h.sc.base) return true;
    const int cap = std::max(T, std::max(2 * h.sc.cap_T, 8));
    const int64_t P = (int64_t)cap * h.k;
    const int64_t rows = P + cap;
    size_t off = 0;
    auto take = [&](size_t b) {
        const size_t o = off;
        off += (b + 255) & ~(size_t)255;
        return o;
    };
    const size_t o_x = take((size_t)cap * h.dp * 4), o_out = take((size_t)cap * h.dp * 4);
    const size_t o_lgs = take((size_t)cap * h.E * 4);
    const size_t o_lg = take((size_t)cap * h.lg_ld * 4), o_w = take((size_t)P * 4), o_sg = take((size_t)cap * 4);
    // the f32 GEMV buffers only need to cover calls that take the GEMV path
    const int64_t gemv_T = h.gemm_ok ? std::min<int64_t>(cap, h.gemm_min_tokens) : cap;
    const int64_t grows = gemv_T * h.k + gemv_T;
    const size_t o_act = take((size_t)grows * h.act_ld * 4);
    // integer forms of the GEMV inputs (quantised experts): x rows, act rows
    const bool qin = h.dtype != AERO_DT_F32;
    const size_t o_xq = take(qin ? qinput_bytes((int)gemv_T, h.dp) : 0);
    const size_t o_aq = take(qin ? qinput_bytes((int)grows, h.act_ld) : 0);
    const size_t o_y = take((size_t)grows * h.dp * 4);
    const size_t o_idx = take((size_t)P * 4), o_off = take((size_t)(h.E + 2) * 4), o_perm = take((size_t)P * 4);
    const size_t o_inv = take((size_t)P * 4), o_ae = take((size_t)h.E * 4), o_ao = take((size_t)(h.E + 1) * 4);
    const size_t o_na = take(4), o_dw = take(dispatch_work_bytes((int)P, h.E + 1));
    const size_t o_bad = take(4), o_tce = take(4);
    const int dT = std::min(cap, kDecodeMaxTokens);
    const bool dec = h.dtype != AERO_DT_F32;
    const size_t o_dxq = take(dec ? (size_t)dT * decode_qx_row_bytes(h.dp) : 0);
    const size_t o_dact = take(dec ? (size_t)(dT * h.k + dT) * h.act_ld * 4 : 0);
    const size_t o_dy = take(dec ? (size_t)(dT * h.k + dT) * h.dp * 4 : 0);
    const size_t o_dbar = take(16);  // decode barrier counter, error word, exit counter
    const size_t o_dst = take(6 * 8);
    // split-K partial logits of the tensor-core router (small batches)
    const int part_rows = h.rtc_ok ? (int)std::min<int64_t>(kRouterPartRows, (int64_t)8 * cap) : 0;
    const size_t o_lgp = take((size_t)part_rows * h.lg_ld * 4);
    const int max_tiles = gemm_max_tiles((int)P, cap, h.E, h.has_shared);
    const size_t gws = h.gemm_ok ? gemm_workspace_bytes(h.dp, h.act_ld, (int)P, cap, max_tiles) : 256;
    const size_t o_gw = take(gws);
    void* base = nullptr;
    const cudaError_t e = guarded_malloc(&base, off, kScratch);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return h.fail("scratch for %d tokens (%s) refused by the memory guard or the device", cap, fmt_bytes(off).c_str());
    }
    if (h.sc.base) {
        cudaStreamSynchronize(h.stream);
        guarded_free(h.sc.base, h.sc.bytes, kScratch);
    }
    char* b = (char*)base;
    Scratch& s = h.sc;
    s.base = base;
    s.bytes = off;
    s.cap_T = cap;
    s.x_stage = (float*)(b + o_x);
    s.out_stage = (float*)(b + o_out);
    s.lg_stage = (float*)(b + o_lgs);
    s.logits = (float*)(b + o_lg);
    s.w = (float*)(b + o_w);
    s.sgate = (float*)(b + o_sg);
    s.act = (float*)(b + o_act);
    s.y = (float*)(b + o_y);
    s.idx = (int32_t*)(b + o_idx);
    s.offsets = (int32_t*)(b + o_off);
    s.perm = (int32_t*)(b + o_perm);
    s.inv = (int32_t*)(b + o_inv);
    s.act_e = (int32_t*)(b + o_ae);
    s.act_off = (int32_t*)(b + o_ao);
    s.n_active = (int32_t*)(b + o_na);
    s.ep_bad = (int32_t*)(b + o_bad);
    s.tc_err = (int32_t*)(b + o_tce);
    s.dxq = dec ? (uint8_t*)(b + o_dxq) : nullptr;
    s.dact = dec ? (float*)(b + o_dact) : nullptr;
    s.dy = dec ? (float*)(b + o_dy) : nullptr;
    s.dbar = (uint32_t*)(b + o_dbar);
    s.derr = (int32_t*)(b + o_dbar + 4);
    s.dstamps = (uint64_t*)(b + o_dst);
    s.lg_part = part_rows ? (float*)(b + o_lgp) : nullptr;
    s.lg_part_rows = part_rows;
    s.dwork = b + o_dw;
    s.gemm_ws = b + o_gw;
    s.gemm_ws_bytes = gws;
    s.gemv_cap = (int)gemv_T;
    s.xq = QInput{};
    s.aq = QInput{};
    s.xq.K = h.dp;
    s.aq.K = h.act_ld;
    if (qin) {
        s.xq = qinput_at(b + o_xq, (int)gemv_T, h.dp);
        s.aq = qinput_at(b + o_aq, (int)grows, h.act_ld);
    }
    h.gb_ready = false;
    if (h.gemm_ok) {
        std::string why;
        if (!gemm_setup(s.gemm_ws, gws, h.dp, h.act_ld, (int)P, cap, max_tiles, &h.gb, &why)) return h.fail("%s", why.c_str());
        h.gb.err_host = h.err_host;
        h.gb_ready = true;
    }
    // zero the padded columns of the staging buffers once
    return h.cuda_ok(cudaMemsetAsync(base, 0, off, h.stream), "scratch clear");
}

// Router logits (+ the shared-gate column E when with_gate and the layer has a
// shared expert) for T rows of x into s.logits (row stride lg_ld): the tensor
// cores for batches of at least kRouterTcMinTokens, SIMT kernels below that.
constexpr int kRouterTcMinTokens = 16;
bool router_logits_dev(Handle& h, const float* x, int T, bool with_gate) {
    Scratch& s = h.sc;
    const bool gate = with_gate && h.has_shared;
    if (h.rtc_ok && h.rtc_enabled && T >= kRouterTcMinTokens) {
        return h.cuda_ok(launch_router_tc(h.rtc, x, T, h.router_bias, h.E, gate ? h.router_ext + (size_t)h.E * h.dp : nullptr,
                                          s.logits, h.lg_ld, s.tc_err, h.err_host, s.lg_part, s.lg_part_rows, h.n_sm,
                                          h.stream),
                         "router (tensor cores)");
    }
    return h.cuda_ok(launch_router(x, T, h.dp, h.router_ext, 0, h.E + (gate ? 1 : 0), h.router_bias, h.E, s.logits,
                                   h.lg_ld, h.stream),
                     "router");
}

// Router projection + top-k for T tokens of x (T, dp): s.idx, s.w, s.sgate.
// When logits_in is non-null it holds (T, E) caller logits on the
// device (row stride E).
bool route_stage(Handle& h, const float* x, int T, const float* logits_in, bool qx) {
    Scratch& s = h.sc;
    cudaStream_t st = h.stream;
    const int ld = h.lg_ld;
    h.mark(0);
    if (!logits_in) {
        if (!h.has_router) return h.fail("this layer has no router weights; use the ffn_block form with logits");
        if (!router_logits_dev(h, x, T, true)) return false;
    } else {
        if (!h.cuda_ok(cudaMemcpy2DAsync(s.logits, (size_t)ld * 4, logits_in, (size_t)h.E * 4, (size_t)h.E * 4, (size_t)T,
                                         cudaMemcpyDeviceToDevice, st),
                       "logits copy"))
            return false;
        if (h.has_shared &&
            !h.cuda_ok(launch_router(x, T, h.dp, h.router_ext, h.E, h.E + 1, nullptr, 0, s.logits, ld, st), "shared gate"))
            return false;
    }
    h.launches += (!logits_in || h.has_shared) ? 1 : 0;
    h.mark(1);
    // the GEMV path reads x in integer form; top-k writes it in the same pass
    QInput xq = qx ? s.xq : QInput{};
    // a single token's dispatch comes from the top-k pass (expert_stage skips the sort)
    SingleDispatch one{};
    if (T == 1 && !h.subset) {
        one.perm = s.perm;
        one.inv = s.inv;
        one.act_e = s.act_e;
        one.act_off = s.act_off;
        one.n_active = s.n_active;
        one.p_real = s.offsets + h.E;
    }
    if (!h.cuda_ok(launch_topk(s.logits, ld, T, h.E, h.k, h.norm, h.has_shared, s.idx, s.w, s.sgate, x, xq, st, one),
                   "top-k"))
        return false;
    h.launches += 1;
    if (h.subset) {
        if (!h.cuda_ok(launch_resident_remap(s.idx, T * h.k, h.slot, s.derr, h.err_host, st), "resident slots"))
            return false;
        h.launches += 1;
    }
    h.mark(2);
    return true;
}

// Dispatch -> expert products -> combine over T rows of x (f32, or f16 for
// the GEMM path) whose pairs are in s.idx / s.w. The shared expert runs on rows
// [0, Tsh). With skip_slots, buckets equal to E mark slots to leave out (their
// experts live on another rank). The GEMM path runs when x is f16 or T reaches
// the handle's threshold.
bool expert_stage(Handle& h, const void* x, bool x_f16, int T, int Tsh, bool skip_slots, void* out,
                  bool out_f16 = false, bool gemm_skip_combine = false) {
    Scratch& s = h.sc;
    cudaStream_t st = h.stream;
    const int P = T * h.k;
    const int n_buckets = skip_slots ? h.E + 1 : h.E;
    // (a single token's pairs were laid out by route_stage's top-k pass)
    if (T != 1 || skip_slots || h.subset) {
        if (!h.cuda_ok(launch_dispatch(s.idx, P, n_buckets, s.offsets, s.perm, s.inv, s.act_e, s.act_off, s.n_active,
                                       s.dwork, st, h.E),
                       "dispatch"))
            return false;
        h.launches += 4;
    }
    h.mark(3);
    const int32_t* skip_idx = skip_slots ? s.idx : nullptr;
    const bool use_gemm = h.gemm_ok && h.gb_ready && (x_f16 || T >= h.gemm_min_tokens);
    if ((x_f16 || out_f16) && !use_gemm)
        return h.fail("f16 rows need the prefill GEMM path, which this layer does not support");
    h.last_gemm = use_gemm;
    h.last_shared_rows = h.has_shared ? Tsh : 0;
    if (use_gemm) {
        PrefillArgs pa{};
        pa.gate = h.gate;
        pa.up = h.up;
        pa.down = h.down;
        pa.sg = h.sg;
        pa.su = h.su;
        pa.sd = h.sd;
        pa.x = x;
        pa.x_f16 = x_f16 ? 1 : 0;
        pa.Tsh = Tsh;
        pa.p_real = s.offsets + h.E;
        pa.perm = s.perm;
        pa.act_e = s.act_e;
        pa.act_off = s.act_off;
        pa.n_active = s.n_active;
        pa.T = T;
        pa.k = h.k;
        pa.dp = h.dp;
        pa.F = h.Fp;
        pa.Fs = h.Fsp;
        pa.has_shared = h.has_shared;
        pa.E = h.E;
        pa.act_ld = h.act_ld;
        pa.e_begin = h.e_begin;
        pa.n_sm = h.n_sm;
        if (!h.cuda_ok(launch_prefill_prep(pa, h.gb, st), "prefill gather")) return false;
        h.mark(3);
        if (!h.cuda_ok(launch_prefill_gemm(pa, h.gb, h.wmaps, true, st), "gate/up GEMM")) return false;
        h.mark(4);
        if (!h.cuda_ok(launch_prefill_gemm(pa, h.gb, h.wmaps, false, st), "down GEMM")) return false;
        h.launches += 5;  // x16, gather, tile list, two GEMMs
        h.mark(5);
        // (the caller may fuse the combine into its own kernel: expert parallel over peer memory)
        if (!gemm_skip_combine) {
            if (!h.cuda_ok(launch_combine_h(h.gb.y, s.inv, s.w, s.sgate, skip_idx, h.E, T, Tsh, h.k, h.dp, h.has_shared,
                                            out, out_f16 ? 1 : 0, st),
                           "combine"))
                return false;
            h.launches += 1;
        }
    } else {
        if (T > s.gemv_cap) return h.fail("internal: GEMV scratch covers %d tokens, call has %d", s.gemv_cap, T);
        GemvArgs a{};
        a.gate = h.gate;
        a.up = h.up;
        a.down = h.down;
        a.sg = h.sg;
        a.su = h.su;
        a.sd = h.sd;
        a.x = static_cast<const float*>(x);
        a.xq = s.xq;
        a.aq = s.aq;
        a.perm = s.perm;
        a.act_e = s.act_e;
        a.act_off = s.act_off;
        a.n_active = s.n_active;
        a.T = T;
        a.Tsh = Tsh;
        a.k = h.k;
        a.d = h.dp;
        a.F = h.Fp;
        a.Fs = h.Fsp;
        a.has_shared = h.has_shared;
        a.max_active = std::min(P, h.E);
        a.max_pairs = T;  // a token selects an expert at most once
        a.act_ld = h.act_ld;
        a.act = s.act;
        a.y = s.y;
        if (!h.cuda_ok(launch_gemv_gateup(a, st), "gate/up")) return false;
        h.mark(4);
        if (!h.cuda_ok(launch_gemv_down(a, st), "down")) return false;
        h.launches += 2 * (1 + (h.has_shared && Tsh > 0));
        h.mark(5);
        if (!h.cuda_ok(launch_combine(s.y, s.inv, s.w, s.sgate, skip_idx, h.E, T, Tsh, h.k, h.dp, h.has_shared,
                                      static_cast<float*>(out), st),
                       "combine"))
            return false;
        h.launches += 1;
    }
    h.mark(6);
    return true;
}

// Accumulates the per-stage event times of a profiled call.
bool finish_profile(Handle& h) {
    if (!h.profiling) return true;
    if (!h.cuda_ok(cudaEventSynchronize(h.sev[6]), "profile")) return false;
    if (h.last_decode) {
        // one kernel: its phases by the stamps of its first CTA (router = A, top-k and
        // dispatch = B, gate/up = C, down = D, combine = E)
        uint64_t t[6];
        if (!h.cuda_ok(cudaMemcpy(t, h.sc.dstamps, sizeof t, cudaMemcpyDeviceToHost), "profile")) return false;
        const double ph[Handle::kStages] = {(t[1] - t[0]) * 1e-6, (t[2] - t[1]) * 1e-6, 0.0,
                                            (t[3] - t[2]) * 1e-6, (t[4] - t[3]) * 1e-6, (t[5] - t[4]) * 1e-6};
        for (int i = 0; i < Handle::kStages; ++i) {
            h.stage_ms[i] += ph[i];
            h.stage_n[i] += 1;
        }
        h.last_decode = false;
    } else {
        for (int i = 0; i < Handle::kStages; ++i) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, h.sev[i], h.sev[i + 1]);
            h.stage_ms[i] += ms;
            h.stage_n[i] += 1;
        }
    }
    cudaMemcpy(&h.last_active, h.sc.n_active, 4, cudaMemcpyDeviceToHost);
    cudaMemcpy(&h.last_pairs, h.sc.offsets + h.E, 4, cudaMemcpyDeviceToHost);
    return true;
}

// The fused decode kernel over the call (calls of up to kDecodeMaxTokens tokens).
bool decode_call(Handle& h, const float* x, int T, const float* logits_in, float* out) {
    Scratch& s = h.sc;
    DecodeArgs a{};
    a.x = x;
    a.logits_in = logits_in;
    a.ld_in = h.E;
    a.router = h.router_ext;
    a.bias = h.router_bias;
    a.gate = h.gate;
    a.up = h.up;
    a.down = h.down;
    a.sg = h.sg;
    a.su = h.su;
    a.sd = h.sd;
    a.T = T;
    a.E = h.E;
    a.k = h.k;
    a.norm = h.norm;
    a.has_shared = h.has_shared;
    a.dp = h.dp;
    a.F = h.Fp;
    a.Fs = h.Fsp;
    a.act_ld = h.act_ld;
    a.logits = s.logits;
    a.lg_ld = h.lg_ld;
    a.xq = s.dxq;
    a.act = s.dact;
    a.sgate_out = s.sgate;
    a.idx_out = s.idx;
    a.w_out = s.w;
    a.n_active_out = s.n_active;
    a.p_real_out = s.offsets + h.E;
    a.y = s.dy;
    a.out = out;
    a.bar = s.dbar;
    a.err = s.derr;
    a.err_host = h.err_host;
    a.wait_ns = 1000000000ull;  // a grid barrier normally completes in microseconds
    a.stamps = h.profiling ? s.dstamps : nullptr;
    for (int i = 0; i < 4; ++i) h.mark(i);
    int grid = 0;
    if (!h.cuda_ok(launch_decode(a, h.n_sm, h.stream, &grid), "decode layer")) return false;
    h.last_decode = true;
    h.launches += 1;
    h.last_gemm = false;
    h.last_shared_rows = h.has_shared ? T : 0;
    for (int i = 4; i < 7; ++i) h.mark(i);
    return true;
}

bool decode_eligible(const Handle& h, int T, const float* logits_in) {
    return h.decode_enabled && h.sc.dxq && (logits_in || h.has_router) &&
           (!h.has_shared || h.sh_dtype == h.dtype) && h.e_begin == 0 && h.e_end == h.E &&
           decode_supported(h.dtype, T, h.E, h.k, h.dp, h.Fp, h.Fsp, h.has_shared);
}

// Core pipeline on device buffers: x (T, dp), out (T, dp).
bool run_block(Handle& h, const float* x, int T, const float* logits_in, float* out) {
    h.last_decode = false;
    if (decode_eligible(h, T, logits_in)) {
        if (!decode_call(h, x, T, logits_in, out)) return false;
        return finish_profile(h);
    }
    const bool gemv = !(h.gemm_ok && h.gb_ready && T >= h.gemm_min_tokens);
    if (!route_stage(h, x, T, logits_in, gemv && h.sc.xq.q1 != nullptr)) return false;
    if (!expert_stage(h, x, false, T, T, false, out)) return false;
    return finish_profile(h);
}

// The prefill kernels record a non-zero code when one of their bounded waits
// expired; report it (and clear it) at the next synchronisation point.
bool check_pipeline(Handle& h) {
    if (h.err_host) *reinterpret_cast<volatile int32_t*>(h.err_host) = 0;  // read below from the device flags
    if (h.sc.base) {
        int32_t code = 0;
        if (cudaMemcpy(&code, h.sc.derr, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            return h.cuda_ok(cudaGetLastError(), "error flag");
        if (code != 0) {
            cudaMemset(h.sc.dbar, 0, 12);
            if (code == kErrNotResident)
                return h.fail("the routing selected an expert this resident-subset layer does not hold (code %d); "
                              "the call's output is invalid",
                              code);
            return h.fail("decode grid barrier wait expired (code %d); the call's output is invalid", code);
        }
    }
    if (h.sc.base && h.rtc_ok) {
        int32_t code = 0;
        if (cudaMemcpy(&code, h.sc.tc_err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
            return h.cuda_ok(cudaGetLastError(), "error flag");
        if (code != 0) {
            cudaMemset(h.sc.tc_err, 0, 4);
            return h.fail("router pipeline wait expired (code %d); the call's output is invalid", code);
        }
    }
    if (!h.gb_ready) return true;
    int32_t code = 0;
    if (cudaMemcpy(&code, h.gb.err, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return h.cuda_ok(cudaGetLastError(), "error flag");
    if (code == 0) return true;
    cudaMemset(h.gb.err, 0, 4);
    return h.fail("prefill GEMM pipeline wait expired (code %d); the call's output is invalid", code);
}

// An earlier call's kernel gave up a bounded wait after that call returned (a
// device-pointer call does not synchronise): report it now, once, and refuse
// this call. The code is the kernel's (router, prefill GEMM or peer exchange).
bool take_async_error(Handle& h) {
    if (!h.err_host) return true;
    const int32_t code = *reinterpret_cast<volatile int32_t*>(h.err_host);
    if (code == 0) return true;
    *reinterpret_cast<volatile int32_t*>(h.err_host) = 0;
    if (h.peer.open && (code == kEpErrRowsWait || code == kEpErrBackWait) && !h.peer.failed) h.peer.failed = code;
    if (h.sc.base) {
        cudaMemsetAsync(h.sc.tc_err, 0, 4, h.stream);
        cudaMemsetAsync(h.sc.dbar, 0, 12, h.stream);  // barrier counter, decode error word, exit counter
    }
    if (h.gb_ready) cudaMemsetAsync(h.gb.err, 0, 4, h.stream);
    if (code == kErrNotResident)
        return h.fail("an earlier call on this handle routed to an expert this resident-subset layer does not hold "
                      "(code %d): that call's output is invalid; this call was not run",
                      code);
    return h.fail("a bounded device wait of an earlier call on this handle gave up (code %d): that call's output is "
                  "invalid; this call was not run",
                  code);
}

// Host/device wrapper: stages x and out when they are host memory or when the
// layer is padded internally.
bool block_entry(Handle& h, const float* x, int T, const float* logits, float* out) {
    if (T < 0) return h.fail("T=%d", T);
    if (!take_async_error(h)) return false;
    if (T == 0) return true;
    if (cudaSetDevice(h.device) != cudaSuccess) return h.fail("cudaSetDevice(%d) failed", h.device);
    if (!ensure_scratch(h, T)) return false;
    Scratch& s = h.sc;
    cudaStream_t st = h.stream;
    const bool x_dev = is_device_ptr(x), out_dev = is_device_ptr(out);
    const bool x_aligned = ((uintptr_t)x & 15) == 0, out_aligned = ((uintptr_t)out & 15) == 0;
    const bool lg_dev = logits ? is_device_ptr(logits) : false;
    const float* xin = x;
    if (!x_dev || h.dp != h.d || !x_aligned) {
        if (!h.cuda_ok(cudaMemcpy2DAsync(s.x_stage, (size_t)h.dp * 4, x, (size_t)h.d * 4, (size_t)h.d * 4, (size_t)T,
                                         x_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st),
                       "input copy"))
            return false;
        xin = s.x_stage;
    }
    const float* lg = logits;
    if (logits && !lg_dev) {
        if (!h.cuda_ok(cudaMemcpyAsync(s.lg_stage, logits, (size_t)T * h.E * 4, cudaMemcpyHostToDevice, st),
                       "logits upload"))
            return false;
        lg = s.lg_stage;
    }
    float* o = (out_dev && h.dp == h.d && out_aligned) ? out : s.out_stage;
    if (h.timing) cudaEventRecord(h.ev0, st);
    if (!run_block(h, xin, T, lg, o)) return false;
    if (h.timing) cudaEventRecord(h.ev1, st);
    if (o != out) {
        if (!h.cuda_ok(cudaMemcpy2DAsync(out, (size_t)h.d * 4, o, (size_t)h.dp * 4, (size_t)h.d * 4, (size_t)T,
                                         out_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st),
                       "output copy"))
            return false;
    }
    if (!out_dev || !x_dev) {
        if (!h.cuda_ok(cudaStreamSynchronize(st), "block")) return false;
        if (h.timing) cudaEventElapsedTime(&h.last_ms, h.ev0, h.ev1);
        if (!check_pipeline(h)) return false;
    }
    h.calls++;
    h.tokens += T;
    return true;
}

void copy_err(const std::string& s, char* err, int errlen) {
    if (err && errlen > 0) std::snprintf(err, (size_t)errlen, "%s", s.c_str());
}

// Device bytes a handle opened from d keeps resident (router rows, the
// tensor-core router split, the expert and shared planes, a resident subset's
// slot table), as the guard charges them; -1 for a description open refuses on
// its face. Scratch is not included (it grows with the calls).
int64_t plan_resident_bytes(const aero_cuda_moe_desc* d) {
    if (!d || d->n_embd <= 0 || d->n_expert <= 0 || d->ffn_len <= 0) return -1;
    const int dt = d->gate_exps.dtype;
    const bool f32 = dt == AERO_DT_F32;
    const int64_t E = d->n_expert, dp = f32 ? round_up(d->n_embd, 16) : d->n_embd;
    const int64_t F = d->ffn_len, Fs = d->has_shared ? (d->ffn_len_shared > 0 ? d->ffn_len_shared : F) : 0;
    int64_t ne = E;
    if (d->n_resident > 0)
        ne = d->n_resident;
    else if (d->expert_begin != 0 || d->expert_end != 0)
        ne = (int64_t)d->expert_end - d->expert_begin;
    auto fam = [&](int t, int64_t rows, int64_t cols, int64_t n) {
        const int64_t pr = t == AERO_DT_F32 ? round_up(rows, 16) : rows;
        const int64_t pc = t == AERO_DT_F32 ? round_up(cols, 16) : cols;
        return n * (align128(pr * qm_row_qs_bytes(t, (int)pc)) + align128(pr * qm_row_meta_bytes(t, (int)pc)));
    };
    int64_t b = (E + 1) * dp * 4;  // router rows + the shared gate input
    if (d->router_bias) b += E * 4;
    if (d->router && router_tc_tile_rows((int)E) > 0 && dp % 32 == 0) b += 2 * E * dp * 4;
    b += 2 * fam(dt, F, d->n_embd, ne) + fam(dt, d->n_embd, F, ne);
    if (d->has_shared) {
        const int st = d->shexp_gate.dtype;
        b += 2 * fam(st, Fs, d->n_embd, 1) + fam(st, d->n_embd, Fs, 1);
    }
    if (d->n_resident > 0 && d->n_resident < E) b += E * 4;
    return b;
}

Handle* open_desc(const aero_cuda_moe_desc* d, std::string* why) {
    if (!d) {
        *why = "null descriptor";
        return nullptr;
    }
    auto* h = new Handle();
    auto bad = [&](const std::string& m) {
        *why = m.empty() ? h->err : m;
        delete h;
        return (Handle*)nullptr;
    };
    if (d->n_embd <= 0 || d->n_expert <= 0 || d->ffn_len <= 0) return bad("n_embd, n_expert and ffn_len must be positive");
    if (d->n_expert_used <= 0 || d->n_expert_used > d->n_expert)
        return bad("n_expert_used=" + std::to_string(d->n_expert_used) + " out of range for " +
                   std::to_string(d->n_expert) + " experts");
    if (d->n_expert_used > 32 || d->n_expert > 1024)
        return bad("this implementation routes at most 32 of at most 1024 experts");
    h->device = d->device;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return bad("no CUDA device is available (this library has no CPU path)");
    }
    if (h->device < 0 || h->device >= ndev) return bad("device " + std::to_string(h->device) + " does not exist");
    cudaSetDevice(h->device);
    if (cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking) != cudaSuccess) return bad("stream creation failed");
    h->stream = h->own_stream;
    if (cudaHostAlloc(reinterpret_cast<void**>(&h->err_host), 4, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
        cudaGetLastError();
        h->err_host = nullptr;
        return bad("host-mapped error word allocation failed");
    }
    *reinterpret_cast<volatile int32_t*>(h->err_host) = 0;
    cudaEventCreate(&h->ev0);
    cudaEventCreate(&h->ev1);
    h->d = d->n_embd;
    h->E = d->n_expert;
    h->k = d->n_expert_used;
    h->F = d->ffn_len;
    h->norm = d->norm_topk_prob ? 1 : 0;
    h->has_shared = d->has_shared ? 1 : 0;
    h->Fs = h->has_shared ? (d->ffn_len_shared > 0 ? d->ffn_len_shared : d->ffn_len) : 0;
    h->e_begin = d->expert_begin;
    h->e_end = d->expert_end;
    if (h->e_begin == 0 && h->e_end == 0) h->e_end = h->E;
    if (h->e_begin < 0 || h->e_end > h->E || h->e_begin >= h->e_end) return bad("bad expert range");
    // resident subset: the expert tensors hold n_resident experts; their slots
    // are [0, n_resident) in the planes (the range bookkeeping below)
    int src_experts = h->E;
    std::vector<int32_t> slot_host;
    if (d->n_resident < 0) return bad("n_resident < 0");
    if (d->n_resident > 0) {
        if (d->expert_begin != 0 || d->expert_end != 0) return bad("a resident subset takes no expert range");
        if (!d->resident_ids) return bad("n_resident > 0 needs resident_ids");
        if (d->n_resident > h->E) return bad("n_resident > n_expert");
        slot_host.assign((size_t)h->E, -1);
        for (int i = 0; i < d->n_resident; ++i) {
            const int g = d->resident_ids[i];
            if (g < 0 || g >= h->E || (i > 0 && g <= d->resident_ids[i - 1]))
                return bad("resident_ids must be ascending, distinct ids in [0, n_expert)");
            slot_host[(size_t)g] = i;
        }
        src_experts = d->n_resident;
        h->subset = d->n_resident < h->E;  // all n_expert ids ascending: the identity map, a whole layer
        h->slot_owner.assign(d->resident_ids, d->resident_ids + d->n_resident);
        h->e_begin = 0;
        h->e_end = d->n_resident;
    }
    h->dtype = d->gate_exps.dtype;
    if (d->up_exps.dtype != h->dtype || d->down_exps.dtype != h->dtype)
        return bad("gate/up/down expert tensors must share one ggml type");
    const bool f32 = h->dtype == AERO_DT_F32;
    h->dp = f32 ? (int)round_up(h->d, 16) : h->d;
    h->Fp = f32 ? (int)round_up(h->F, 16) : h->F;
    if (h->dp % 16 || h->Fp % 16) return bad("n_embd and ffn_len must be multiples of 16");
    if (h->has_shared) {
        if (!d->shexp_gate_inp) return bad("has_shared needs shexp_gate_inp");
        h->sh_dtype = d->shexp_gate.dtype;
        if (d->shexp_up.dtype != h->sh_dtype || d->shexp_down.dtype != h->sh_dtype)
            return bad("shared gate/up/down must share one ggml type");
        if ((h->sh_dtype == AERO_DT_F32) != f32) return bad("shared expert and routed experts must both be F32 or both quantised");
        h->Fsp = f32 ? (int)round_up(h->Fs, 16) : h->Fs;
        if (h->Fsp % 16) return bad("ffn_len_shared must be a multiple of 16");
    }
    h->act_ld = (int)round_up(std::max(h->Fp, h->Fsp), 64);
    // the grouped GEMM dequantises routed and shared blocks with one type's code: a shared
    // expert of another type (allowed by the GGUF format) runs prefill on the GEMV path
    h->gemm_ok = !f32 && h->dp % 128 == 0 && h->Fp % 128 == 0 &&
                 (!h->has_shared || (h->Fsp % 128 == 0 && h->sh_dtype == h->dtype));
    if (const char* v = std::getenv("AERO_GEMM_MIN_TOKENS")) h->gemm_min_tokens = std::max(1, std::atoi(v));
    const int ne = h->e_end - h->e_begin;
    (void)ne;
    // router (+ shared gate row) as f32 (E + 1, dp)
    h->router_ext = (float*)h->dalloc((size_t)(h->E + 1) * h->dp * 4, kWeightsResident, "router");
    if (!h->router_ext) return bad("");
    if (!h->cuda_ok(cudaMemsetAsync(h->router_ext, 0, (size_t)(h->E + 1) * h->dp * 4, h->stream), "router")) return bad("");
    auto put_rows = [&](float* dst, const float* src, int rows) {
        const bool dev = is_device_ptr(src);
        return h->cuda_ok(cudaMemcpy2DAsync(dst, (size_t)h->dp * 4, src, (size_t)h->d * 4, (size_t)h->d * 4, (size_t)rows,
                                            dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, h->stream),
                          "router upload");
    };
    if (d->router) {
        h->has_router = 1;
        if (!put_rows(h->router_ext, d->router, h->E)) return bad("");
    }
    if (h->has_shared && !put_rows(h->router_ext + (size_t)h->E * h->dp, d->shexp_gate_inp, 1)) return bad("");
    if (d->router_bias) {
        h->router_bias = (float*)h->dalloc((size_t)h->E * 4, kWeightsResident, "router bias");
        if (!h->router_bias) return bad("");
        if (!h->cuda_ok(cudaMemcpyAsync(h->router_bias, d->router_bias, (size_t)h->E * 4,
                                        is_device_ptr(d->router_bias) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                                        h->stream),
                        "router bias"))
            return bad("");
    }
    h->lg_ld = (int)round_up(h->E + 1, 4);
    const bool want_rtc = h->has_router && router_tc_tile_rows(h->E) > 0 && h->dp % 32 == 0;
    // plan the whole upload before allocating (admit_plan, src/memory_guard.cpp:192-213)
    {
        size_t plan = want_rtc ? 2 * (size_t)h->E * h->dp * 4 : 0;
        auto fam = [&](int dt, int rows, int cols, int ne_) {
            const int pr = dt == AERO_DT_F32 ? (int)round_up(rows, 16) : rows;
            const int pc = dt == AERO_DT_F32 ? (int)round_up(cols, 16) : cols;
            return (size_t)ne_ * (size_t)(align128((int64_t)pr * qm_row_qs_bytes(dt, pc)) +
                                          align128((int64_t)pr * qm_row_meta_bytes(dt, pc)));
        };
        plan += 2 * fam(h->dtype, h->F, h->d, h->e_end - h->e_begin) + fam(h->dtype, h->d, h->F, h->e_end - h->e_begin);
        if (h->has_shared) plan += 2 * fam(h->sh_dtype, h->Fs, h->d, 1) + fam(h->sh_dtype, h->d, h->Fs, 1);
        char why2[256];
        if (!aero_cuda_guard_admit_plan(plan, why2, sizeof(why2))) return bad(std::string("load refused: ") + why2);
    }
    if (want_rtc) {
        float* w_hi = (float*)h->dalloc((size_t)h->E * h->dp * 4, kWeightsResident, "router split (hi)");
        float* w_lo = w_hi ? (float*)h->dalloc((size_t)h->E * h->dp * 4, kWeightsResident, "router split (lo)") : nullptr;
        if (!w_lo) return bad("");
        if (!h->cuda_ok(router_tc_prepare(h->router_ext, h->E, h->dp, w_hi, w_lo, &h->rtc, h->stream), "router split"))
            return bad("");
        h->rtc_ok = true;
    }
    if (!upload_family(*h, d->gate_exps, src_experts, h->e_begin, h->e_end, h->F, h->d, h->Fp, h->dp, h->gate,
                       "ffn_gate_exps"))
        return bad("");
    if (!upload_family(*h, d->up_exps, src_experts, h->e_begin, h->e_end, h->F, h->d, h->Fp, h->dp, h->up, "ffn_up_exps"))
        return bad("");
    if (!upload_family(*h, d->down_exps, src_experts, h->e_begin, h->e_end, h->d, h->F, h->dp, h->Fp, h->down,
                       "ffn_down_exps"))
        return bad("");
    if (h->subset) {
        h->slot = (int32_t*)h->dalloc((size_t)h->E * 4, kWeightsResident, "resident slots");
        if (!h->slot) return bad("");
        // pageable source: the copy has taken the bytes when the call returns
        if (!h->cuda_ok(cudaMemcpyAsync(h->slot, slot_host.data(), (size_t)h->E * 4, cudaMemcpyHostToDevice, h->stream),
                        "resident slots"))
            return bad("");
    }
    if (h->has_shared) {
        if (!upload_family(*h, d->shexp_gate, 1, 0, 1, h->Fs, h->d, h->Fsp, h->dp, h->sg, "ffn_gate_shexp")) return bad("");
        if (!upload_family(*h, d->shexp_up, 1, 0, 1, h->Fs, h->d, h->Fsp, h->dp, h->su, "ffn_up_shexp")) return bad("");
        if (!upload_family(*h, d->shexp_down, 1, 0, 1, h->d, h->Fs, h->dp, h->Fsp, h->sd, "ffn_down_shexp")) return bad("");
    }
    if (!h->cuda_ok(cudaStreamSynchronize(h->stream), "upload")) return bad("");
    // expert indices in the planes are local to [e_begin, e_end); the routed
    // paths below index them by global expert id, so shift the plane bases.
    if (h->gemm_ok) {
        std::string why;
        if (!gemm_weight_maps(h->gate, h->up, h->down, h->sg, h->su, h->sd, h->e_end - h->e_begin, h->has_shared,
                              &h->wmaps, &why))
            h->gemm_ok = false;  // the layer still runs, on the GEMV path
    }
    {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, h->device) == cudaSuccess) h->n_sm = prop.multiProcessorCount;
    }
    auto shift = [&](QMat& m) {
        m.qs -= (int64_t)h->e_begin * m.qs_estride;
        if (m.meta) m.meta -= (int64_t)h->e_begin * m.meta_estride;
    };
    shift(h->gate);
    shift(h->up);
    shift(h->down);
    return h;
}

}  // namespace

void set_free_error(const std::string& msg) { g_free_error = msg; }

}  // namespace aero

using aero::Handle;

extern "C" {

void* aero_cuda_moe_open(const aero_cuda_moe_desc* desc, char* err, int errlen) {
    std::string why;
    Handle* h = aero::open_desc(desc, &why);
    if (!h) aero::copy_err(why, err, errlen);
    return h;
}

void aero_cuda_moe_close(void* handle) { delete static_cast<Handle*>(handle); }

int64_t aero_cuda_moe_plan_bytes(const aero_cuda_moe_desc* desc) { return aero::plan_resident_bytes(desc); }

int aero_cuda_moe_page_in(void* handle, int slot, int expert, const void* gate, const void* up, const void* down) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (!h->subset) return h->fail("paging needs a resident-subset handle (n_resident < n_expert at open)"), -1;
    if (h->dtype != AERO_DT_Q8_0 && h->dtype != AERO_DT_Q4_K) return h->fail("paging takes Q8_0 or Q4_K experts"), -1;
    const int n_res = (int)h->slot_owner.size();
    if (slot < 0 || slot >= n_res) return h->fail("slot %d outside [0, %d)", slot, n_res), -1;
    if (expert < 0 || expert >= h->E) return h->fail("expert %d outside [0, %d)", expert, h->E), -1;
    for (int i = 0; i < n_res; ++i)
        if (h->slot_owner[(size_t)i] == expert && i != slot)
            return h->fail("expert %d is resident in slot %d already", expert, i), -1;
    if (!gate || !up || !down) return h->fail("null expert bytes"), -1;
    cudaSetDevice(h->device);
    // one expert of each family into plane slot `slot`, through a staging buffer for host bytes
    struct Fam {
        QMat* m;
        const void* src;
        int rows, cols;
    } fams[3] = {{&h->gate, gate, h->F, h->d}, {&h->up, up, h->F, h->d}, {&h->down, down, h->d, h->F}};
    const int64_t per = aero::gguf_bytes(h->dtype, (int64_t)h->F * h->d);
    void* stage = nullptr;
    if (aero::guarded_malloc(&stage, (size_t)per, aero::kScratch) != cudaSuccess) {
        cudaGetLastError();
        return h->fail("staging buffer of %lld bytes refused", (long long)per), -1;
    }
    bool ok = true;
    for (auto& f : fams) {
        const void* src = f.src;
        if (!aero::is_device_ptr(src)) {
            ok = h->cuda_ok(cudaMemcpyAsync(stage, src, (size_t)per, cudaMemcpyHostToDevice, h->stream), "expert copy");
            src = stage;
        } else if (((uintptr_t)src & 15) != 0) {
            ok = h->fail("device expert bytes must be 16-byte aligned");
        }
        // the planes' bases are unshifted (slots count from 0)
        ok = ok && h->cuda_ok(aero::launch_repack(h->dtype, static_cast<const uint8_t*>(src), f.rows, f.cols, f.rows, slot,
                                                  const_cast<uint8_t*>(f.m->qs), const_cast<uint8_t*>(f.m->meta),
                                                  f.m->qs_estride, f.m->meta_estride, h->stream),
                              "expert repack");
        ok = ok && h->cuda_ok(cudaStreamSynchronize(h->stream), "expert upload");  // staging reuse
        if (!ok) break;
    }
    aero::guarded_free(stage, (size_t)per, aero::kScratch);
    // the slot map: the previous owner leaves (also when the copy failed part way: the
    // slot then holds no expert, and a call that selects its old owner is refused)
    const int32_t none = -1, s32 = slot;
    const int old = h->slot_owner[(size_t)slot];
    if (!ok) {
        if (old >= 0) {
            cudaGetLastError();
            cudaMemcpy(h->slot + old, &none, 4, cudaMemcpyHostToDevice);
            h->slot_owner[(size_t)slot] = -1;
        }
        return -1;
    }
    if (old >= 0 && old != expert &&
        !h->cuda_ok(cudaMemcpyAsync(h->slot + old, &none, 4, cudaMemcpyHostToDevice, h->stream), "slot map"))
        return -1;
    if (!h->cuda_ok(cudaMemcpyAsync(h->slot + expert, &s32, 4, cudaMemcpyHostToDevice, h->stream), "slot map") ||
        !h->cuda_ok(cudaStreamSynchronize(h->stream), "slot map"))
        return -1;
    h->slot_owner[(size_t)slot] = expert;
    return 0;
}

int aero_cuda_moe_resident(void* handle, int32_t* slot_expert, int n) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    const int n_res = (int)h->slot_owner.size();
    if (!slot_expert || n < n_res) return n_res;
    for (int i = 0; i < n_res; ++i) slot_expert[i] = h->slot_owner[(size_t)i];
    return n_res;
}

int aero_cuda_moe_forward(void* handle, int layer, const float* h_in, int T, int n_embd, float* out) {
    (void)layer;
    auto* h = static_cast<Handle*>(handle);
    if (!h) return 0;
    std::lock_guard<std::mutex> lk(h->mu);
    if (n_embd != h->d) {
        h->fail("hidden width %d != n_embd %d", n_embd, h->d);
        return 0;
    }
    if (!h->subset && (h->e_begin != 0 || h->e_end != h->E)) {
        h->fail("this handle owns experts [%d, %d) only; use the expert-parallel entry points", h->e_begin, h->e_end);
        return 0;
    }
    return aero::block_entry(*h, h_in, T, nullptr, out) ? 1 : 0;
}

int aero_cuda_moe_wait(void* handle, int slot) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (slot < 0 || slot >= aero::kAsyncSlots) return h->fail("slot %d outside [0, %d)", slot, aero::kAsyncSlots), -1;
    auto& q = h->aslot[slot];
    if (!q.pending) return 0;
    q.pending = false;
    if (!h->cuda_ok(cudaEventSynchronize(q.copied), "asynchronous call")) return -1;
    if (!aero::take_async_error(*h)) return -1;
    h->calls++;
    h->tokens += q.T;
    return 0;
}

int aero_cuda_moe_submit(void* handle, int slot, const float* h_in, int T, float* out) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    if (slot < 0 || slot >= aero::kAsyncSlots) return h->fail("slot %d outside [0, %d)", slot, aero::kAsyncSlots), -1;
    if (h->aslot[slot].pending && aero_cuda_moe_wait(handle, slot) != 0) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (!h->subset && (h->e_begin != 0 || h->e_end != h->E))
        return h->fail("this handle owns experts [%d, %d) only", h->e_begin, h->e_end), -1;
    if (T < 0) return h->fail("T=%d", T), -1;
    if (T == 0) return 0;
    if (!h_in || !out) return h->fail("null buffer"), -1;
    if (aero::is_device_ptr(h_in) || aero::is_device_ptr(out))
        return h->fail("submit takes host buffers (device buffers: aero_cuda_moe_forward enqueues already)"), -1;
    if (!aero::take_async_error(*h)) return -1;
    if (cudaSetDevice(h->device) != cudaSuccess) return h->fail("cudaSetDevice(%d) failed", h->device), -1;
    auto& q = h->aslot[slot];
    if (!h->s_in && (cudaStreamCreateWithFlags(&h->s_in, cudaStreamNonBlocking) != cudaSuccess ||
                     cudaStreamCreateWithFlags(&h->s_out, cudaStreamNonBlocking) != cudaSuccess))
        return h->fail("copy stream creation failed"), -1;
    if (!q.in && (cudaEventCreateWithFlags(&q.in, cudaEventDisableTiming) != cudaSuccess ||
                  cudaEventCreateWithFlags(&q.done, cudaEventDisableTiming) != cudaSuccess ||
                  cudaEventCreateWithFlags(&q.copied, cudaEventDisableTiming) != cudaSuccess))
        return h->fail("event creation failed"), -1;
    if (T > q.cap) {
        const int cap = std::max(T, 2 * q.cap);
        const size_t rows = (size_t)cap * h->dp * 4;
        void* p = nullptr;
        if (aero::guarded_malloc(&p, 2 * rows, aero::kScratch) != cudaSuccess) {
            cudaGetLastError();
            return h->fail("device rows for asynchronous calls of %d tokens refused", cap), -1;
        }
        if (q.x) aero::guarded_free(q.x, q.bytes, aero::kScratch);  // the slot's earlier call has completed
        q.x = static_cast<float*>(p);
        q.out = q.x + (size_t)cap * h->dp;
        q.bytes = 2 * rows;
        q.cap = cap;
        if (h->dp != h->d && !h->cuda_ok(cudaMemsetAsync(q.x, 0, rows, h->s_in), "rows")) return -1;
    }
    if (!aero::ensure_scratch(*h, T)) return -1;
    const size_t rb = (size_t)h->d * 4, pitch = (size_t)h->dp * 4;
    // in: copy stream; block: the handle's stream after the copy; out: copy stream after the block
    if (!h->cuda_ok(cudaMemcpy2DAsync(q.x, pitch, h_in, rb, rb, (size_t)T, cudaMemcpyHostToDevice, h->s_in), "input copy") ||
        !h->cuda_ok(cudaEventRecord(q.in, h->s_in), "event") ||
        !h->cuda_ok(cudaStreamWaitEvent(h->stream, q.in, 0), "event"))
        return -1;
    if (!aero::run_block(*h, q.x, T, nullptr, q.out)) return -1;
    if (!h->cuda_ok(cudaEventRecord(q.done, h->stream), "event") ||
        !h->cuda_ok(cudaStreamWaitEvent(h->s_out, q.done, 0), "event") ||
        !h->cuda_ok(cudaMemcpy2DAsync(out, rb, q.out, pitch, rb, (size_t)T, cudaMemcpyDeviceToHost, h->s_out),
                    "output copy") ||
        !h->cuda_ok(cudaEventRecord(q.copied, h->s_out), "event"))
        return -1;
    q.T = T;
    q.pending = true;
    return 0;
}

int aero_cuda_moe_ffn_block(void* handle, const float* h_in, const float* router_logits, int T, float* out) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (!router_logits) {
        h->fail("router_logits is required");
        return -1;
    }
    if (!h->subset && (h->e_begin != 0 || h->e_end != h->E)) {
        h->fail("this handle owns experts [%d, %d) only", h->e_begin, h->e_end);
        return -1;
    }
    return aero::block_entry(*h, h_in, T, router_logits, out) ? 0 : -1;
}

int aero_cuda_moe_router_logits(void* handle, const float* x, int T, float* logits) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (!h->has_router) {
        h->fail("this layer has no router weights");
        return -1;
    }
    if (T <= 0) return T == 0 ? 0 : -1;
    cudaSetDevice(h->device);
    if (!aero::ensure_scratch(*h, T)) return -1;
    auto& s = h->sc;
    const bool xd = aero::is_device_ptr(x), ld = aero::is_device_ptr(logits);
    if (!h->cuda_ok(cudaMemcpy2DAsync(s.x_stage, (size_t)h->dp * 4, x, (size_t)h->d * 4, (size_t)h->d * 4, (size_t)T,
                                      xd ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, h->stream),
                    "input copy"))
        return -1;
    if (!aero::router_logits_dev(*h, s.x_stage, T, false)) return -1;
    if (!h->cuda_ok(cudaMemcpy2DAsync(logits, (size_t)h->E * 4, s.logits, (size_t)h->lg_ld * 4, (size_t)h->E * 4, (size_t)T,
                                      ld ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, h->stream),
                    "logits copy"))
        return -1;
    return h->cuda_ok(cudaStreamSynchronize(h->stream), "router") ? 0 : -1;
}

// Route T rows on a device, staging through guarded scratch.
static int route_impl(const float* logits, int T, int E, int k, int norm, int64_t* idx, float* w, cudaStream_t st,
                      std::string* err) {
    if (k <= 0 || k > E) {
        *err = "n_expert_used=" + std::to_string(k) + " out of range for " + std::to_string(E) + " experts";
        return -1;
    }
    if (k > 32 || E > 1024) {
        *err = "this implementation routes at most 32 of at most 1024 experts";
        return -1;
    }
    if (T <= 0) return T == 0 ? 0 : -1;
    const size_t lg_b = (size_t)T * E * 4, i_b = (size_t)T * k * 4, w_b = (size_t)T * k * 4, o_b = (size_t)T * k * 8;
    const size_t total = lg_b + i_b + w_b + o_b + 1024;
    void* base = nullptr;
    if (aero::guarded_malloc(&base, total, aero::kScratch) != cudaSuccess) {
        cudaGetLastError();
        *err = "scratch allocation refused";
        return -1;
    }
    char* b = (char*)base;
    float* dlg = (float*)b;
    int32_t* didx = (int32_t*)(b + ((lg_b + 255) & ~(size_t)255));
    float* dw = (float*)((char*)didx + ((i_b + 255) & ~(size_t)255));
    bool ok = cudaMemcpyAsync(dlg, logits, lg_b, aero::is_device_ptr(logits) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                              st) == cudaSuccess;
    ok = ok && aero::launch_topk(dlg, E, T, E, k, norm, 0, didx, dw, nullptr, nullptr, aero::QInput{}, st) == cudaSuccess;
    std::vector<int32_t> hidx((size_t)T * k);
    ok = ok && cudaMemcpyAsync(hidx.data(), didx, i_b, cudaMemcpyDeviceToHost, st) == cudaSuccess;
    const bool w_dev = aero::is_device_ptr(w);
    ok = ok && cudaMemcpyAsync(w, dw, w_b, w_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, st) == cudaSuccess;
    ok = ok && cudaStreamSynchronize(st) == cudaSuccess;
    if (ok) {
        if (aero::is_device_ptr(idx)) {
            std::vector<int64_t> tmp(hidx.begin(), hidx.end());
            ok = cudaMemcpy(idx, tmp.data(), o_b, cudaMemcpyHostToDevice) == cudaSuccess;
        } else {
            for (size_t i = 0; i < hidx.size(); ++i) idx[i] = hidx[i];
        }
    }
    if (!ok) {
        *err = std::string("route: ") + cudaGetErrorString(cudaGetLastError());
    }
    aero::guarded_free(base, total, aero::kScratch);
    return ok ? 0 : -1;
}

int aero_cuda_moe_route(void* handle, const float* logits, int T, int64_t* idx, float* w) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    cudaSetDevice(h->device);
    return route_impl(logits, T, h->E, h->k, h->norm, idx, w, h->stream, &h->err);
}

int aero_cuda_route(const float* logits, int T, int n_expert, int k, int norm, int64_t* idx, float* w) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        aero::g_free_error = "no CUDA device is available (this library has no CPU path)";
        return -1;
    }
    return route_impl(logits, T, n_expert, k, norm, idx, w, 0, &aero::g_free_error);
}

int aero_cuda_dispatch(const int64_t* idx, int T, int k, int n_expert, int32_t* offsets, int32_t* perm) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        aero::g_free_error = "no CUDA device is available (this library has no CPU path)";
        return -1;
    }
    if (T < 0 || k <= 0 || n_expert <= 0) return -1;
    const int P = T * k;
    std::vector<int32_t> h32((size_t)P);
    const bool dev_in = aero::is_device_ptr(idx);
    std::vector<int64_t> h64;
    const int64_t* src = idx;
    if (dev_in) {
        h64.resize((size_t)P);
        if (cudaMemcpy(h64.data(), idx, (size_t)P * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
        src = h64.data();
    }
    for (int p = 0; p < P; ++p) {
        if (src[p] < 0 || src[p] >= n_expert) {
            aero::g_free_error = "expert index out of range";
            return -1;
        }
        h32[(size_t)p] = (int32_t)src[p];
    }
    const size_t work = aero::dispatch_work_bytes(P, n_expert);
    const size_t total = (size_t)P * 12 + (size_t)(n_expert * 3 + 8) * 4 + work + 2048;
    void* base = nullptr;
    if (aero::guarded_malloc(&base, total, aero::kScratch) != cudaSuccess) {
        cudaGetLastError();
        aero::g_free_error = "scratch allocation refused";
        return -1;
    }
    char* b = (char*)base;
    auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
    int32_t* didx = (int32_t*)b;
    int32_t* doff = (int32_t*)(b + al((size_t)P * 4));
    int32_t* dperm = (int32_t*)((char*)doff + al((size_t)(n_expert + 1) * 4));
    int32_t* dinv = (int32_t*)((char*)dperm + al((size_t)P * 4));
    int32_t* dae = (int32_t*)((char*)dinv + al((size_t)P * 4));
    int32_t* dao = (int32_t*)((char*)dae + al((size_t)n_expert * 4));
    int32_t* dna = (int32_t*)((char*)dao + al((size_t)(n_expert + 1) * 4));
    void* dw = (char*)dna + 256;
    bool ok = cudaMemcpy(didx, h32.data(), (size_t)P * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    ok = ok && aero::launch_dispatch(didx, P, n_expert, doff, dperm, dinv, dae, dao, dna, dw, 0) == cudaSuccess;
    ok = ok && cudaMemcpy(offsets, doff, (size_t)(n_expert + 1) * 4, cudaMemcpyDefault) == cudaSuccess;
    ok = ok && (P == 0 || cudaMemcpy(perm, dperm, (size_t)P * 4, cudaMemcpyDefault) == cudaSuccess);
    if (!ok) aero::g_free_error = std::string("dispatch: ") + cudaGetErrorString(cudaGetLastError());
    aero::guarded_free(base, total, aero::kScratch);
    return ok ? 0 : -1;
}

int aero_cuda_dequant(int dtype, const uint8_t* raw, int64_t raw_len, float* out, int64_t n) {
    const int64_t bv = aero::dtype_block_values(dtype);
    if (bv <= 0 || n < 0 || n % bv) return 0;
    if (raw_len < aero::gguf_bytes(dtype, n)) return 0;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        aero::g_free_error = "no CUDA device is available (this library has no CPU path)";
        return 0;
    }
    if (n == 0) return 1;
    const size_t rb = (size_t)aero::gguf_bytes(dtype, n), ob = (size_t)n * 4;
    void* base = nullptr;
    const size_t total = ((rb + 255) & ~(size_t)255) + ob;
    if (aero::guarded_malloc(&base, total, aero::kScratch) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    uint8_t* draw = (uint8_t*)base;
    float* dout = (float*)((char*)base + ((rb + 255) & ~(size_t)255));
    bool ok = cudaMemcpy(draw, raw, rb, cudaMemcpyDefault) == cudaSuccess;
    ok = ok && aero::launch_dequant_gguf(dtype, draw, n, dout, 0) == cudaSuccess;
    ok = ok && cudaMemcpy(out, dout, ob, cudaMemcpyDefault) == cudaSuccess;
    if (!ok) cudaGetLastError();
    aero::guarded_free(base, total, aero::kScratch);
    return ok ? 1 : 0;
}

int aero_cuda_quantize(int dtype, const float* x, int64_t n, uint8_t* out, int64_t out_len) {
    if (dtype != AERO_DT_Q8_0 && dtype != AERO_DT_Q4_K) return 0;
    const int64_t bv = aero::dtype_block_values(dtype);
    if (n < 0 || n % bv || out_len < aero::gguf_bytes(dtype, n)) return 0;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        aero::g_free_error = "no CUDA device is available (this library has no CPU path)";
        return 0;
    }
    if (n == 0) return 1;
    const bool xd = aero::is_device_ptr(x), od = aero::is_device_ptr(out);
    const size_t xb = (size_t)n * 4, ob = (size_t)aero::gguf_bytes(dtype, n);
    void* base = nullptr;
    size_t total = 0;
    const float* dx = x;
    uint8_t* dout = out;
    if (!xd || !od) {
        total = (xd ? 0 : ((xb + 255) & ~(size_t)255)) + (od ? 0 : ob);
        if (aero::guarded_malloc(&base, total, aero::kScratch) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
        char* b = (char*)base;
        if (!xd) {
            dx = (const float*)b;
            b += (xb + 255) & ~(size_t)255;
        }
        if (!od) dout = (uint8_t*)b;
    }
    bool ok = xd || cudaMemcpy((void*)dx, x, xb, cudaMemcpyHostToDevice) == cudaSuccess;
    ok = ok && aero::launch_quantize(dtype, dx, n, dout, 0) == cudaSuccess;
    ok = ok && (od || cudaMemcpy(out, dout, ob, cudaMemcpyDeviceToHost) == cudaSuccess);
    ok = ok && cudaDeviceSynchronize() == cudaSuccess;
    if (!ok) cudaGetLastError();
    if (base) aero::guarded_free(base, total, aero::kScratch);
    return ok ? 1 : 0;
}

int aero_cuda_moe_set_stream(void* handle, void* stream) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    h->stream = stream ? (cudaStream_t)stream : h->own_stream;
    return 0;
}

int aero_cuda_moe_set_profiling(void* handle, int on) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    cudaSetDevice(h->device);
    if (on && !h->sev[0])
        for (auto& e : h->sev)
            if (cudaEventCreate(&e) != cudaSuccess) return -1;
    h->profiling = on != 0;
    for (int i = 0; i < Handle::kStages; ++i) {
        h->stage_ms[i] = 0.0;
        h->stage_n[i] = 0;
    }
    return 0;
}

int aero_cuda_moe_stage_times(void* handle, double* ms, int64_t* counts, int n) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    const int m = std::min(n, (int)Handle::kStages);
    for (int i = 0; i < m; ++i) {
        if (ms) ms[i] = h->stage_ms[i];
        if (counts) counts[i] = h->stage_n[i];
    }
    return m;
}

int aero_cuda_moe_set_option(void* handle, int option, int64_t value) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (option == AERO_CUDA_OPT_GEMM_MIN_TOKENS) {
        if (value < 1) return -1;
        h->gemm_min_tokens = (int)std::min<int64_t>(value, 1 << 30);
        h->sc.cap_T = 0;  // re-plan scratch on the next call
        return 0;
    }
    if (option == AERO_CUDA_OPT_ROUTER_TC) {
        if (value != 0 && value != 1) return -1;
        h->rtc_enabled = value != 0;
        return 0;
    }
    if (option == AERO_CUDA_OPT_DECODE_FUSED) {
        if (value != 0 && value != 1) return -1;
        h->decode_enabled = value != 0;
        return 0;
    }
    if (option == AERO_CUDA_OPT_PEER_WAIT_MS) {
        if (value < 1 || value > 600000) return h->fail("peer wait limit %lld ms outside [1, 600000]", (long long)value), -1;
        h->peer_wait_ns = (uint64_t)value * 1000000ull;
        h->peer.tab.wait_ns = h->peer_wait_ns;  // applies to the next step of an open exchange
        return 0;
    }
    h->fail("unknown option %d", option);
    return -1;
}

int aero_cuda_moe_status(void* handle) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    cudaSetDevice(h->device);
    if (!h->cuda_ok(cudaStreamSynchronize(h->stream), "status")) return -1;
    int32_t code = h->err_host ? *reinterpret_cast<volatile int32_t*>(h->err_host) : 0;
    int32_t dev[4] = {0, 0, 0, 0};
    if (h->sc.base) cudaMemcpy(&dev[3], h->sc.derr, 4, cudaMemcpyDeviceToHost);
    if (h->sc.base && h->rtc_ok) cudaMemcpy(&dev[0], h->sc.tc_err, 4, cudaMemcpyDeviceToHost);
    if (h->gb_ready) cudaMemcpy(&dev[1], h->gb.err, 4, cudaMemcpyDeviceToHost);
    if (h->peer.open) cudaMemcpy(&dev[2], h->peer.window + h->peer.tab.off_err, 4, cudaMemcpyDeviceToHost);
    for (int32_t v : dev)
        if (code == 0) code = v;
    if (dev[2] != 0 && !h->peer.failed) h->peer.failed = dev[2];
    // the pipeline codes are cleared; a peer exchange's code stays (its waits return at once from then on)
    if (h->err_host) *reinterpret_cast<volatile int32_t*>(h->err_host) = 0;
    if (h->sc.base && h->rtc_ok) cudaMemset(h->sc.tc_err, 0, 4);
    if (h->gb_ready) cudaMemset(h->gb.err, 0, 4);
    if (dev[3] != 0) {
        cudaMemset(h->sc.dbar, 0, 12);
    }
    if (!h->cuda_ok(cudaGetLastError(), "status")) return -1;
    return code;
}

int aero_cuda_moe_info(void* handle, int32_t* out8) {
    auto* h = static_cast<Handle*>(handle);
    if (!h || !out8) return -1;
    const int32_t v[8] = {h->d, h->E, h->k, h->F, h->Fs, h->has_shared, h->dtype, h->norm};
    std::memcpy(out8, v, sizeof(v));
    return 0;
}

// ------------------------------------------------------------ expert parallel
// The exchange itself (NCCL all-to-all) belongs to the caller; these three
// calls are the device work on either side of it. All pointers are device
// pointers; the work is enqueued on the handle's stream and the calls return
// without synchronising.

int aero_cuda_ep_meta_ld(void* handle) {
    auto* h = static_cast<Handle*>(handle);
    return h ? 2 * h->k + 2 : -1;
}

static bool ep_rank_table(Handle& h, int n_ranks, int rank, const int32_t* begin, aero::EpRankTable* rt) {
    if (h.subset) return h.fail("a resident-subset handle takes no expert-parallel entry points");
    if (n_ranks < 1 || n_ranks > aero::kEpMaxRanks) return h.fail("n_ranks=%d outside [1, %d]", n_ranks, aero::kEpMaxRanks);
    if (rank < 0 || rank >= n_ranks) return h.fail("rank %d outside [0, %d)", rank, n_ranks);
    if (!begin) return h.fail("rank_expert_begin is required");
    if (begin[0] != 0 || begin[n_ranks] != h.E) return h.fail("rank_expert_begin must run from 0 to %d", h.E);
    for (int r = 0; r < n_ranks; ++r)
        if (begin[r + 1] < begin[r]) return h.fail("rank_expert_begin is not ascending at rank %d", r);
    if (begin[rank] != h.e_begin || begin[rank + 1] != h.e_end)
        return h.fail("rank %d owns [%d, %d) in the table but this handle holds [%d, %d)", rank, begin[rank],
                      begin[rank + 1], h.e_begin, h.e_end);
    rt->n = n_ranks;
    for (int r = 0; r <= n_ranks; ++r) rt->begin[r] = begin[r];
    return true;
}

int aero_cuda_ep_dispatch(void* handle, const float* x, int T, int n_ranks, int rank, const int32_t* rank_expert_begin,
                          int row_dtype, void* self_rows, int32_t* self_meta, void* send_rows, int32_t* send_meta,
                          int slab_rows, int32_t* counts, int32_t* pos) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    aero::EpRankTable rt{};
    if (!ep_rank_table(*h, n_ranks, rank, rank_expert_begin, &rt)) return -1;
    if (T < 0) return h->fail("T=%d", T), -1;
    if (row_dtype != AERO_EP_ROWS_F32 && row_dtype != AERO_EP_ROWS_F16) return h->fail("row_dtype %d", row_dtype), -1;
    if (h->d != h->dp) return h->fail("expert parallel needs n_embd %% 128 == 0 (n_embd=%d)", h->d), -1;
    if (slab_rows < std::max(T, 1)) return h->fail("slab_rows %d < T = %d", slab_rows, T), -1;
    if (!counts || !pos || !send_rows || !send_meta || (T > 0 && (!x || !self_rows || !self_meta)))
        return h->fail("null buffer"), -1;
    for (const void* p : {(const void*)x, (const void*)self_rows, (const void*)send_rows})
        if (p && (!aero::is_device_ptr(p) || ((uintptr_t)p & 15) != 0))
            return h->fail("row buffers must be 16-byte aligned device memory"), -1;
    cudaSetDevice(h->device);
    if (!aero::ensure_scratch(*h, std::max(T, 1))) return -1;
    auto& s = h->sc;
    if (T > 0 && !aero::route_stage(*h, x, T, nullptr, false)) return -1;
    // the plan reuses the dispatch buffers: perm holds send_tok, inv send_rank
    if (!h->cuda_ok(aero::launch_ep_plan(s.idx, T, h->k, rt, rank, slab_rows, s.perm, s.inv, counts, pos, h->stream),
                    "exchange plan"))
        return -1;
    if (!h->cuda_ok(aero::launch_ep_pack(x, T, h->dp, h->k, s.idx, s.w, s.sgate, h->has_shared, rt, rank, slab_rows,
                                         s.perm, counts, row_dtype == AERO_EP_ROWS_F16, self_rows, self_meta, send_rows,
                                         send_meta, 2 * h->k + 2, h->n_sm, h->stream),
                    "exchange pack"))
        return -1;
    h->launches += 2;
    return 0;
}

int aero_cuda_ep_expert_block(void* handle, const void* rows, int row_dtype, const int32_t* meta, int R, int n_shared,
                              void* out, int out_dtype) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (h->subset) return h->fail("a resident-subset handle takes no expert-parallel entry points"), -1;
    if (R < 0 || n_shared < 0 || n_shared > R) return h->fail("R=%d n_shared=%d", R, n_shared), -1;
    if (row_dtype != AERO_EP_ROWS_F32 && row_dtype != AERO_EP_ROWS_F16) return h->fail("row_dtype %d", row_dtype), -1;
    if (out_dtype != AERO_EP_ROWS_F32 && out_dtype != AERO_EP_ROWS_F16) return h->fail("out_dtype %d", out_dtype), -1;
    if (h->d != h->dp) return h->fail("expert parallel needs n_embd %% 128 == 0 (n_embd=%d)", h->d), -1;
    if (R == 0) return 0;
    if (!rows || !meta || !out) return h->fail("null buffer"), -1;
    for (const void* p : {(const void*)rows, (const void*)out})
        if (!aero::is_device_ptr(p) || ((uintptr_t)p & 15) != 0)
            return h->fail("rows and out must be 16-byte aligned device memory"), -1;
    cudaSetDevice(h->device);
    if (!aero::ensure_scratch(*h, R)) return -1;
    auto& s = h->sc;
    const bool f16 = row_dtype == AERO_EP_ROWS_F16;
    h->mark(0);
    h->mark(1);
    if (!h->cuda_ok(aero::launch_ep_prep(meta, 2 * h->k + 2, R, h->k, n_shared, h->e_begin, h->e_end, h->E, s.idx, s.w,
                                         s.sgate, s.ep_bad, h->stream),
                    "exchange unpack"))
        return -1;
    h->launches += 1;
    const bool gemv = !f16 && !(h->gemm_ok && h->gb_ready && R >= h->gemm_min_tokens);
    if (gemv && s.xq.q1) {
        if (!h->cuda_ok(aero::launch_qinput(static_cast<const float*>(rows), R, h->dp, s.xq, h->stream), "row codes"))
            return -1;
        h->launches += 1;
    }
    h->mark(2);
    if (!aero::expert_stage(*h, rows, f16, R, n_shared, true, out, out_dtype == AERO_EP_ROWS_F16)) return -1;
    return aero::finish_profile(*h) ? 0 : -1;
}

int aero_cuda_ep_combine(void* handle, const void* self_out, const void* back, int parts_dtype, const int32_t* pos, int T,
                         int n_ranks, int rank, float* out) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (n_ranks < 1 || n_ranks > aero::kEpMaxRanks || rank < 0 || rank >= n_ranks)
        return h->fail("n_ranks=%d rank=%d", n_ranks, rank), -1;
    if (T < 0) return h->fail("T=%d", T), -1;
    if (parts_dtype != AERO_EP_ROWS_F32 && parts_dtype != AERO_EP_ROWS_F16)
        return h->fail("parts_dtype %d", parts_dtype), -1;
    if (T == 0) return 0;
    if (!self_out || !pos || !out || (n_ranks > 1 && !back)) return h->fail("null buffer"), -1;
    cudaSetDevice(h->device);
    if (!h->cuda_ok(aero::launch_ep_combine(self_out, back, parts_dtype == AERO_EP_ROWS_F16, pos, T, n_ranks, rank, h->dp,
                                            out, h->stream),
                    "exchange combine"))
        return -1;
    h->launches += 1;
    return 0;
}

// Number of metadata ids that named an expert this rank does not own, since
// the last call (reading it synchronises the handle's stream).
int aero_cuda_ep_bad_ids(void* handle) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (!h->sc.base) return 0;
    int32_t v = 0;
    if (!h->cuda_ok(cudaMemcpyAsync(&v, h->sc.ep_bad, 4, cudaMemcpyDeviceToHost, h->stream), "bad-id count") ||
        !h->cuda_ok(cudaStreamSynchronize(h->stream), "bad-id count"))
        return -1;
    if (v) cudaMemsetAsync(h->sc.ep_bad, 0, 4, h->stream);
    return v;
}

// ------------------------------------------------ expert parallel, peer memory

// The window layout a rank opened, carried in its IPC blob after the handle and
// the GPU UUID; connect compares every rank's with its own.
struct PeerLayout {
    uint32_t magic, n_ranks, slab_rows, row_dtype, dp, k, n_expert, reserved;
    uint64_t window_bytes, table_hash;
};
constexpr size_t kBlobLayoutOff = sizeof(cudaIpcMemHandle_t) + sizeof(cudaUUID_t);
constexpr uint32_t kPeerLayoutMagic = 0x41455031u;  // "AEP1"

static PeerLayout peer_layout_of(int n, int slab, int row_dtype, int dp, int k, int E, size_t wbytes,
                                 const aero::EpRankTable& rt) {
    PeerLayout l{};
    l.magic = kPeerLayoutMagic;
    l.n_ranks = (uint32_t)n;
    l.slab_rows = (uint32_t)slab;
    l.row_dtype = (uint32_t)row_dtype;
    l.dp = (uint32_t)dp;
    l.k = (uint32_t)k;
    l.n_expert = (uint32_t)E;
    l.window_bytes = wbytes;
    uint64_t hsh = 1469598103934665603ull;  // FNV-1a over the expert table
    for (int r = 0; r <= rt.n; ++r) {
        hsh ^= (uint64_t)(uint32_t)rt.begin[r];
        hsh *= 1099511628211ull;
    }
    l.table_hash = hsh;
    return l;
}

static bool peer_layout_equal(const PeerLayout& a, const PeerLayout& b, std::string* why) {
    char buf[160];
    auto diff = [&](const char* what, unsigned long long x, unsigned long long y) {
        std::snprintf(buf, sizeof buf, "%s %llu here, %llu there", what, x, y);
        *why = buf;
        return false;
    };
    if (b.magic != kPeerLayoutMagic) return diff("layout tag", a.magic, b.magic);
    if (a.n_ranks != b.n_ranks) return diff("n_ranks", a.n_ranks, b.n_ranks);
    if (a.slab_rows != b.slab_rows) return diff("slab_rows", a.slab_rows, b.slab_rows);
    if (a.row_dtype != b.row_dtype) return diff("row type", a.row_dtype, b.row_dtype);
    if (a.dp != b.dp) return diff("row width", a.dp, b.dp);
    if (a.k != b.k) return diff("k", a.k, b.k);
    if (a.n_expert != b.n_expert) return diff("n_expert", a.n_expert, b.n_expert);
    if (a.window_bytes != b.window_bytes) return diff("window bytes", a.window_bytes, b.window_bytes);
    if (a.table_hash != b.table_hash) return diff("expert table hash", a.table_hash, b.table_hash);
    return true;
}

int aero_cuda_ep_peer_open(void* handle, int n_ranks, int rank, const int32_t* rank_expert_begin, int slab_rows,
                           int row_dtype, void* ipc_out) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    auto& pc = h->peer;
    if (pc.open) return h->fail("the peer exchange is already open on this handle"), -1;
    aero::EpRankTable rt{};
    if (!ep_rank_table(*h, n_ranks, rank, rank_expert_begin, &rt)) return -1;
    if (n_ranks < 2 || n_ranks > 32) return h->fail("the peer exchange runs on 2 to 32 ranks (%d)", n_ranks), -1;
    if (row_dtype != AERO_EP_ROWS_F32 && row_dtype != AERO_EP_ROWS_F16) return h->fail("row_dtype %d", row_dtype), -1;
    if (h->d != h->dp) return h->fail("expert parallel needs n_embd %% 128 == 0 (n_embd=%d)", h->d), -1;
    if (slab_rows < 1) return h->fail("slab_rows %d", slab_rows), -1;
    if (h->dp % 256 || h->dp > 2048)
        return h->fail("the peer exchange moves rows of up to 2048 values in 256-value chunks (n_embd=%d)", h->d), -1;
    if ((int64_t)n_ranks * slab_rows > (1 << 24)) return h->fail("n_ranks * slab_rows too large"), -1;
    if (!ipc_out) return h->fail("null ipc_out"), -1;
    cudaSetDevice(h->device);
    const int R = n_ranks * slab_rows;
    if (!aero::ensure_scratch(*h, R)) return -1;
    if (row_dtype == AERO_EP_ROWS_F16 && !(h->gemm_ok && h->gb_ready))
        return h->fail("f16 rows need the prefill GEMM path, which this layer does not support"), -1;
    size_t wbytes = 0;
    aero::EpPeerTable tab = aero::ep_peer_layout(n_ranks, rank, slab_rows, h->dp, h->k,
                                                 row_dtype == AERO_EP_ROWS_F16, &wbytes);
    const size_t esz = row_dtype == AERO_EP_ROWS_F16 ? 2 : 4;
    const size_t ybytes = (size_t)R * h->dp * esz;
    const size_t abytes = ((size_t)n_ranks + n_ranks + 1 + (size_t)slab_rows * n_ranks + n_ranks) * 4;
    void *w = nullptr, *y = nullptr, *a = nullptr;
    cudaError_t e = aero::guarded_malloc(&w, wbytes, aero::kScratch);
    if (e == cudaSuccess) e = aero::guarded_malloc(&y, ybytes, aero::kScratch);
    if (e == cudaSuccess) e = aero::guarded_malloc(&a, abytes, aero::kScratch);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (w) aero::guarded_free(w, wbytes, aero::kScratch);
        if (y) aero::guarded_free(y, ybytes, aero::kScratch);
        return h->fail("peer exchange buffers (%s) refused by the memory guard or the device",
                       aero::fmt_bytes(wbytes + ybytes + abytes).c_str()),
               -1;
    }
    pc.window = static_cast<char*>(w);
    pc.window_bytes = wbytes;
    pc.y = y;
    pc.y_bytes = ybytes;
    pc.aux = static_cast<int32_t*>(a);
    pc.aux_bytes = abytes;
    pc.open = true;
    pc.rt = rt;
    tab.base[rank] = pc.window;
    tab.wait_ns = h->peer_wait_ns;
    tab.err_host = h->err_host;
    pc.tab = tab;
    cudaIpcMemHandle_t ih;
    if (!h->cuda_ok(cudaMemsetAsync(pc.window, 0, wbytes, h->stream), "window clear") ||
        !h->cuda_ok(cudaMemsetAsync(pc.aux, 0, abytes, h->stream), "window clear") ||
        !h->cuda_ok(cudaStreamSynchronize(h->stream), "window clear") ||
        !h->cuda_ok(cudaIpcGetMemHandle(&ih, pc.window), "IPC handle of the window")) {
        h->peer_release();
        return -1;
    }
    // the blob: the window's IPC handle, this GPU's UUID (ranks on one GPU are
    // refused at connect), then the window layout every rank must share
    static_assert(kBlobLayoutOff + sizeof(PeerLayout) <= AERO_EP_IPC_BYTES, "IPC blob size");
    cudaDeviceProp prop{};
    if (!h->cuda_ok(cudaGetDeviceProperties(&prop, h->device), "device properties")) {
        h->peer_release();
        return -1;
    }
    const PeerLayout lay = peer_layout_of(n_ranks, slab_rows, row_dtype, h->dp, h->k, h->E, wbytes, rt);
    std::memset(ipc_out, 0, AERO_EP_IPC_BYTES);
    std::memcpy(ipc_out, &ih, sizeof ih);
    std::memcpy(static_cast<char*>(ipc_out) + sizeof ih, &prop.uuid, sizeof prop.uuid);
    std::memcpy(static_cast<char*>(ipc_out) + kBlobLayoutOff, &lay, sizeof lay);
    return 0;
}

int aero_cuda_ep_peer_connect(void* handle, const void* ipc_all) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    auto& pc = h->peer;
    if (!pc.open) return h->fail("aero_cuda_ep_peer_open first"), -1;
    if (pc.connected) return h->fail("the peer exchange is already connected"), -1;
    if (!ipc_all) return h->fail("null ipc_all"), -1;
    cudaSetDevice(h->device);
    const int n = pc.tab.n;
    const char* blobs = static_cast<const char*>(ipc_all);
    // every rank must have opened the same window layout: a rank whose slabs or
    // rows were larger would store past the end of its peers' windows
    PeerLayout mine;
    std::memcpy(&mine, blobs + (size_t)pc.tab.me * AERO_EP_IPC_BYTES + kBlobLayoutOff, sizeof mine);
    for (int r = 0; r < n; ++r) {
        PeerLayout o;
        std::memcpy(&o, blobs + (size_t)r * AERO_EP_IPC_BYTES + kBlobLayoutOff, sizeof o);
        std::string why;
        if (!peer_layout_equal(mine, o, &why))
            return h->fail("rank %d opened a different exchange window layout (%s); every rank must pass the same "
                           "n_ranks, slab_rows (max_tokens), row type, expert table and layer shape",
                           r, why.c_str()),
                   -1;
    }
    // ranks on one GPU would run kernels that wait on each other side by side
    const char* my_uuid = blobs + (size_t)pc.tab.me * AERO_EP_IPC_BYTES + sizeof(cudaIpcMemHandle_t);
    for (int r = 0; r < n; ++r)
        if (r != pc.tab.me &&
            std::memcmp(blobs + (size_t)r * AERO_EP_IPC_BYTES + sizeof(cudaIpcMemHandle_t), my_uuid,
                        sizeof(cudaUUID_t)) == 0)
            return h->fail("rank %d runs on this rank's GPU %d: the peer exchange needs one GPU per rank", r, h->device),
                   -1;
    pc.mapped.assign(n, nullptr);
    for (int r = 0; r < n; ++r) {
        if (r == pc.tab.me) continue;
        cudaIpcMemHandle_t ih;
        std::memcpy(&ih, blobs + (size_t)r * AERO_EP_IPC_BYTES, sizeof ih);
        void* p = nullptr;
        if (!h->cuda_ok(cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess), "opening a peer's window"))
            return h->fail("rank %d's window: %s", r, h->err.c_str()), -1;
        pc.mapped[r] = static_cast<char*>(p);
        pc.tab.base[r] = static_cast<char*>(p);
    }
    pc.connected = true;
    return 0;
}

int aero_cuda_ep_peer_step(void* handle, const float* x, int T, float* out) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    auto& pc = h->peer;
    if (!pc.connected) return h->fail("the peer exchange is not connected"), -1;
    const auto& tab = pc.tab;
    if (T < 0 || T > tab.slab) return h->fail("T=%d outside [0, slab_rows=%d]", T, tab.slab), -1;
    if (!aero::take_async_error(*h)) return -1;
    if (pc.failed)
        return h->fail("a wait of this peer exchange gave up earlier (code %d); close and reopen the exchange",
                       pc.failed),
               -1;
    if (T > 0) {
        if (!x || !out) return h->fail("null buffer"), -1;
        for (const void* p : {(const void*)x, (const void*)out})
            if (!aero::is_device_ptr(p) || ((uintptr_t)p & 15) != 0)
                return h->fail("x and out must be 16-byte aligned device memory"), -1;
    }
    cudaSetDevice(h->device);
    auto& s = h->sc;
    const int n = tab.n, me = tab.me, R = n * tab.slab;
    const bool f16 = tab.rows_f16 != 0;
    int32_t* slot_ctr = pc.aux;
    int32_t* counts = pc.aux + n;
    int32_t* pos = counts + n + 1;
    int32_t* received = pos + (size_t)tab.slab * n;
    const uint32_t epoch = ++pc.epoch;
    cudaStream_t st = h->stream;
    auto mark = [&](int i) {
        if (pc.prof) cudaEventRecord(pc.ev[i], st);
    };
    bool ok = true;
    mark(0);
    if (T > 0) {
        ok = aero::route_stage(*h, x, T, nullptr, false);
    } else {
        for (int i = 0; i < 3; ++i) h->mark(i);
    }
    mark(1);
    mark(2);  // (the plan is part of the pack: one phase is empty)
    ok = ok && h->cuda_ok(aero::launch_ep_peer_pack(tab, x, T, s.idx, s.w, s.sgate, h->has_shared, pc.rt, slot_ctr,
                                                    counts, pos, epoch, h->n_sm, st),
                          "exchange pack");
    mark(3);
    ok = ok && h->cuda_ok(aero::launch_ep_peer_prep(tab, T, h->e_begin, h->e_end, h->E, epoch, s.idx, s.w, s.sgate,
                                                    s.ep_bad, h->n_sm, st),
                          "exchange unpack");
    const void* rows = tab.base[me] + tab.off_rows;
    const bool gemv = !f16 && !(h->gemm_ok && h->gb_ready && R >= h->gemm_min_tokens);
    if (ok && gemv && s.xq.q1)
        ok = h->cuda_ok(aero::launch_qinput(static_cast<const float*>(rows), R, h->dp, s.xq, st), "row codes");
    mark(4);
    // GEMM path: its combine is fused with the return (rows written straight to their owners)
    const bool fused = h->gemm_ok && h->gb_ready && (f16 || R >= h->gemm_min_tokens);
    ok = ok && aero::expert_stage(*h, rows, f16, R, T, true, pc.y, f16, fused);
    mark(5);
    if (fused)
        ok = ok && h->cuda_ok(aero::launch_ep_peer_combine_return(tab, h->gb.y, s.inv, s.w, s.sgate, s.idx, h->E, T,
                                                                  h->has_shared, pc.y, epoch, received, h->n_sm, st),
                              "exchange combine + return");
    else
        ok = ok && h->cuda_ok(aero::launch_ep_peer_return(tab, pc.y, epoch, received, h->n_sm, st), "exchange return");
    mark(6);
    ok = ok && h->cuda_ok(aero::launch_ep_peer_combine(tab, pc.y, pos, T, epoch, out, h->n_sm, st), "exchange combine");
    mark(7);
    h->launches += 5 + (gemv ? 1 : 0);
    if (!ok) return -1;
    if (h->profiling && !aero::finish_profile(*h)) return -1;
    if (pc.prof) {
        if (!h->cuda_ok(cudaEventSynchronize(pc.ev[aero::PeerCtx::kPhases]), "profile")) return -1;
        for (int i = 0; i < aero::PeerCtx::kPhases; ++i) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, pc.ev[i], pc.ev[i + 1]);
            pc.ms[i] += ms;
        }
        pc.n_prof += 1;
    }
    h->calls += 1;
    h->tokens += T;
    return 0;
}

// 0: every wait of the steps so far completed; otherwise the code of the first
// that gave up (21: rows, 22: returns). Synchronises the handle's stream.
int aero_cuda_ep_peer_status(void* handle) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    auto& pc = h->peer;
    if (!pc.open) return h->fail("the peer exchange is not open"), -1;
    cudaSetDevice(h->device);
    int32_t v = 0;
    if (!h->cuda_ok(cudaMemcpyAsync(&v, pc.window + pc.tab.off_err, 4, cudaMemcpyDeviceToHost, h->stream), "status") ||
        !h->cuda_ok(cudaStreamSynchronize(h->stream), "status"))
        return -1;
    if (v != 0 && !pc.failed) pc.failed = v;
    return v;
}

int aero_cuda_ep_peer_counts(void* handle, int32_t* sent, int32_t* received) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    auto& pc = h->peer;
    if (!pc.connected) return h->fail("the peer exchange is not connected"), -1;
    cudaSetDevice(h->device);
    const int n = pc.tab.n, me = pc.tab.me;
    std::vector<int32_t> c(n + 1), w(n);
    // (the window's own counts may already hold a peer's next step: read the step's copy)
    const int32_t* step_recv = pc.aux + n + n + 1 + (size_t)pc.tab.slab * n;
    if (!h->cuda_ok(cudaMemcpyAsync(c.data(), pc.aux + n, (size_t)n * 4, cudaMemcpyDeviceToHost, h->stream), "counts") ||
        !h->cuda_ok(cudaMemcpyAsync(w.data(), step_recv, (size_t)n * 4, cudaMemcpyDeviceToHost, h->stream), "counts") ||
        !h->cuda_ok(cudaStreamSynchronize(h->stream), "counts"))
        return -1;
    for (int r = 0; r < n; ++r) {
        if (sent) sent[r] = r == me ? 0 : c[r];
        if (received) received[r] = r == me ? 0 : w[(r - me + n) % n];
    }
    return 0;
}

// on != 0: time the phases of every step (synchronises each step); ms (7
// doubles, may be null) receives the mean per phase since the last read:
// route, plan, pack, rows wait + unpack, experts, return, combine. Returns the
// number of steps averaged.
int aero_cuda_ep_peer_profile(void* handle, int on, double* ms) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    auto& pc = h->peer;
    if (!pc.open) return h->fail("the peer exchange is not open"), -1;
    cudaSetDevice(h->device);
    const long n = pc.n_prof;
    for (int i = 0; i < aero::PeerCtx::kPhases; ++i) {
        if (ms) ms[i] = n ? pc.ms[i] / n : 0.0;
        pc.ms[i] = 0.0;
    }
    pc.n_prof = 0;
    if (on && !pc.ev[0])
        for (auto& e : pc.ev)
            if (!h->cuda_ok(cudaEventCreate(&e), "profile events")) return -1;
    pc.prof = on != 0;
    return (int)n;
}

int aero_cuda_ep_peer_close(void* handle) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    std::lock_guard<std::mutex> lk(h->mu);
    if (!h->peer.open) return 0;
    cudaSetDevice(h->device);
    cudaStreamSynchronize(h->stream);
    h->peer_release();
    return 0;
}

const char* aero_cuda_moe_last_error(void* handle) {
    if (!handle) return aero::g_free_error.c_str();
    return static_cast<Handle*>(handle)->err.c_str();
}

int aero_cuda_moe_stats(void* handle, char* buf, int len) {
    auto* h = static_cast<Handle*>(handle);
    if (!h) return -1;
    size_t wbytes = 0;
    for (auto& a : h->allocs) wbytes += a.bytes;
    const int n = std::snprintf(buf, (size_t)std::max(0, len),
                                "{\"calls\": %ld, \"tokens\": %ld, \"launches\": %ld, \"weight_bytes\": %zu, "
                                "\"scratch_bytes\": %zu, \"scratch_tokens\": %d, \"guard_committed\": %zu, "
                                "\"last_active\": %d, \"last_pairs\": %d, \"last_shared_rows\": %d, "
                                "\"last_gemm\": %d, \"last_ms\": %.6f}",
                                h->calls, h->tokens, h->launches, wbytes, h->sc.bytes, h->sc.cap_T,
                                aero_cuda_guard_committed(-1), h->last_active, h->last_pairs, h->last_shared_rows,
                                h->last_gemm ? 1 : 0, (double)h->last_ms);
    return n;
}

int aero_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

}  // extern "C"
