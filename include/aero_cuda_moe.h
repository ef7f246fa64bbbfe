/*
 * aero_cuda_moe — B200 (sm_100a) mixture-of-experts FFN library, plain C ABI.
 *
 * Drop-in replacement for the MoE FFN path of the Aero engine. The reference
 * interfaces each entry point replaces are cited beside it (paths within the
 * Aero project). Conventions kept from the reference:
 *   - caller-owned, contiguous, row-major f32 buffers (include/aero/moe.hpp:43-52);
 *   - aero_moe_* style calls return 0 on success and -1 on refusal
 *     (include/aero/moe.hpp:17-18); the block hook returns non-zero on success
 *     (src/model.cpp:169); dequant returns 1 on success (src/kernels.cpp:591);
 *   - ggml type ids: 0 F32, 1 F16, 8 Q8_0, 12 Q4_K (engine/native.py:23-30).
 * Pointers to activations may be host or device memory; the library checks with
 * cudaPointerGetAttributes. With host pointers a call returns when the result is
 * in the caller's buffer. With device pointers a call is ordered on the handle's
 * stream and returns once the work is enqueued.
 * There is no CPU fallback: every compute call runs on the GPU or is refused.
 */
#ifndef AERO_CUDA_MOE_H
#define AERO_CUDA_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AERO_CUDA_DTYPE_F32 0
#define AERO_CUDA_DTYPE_F16 1
#define AERO_CUDA_DTYPE_Q8_0 8
#define AERO_CUDA_DTYPE_Q4_K 12

/* One tensor given as GGUF bytes (host or device memory). */
typedef struct aero_cuda_tensor {
    int32_t dtype;
    int32_t reserved;
    const void* data;
    int64_t nbytes;
} aero_cuda_tensor;

/* Layer description for aero_cuda_moe_open. Shapes are row-major (out, in):
 * gate/up (n_expert, ffn_len, n_embd), down (n_expert, n_embd, ffn_len),
 * router (n_expert, n_embd) f32, shexp gate/up (ffn_len_shared, n_embd),
 * shexp down (n_embd, ffn_len_shared), shexp_gate_inp (n_embd,) f32.
 * Mirrors the tensors engine/moe.py:5-12 lists and MoeConfig
 * (engine/moe.py:46-57). */
typedef struct aero_cuda_moe_desc {
    int32_t n_embd, n_expert, n_expert_used, ffn_len;
    int32_t norm_topk_prob, has_shared, ffn_len_shared, device;
    /* Expert-parallel ownership: this handle uploads and computes experts
     * [expert_begin, expert_end); 0,0 means all. Routing is over all experts. */
    int32_t expert_begin, expert_end;
    /* Resident subset: when n_resident > 0 the expert tensors hold only
     * n_resident experts, those with the global ids resident_ids[0..n_resident)
     * (ascending, distinct, < n_expert), in that order. Routing stays over all
     * n_expert logits (same selection and weights as the whole layer); a call
     * whose routing selects an expert that is not resident fails with status
     * code 41 and its output is invalid. Not combined with an expert range nor
     * with the expert-parallel entry points. 0: the tensors hold all experts. */
    int32_t n_resident;
    int32_t reserved[5];
    aero_cuda_tensor gate_exps, up_exps, down_exps;
    const float* router;         /* may be NULL: then only the *_ffn_block and route calls work */
    const float* router_bias;    /* (n_expert,) added to the logits, or NULL */
    const float* shexp_gate_inp; /* required when has_shared */
    aero_cuda_tensor shexp_gate, shexp_up, shexp_down;
    const int32_t* resident_ids; /* host array of n_resident ids; read only when n_resident > 0 */
} aero_cuda_moe_desc;

/* Open a layer: upload the experts once into device-resident, expert-major,
 * 128-byte-aligned quant-block planes. Every device allocation is charged to
 * the memory guard below; a refusal returns NULL with the reason in err.
 * Replaces the per-token fetch path engine/model.py:523-547 + 651-678. */
void* aero_cuda_moe_open(const aero_cuda_moe_desc* desc, char* err, int errlen);

/* Open layer `layer` straight from a GGUF file (mmap), reading
 * blk.<layer>.ffn_{gate_inp,gate_exps,up_exps,down_exps}.weight and the
 * optional shared-expert tensors, expert_count/expert_used_count from the
 * metadata, norm_topk_prob = 1 (engine/model.py:193-224). Replaces
 * GgufReader (src/gguf.cpp:150-275) + GGUFReader.tensor_rows
 * (engine/gguf.py:297-314) on this path. */
void* aero_cuda_moe_open_gguf(const char* path, int layer, int device, int expert_begin,
                              int expert_end, char* err, int errlen);
/* The same layer's description without opening it (no device work): out8 =
 * n_embd, n_expert, n_expert_used, ffn_len, ffn_len_shared, has_shared, the
 * expert tensors' ggml type, whether ffn_gate_inp.weight is present. The
 * shape checks are aero_cuda_moe_open_gguf's. 0 / -1 with the reason in err.
 * Replaces the metadata reads of GGUFReader (engine/gguf.py:186-230) that the
 * reference's loader makes before it plans a layer (engine/model.py:193-224). */
int aero_cuda_moe_gguf_info(const char* path, int layer, int64_t* out8, char* err, int errlen);

void aero_cuda_moe_close(void* handle);

/* Expert paging on a resident-subset handle (its n_resident slots; for models
 * whose experts exceed device memory): put expert `expert`'s gate, up and down
 * bytes (one expert of each tensor, the layer's GGUF type Q8_0 / Q4_K, host or
 * 16-byte aligned device memory) into plane slot `slot`; the expert the slot
 * held is no longer resident. Ordered after the handle's earlier calls; returns
 * when the slot is ready. Refused for an expert resident in another slot. With
 * the routing computed first (aero_cuda_moe_router_logits + aero_cuda_moe_route,
 * exact, not speculative) a caller pages in a call's experts before the block
 * runs on the same logits: the router-ahead prefetch of ENGINE_DESIGN.md
 * §3.3 (ENGINE_DESIGN.md:99-101). 0 / -1. */
int aero_cuda_moe_page_in(void* handle, int slot, int expert, const void* gate, const void* up,
                          const void* down);
/* The expert held by each slot into slot_expert[0..n_resident) when n is at
 * least n_resident; returns n_resident (-1 for a NULL handle). */
int aero_cuda_moe_resident(void* handle, int32_t* slot_expert, int n);

/* Device bytes a handle opened from desc keeps resident (router rows, the
 * tensor-core router's split copy, the quantised expert and shared-expert
 * planes), as the memory guard charges them; no device work, the tensor data
 * is not read. The expert term of the reference's plan_footprint
 * (engine/model.py:828-832: fp32 bytes of the active experts) in the device
 * bytes this library actually holds. -1 for an invalid description. */
int64_t aero_cuda_moe_plan_bytes(const aero_cuda_moe_desc* desc);

/* Every MoE layer of a GGUF file as one table (n_layer <= 0: "<arch>.block_count").
 * Layers without expert tensors stay empty and their hook call returns 0.
 * aero_cuda_moe_model_forward has the aero_moe_fn signature and dispatches on
 * `layer`, so the reference's block loop takes the whole model with one call:
 *   aero_model_set_moe(model, aero_cuda_moe_model_forward, table);
 * (src/model.cpp:166-170, 385-387; the loop's is_moe flag marks the layers).
 * _layer returns the layer's handle (NULL for an empty layer) for the per-layer
 * calls above; _close closes every handle. */
void* aero_cuda_moe_model_open_gguf(const char* path, int n_layer, int device, char* err, int errlen);
int aero_cuda_moe_model_forward(void* table, int layer, const float* h, int T, int n_embd, float* out);
void* aero_cuda_moe_model_layer(void* table, int layer);
void aero_cuda_moe_model_close(void* table);

/* The block hook: exactly the aero_moe_fn signature (include/aero/model.hpp:83-84,
 * 176-177), so aero_model_set_moe(model, aero_cuda_moe_forward, handle) plugs it
 * in. Router logits are computed on the device from the layer's router
 * (engine/model.py:665-666). `layer` is not used to select weights (one handle
 * per layer). Returns 1 on success, 0 on refusal (src/model.cpp:169). */
int aero_cuda_moe_forward(void* handle, int layer, const float* h, int T, int n_embd, float* out);

/* Asynchronous calls with host buffers, for a stream of layer calls (serving):
 * submit enqueues the copy of h (T rows, host memory; pinned memory lets the
 * copies overlap the GPU's work) into slot `slot` (0 to 3), the block, and the
 * copy of the result into out, and returns at once; aero_cuda_moe_wait(handle,
 * slot) returns when that output is in `out` (and reports a bounded device wait
 * that gave up). Copies run on two streams of the handle besides its compute
 * stream, so later slots' inputs and earlier slots' outputs cross PCIe while
 * a block computes (three slots in turn keep both directions busy). h and out must stay untouched until the wait; a submit to a
 * slot still pending waits for it first. No reference counterpart (the
 * reference's calls are synchronous). 0 / -1. */
int aero_cuda_moe_submit(void* handle, int slot, const float* h, int T, float* out);
int aero_cuda_moe_wait(void* handle, int slot);

/* The block with caller-supplied router logits (T, n_expert): the contract of
 * aero_moe_ffn_block (include/aero/moe.hpp:43-52) with the experts already
 * resident. Returns 0 on success, -1 on refusal. */
int aero_cuda_moe_ffn_block(void* handle, const float* h, const float* router_logits, int T, float* out);

/* Router logits only, (T, n_expert): exposes the router kernel for the two-level
 * routing parity check. 0 / -1. */
int aero_cuda_moe_router_logits(void* handle, const float* h, int T, float* logits);

/* Batched top-k over (T, n_expert) logits with the handle's k and
 * norm_topk_prob; idx (T, k) int64, w (T, k) f32. aero_moe_route
 * (include/aero/moe.hpp:17-18) applied to T rows. 0 / -1. */
int aero_cuda_moe_route(void* handle, const float* logits, int T, int64_t* idx, float* w);

/* Handle-free batched aero_moe_route (src/moe.cpp:26-66): ties go to the lower
 * index; refuses k outside [1, n_expert], and (a limit of this implementation)
 * k > 32 or n_expert > 1024. 0 / -1. */
int aero_cuda_route(const float* logits, int T, int n_expert, int k, int norm_topk_prob,
                    int64_t* idx, float* w);

/* Dispatch permutation of the T*k (token, slot) pairs of idx (T, k): offsets
 * (n_expert + 1) is the exclusive prefix sum of per-expert counts and perm (T*k)
 * lists pair ids t*k+s ordered by (expert, token, slot). No reference
 * counterpart (the reference routes token by token, src/moe.cpp:136-154).
 * 0 / -1. */
int aero_cuda_dispatch(const int64_t* idx, int T, int k, int n_expert, int32_t* offsets,
                       int32_t* perm);

/* aero_cuda_dispatch without any device allocation. No counterpart in the
 * reference. For callers that must not allocate device memory when they route:
 * a process whose device budget is fully committed (the memory guard refuses
 * more), or a pipeline that cannot take cudaMalloc's implicit device-wide
 * synchronisation. Its scratch is one fixed 2 MiB device array inside this
 * library, which every GPU that loads the library holds until exit.
 * Limits: T*k <= 65536 pairs and n_expert <= 1024; larger calls are refused
 * (use aero_cuda_dispatch). idx (T, k) int64, offsets (n_expert + 1) and perm
 * (T*k) int32 must be device memory; the work runs on `stream` (NULL: the
 * default stream) and every call waits for that work to finish before it
 * returns (it reads the kernels' error flag back to the host). The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress); make that
 * first call before any stream capture. All calls share the array: calls whose
 * work overlaps on the GPU race and corrupt each other's results. 0 / -1; the
 * reason for -1 is in aero_cuda_moe_last_error(NULL). */
int aero_cuda_dispatch_noalloc(const int64_t* idx, int T, int k, int n_expert, int32_t* offsets,
                               int32_t* perm, void* stream);

/* GGUF dequantisation to f32, bit-identical to aero_dequant_ref
 * (src/kernels.cpp:591-606) for Q8_0, Q4_K and F32. 1 ok / 0 refusal (unknown
 * type, n not whole blocks, raw_len too short). */
int aero_cuda_dequant(int dtype, const uint8_t* raw, int64_t raw_len, float* out, int64_t n_values);

/* Block quantiser for Q8_0 / Q4_K (no reference counterpart: the reference only
 * reads these formats). Bytes equal aero_b200.quant.quantize. 1 ok / 0. */
int aero_cuda_quantize(int dtype, const float* x, int64_t n_values, uint8_t* out, int64_t out_len);

/* Per-stage device timing with CUDA events on the handle's stream (router,
 * top-k, dispatch, gate/up, down, combine). While on, each call waits for its
 * own events. stage_times returns the accumulated milliseconds and call
 * counts per stage since profiling was switched on. */
int aero_cuda_moe_set_profiling(void* handle, int on);
int aero_cuda_moe_stage_times(void* handle, double* ms, int64_t* counts, int n);

/* Options. AERO_CUDA_OPT_GEMM_MIN_TOKENS: calls with at least this many tokens
 * run the expert products as tcgen05 grouped GEMMs (f16 operands, fp32
 * accumulate); smaller calls use the fp32 GEMV path (default 64; also read from
 * the AERO_GEMM_MIN_TOKENS environment variable at open). 0 / -1. */
#define AERO_CUDA_OPT_GEMM_MIN_TOKENS 1
/* AERO_CUDA_OPT_ROUTER_TC: 1 (default) projects the router of calls with at
 * least 16 tokens on the tensor cores (three TF32 products of split f32
 * operands, f32 accumulate: f32-level accuracy); 0 keeps the f32 SIMT kernels. */
#define AERO_CUDA_OPT_ROUTER_TC 2
/* AERO_CUDA_OPT_PEER_WAIT_MS: how long a peer-exchange kernel waits for a
 * peer's step flag before it gives up and records code 21 / 22 (default 5000;
 * 1 to 600000). Applies from the next step. */
#define AERO_CUDA_OPT_PEER_WAIT_MS 3
/* AERO_CUDA_OPT_DECODE_FUSED: 1 (default) runs calls of up to 32 tokens on Q8_0 /
 * Q4_K layers as one cooperative kernel (router, top-k, dispatch, gate/up,
 * down, combine); 0 runs them as the separate router / top-k / dispatch / GEMV /
 * combine kernels. */
#define AERO_CUDA_OPT_DECODE_FUSED 4
int aero_cuda_moe_set_option(void* handle, int option, int64_t value);

/* 0, or the code of the first bounded device wait of this handle's kernels that
 * gave up since the last status read (router pipeline, prefill GEMM pipeline,
 * fused decode: 31, peer exchange: 21 rows, 22 returns), or 41 when a routing
 * selected an expert that a resident-subset handle does not hold, after
 * synchronising the handle's stream. Such a code raised during a call with
 * device pointers (which returns without synchronising) is also reported by the
 * handle's next call, which is then refused. No reference counterpart (the
 * reference has no device waits). The pipeline codes are cleared by the read;
 * a peer-exchange code stays. */
int aero_cuda_moe_status(void* handle);

/* ------------------------------------------------------- expert parallel
 * No reference counterpart: the reference runs a layer in one process
 * (src/moe.cpp:122-161). One process per GPU; rank r opens its layer with
 * experts [begin[r], begin[r+1]) (aero_cuda_moe_open / _open_gguf expert
 * range) and a step over its T local tokens is
 *   1. aero_cuda_ep_dispatch: route the T tokens (router + top-k over all
 *      experts), write the T self rows, and the send buffer as n_ranks slabs
 *      of slab_rows rows: slab r holds one row per token with at least one
 *      expert on rank r (tokens in order), then padding rows whose metadata
 *      names no expert; counts[r] real rows per slab;
 *   2. the caller exchanges the slabs with equal splits (NCCL all-to-all, no
 *      host synchronisation) so that the slabs from all ranks follow the
 *      self rows in one buffer;
 *   3. aero_cuda_ep_expert_block over the R = T + n_ranks * slab_rows rows
 *      (self rows first; they also take the shared expert): out[r] = sum of
 *      w * expert(x) over the row's slots this rank owns (+ the shared expert),
 *      as f32 or f16 partial rows;
 *   4. the caller sends rows [T, R) of that output back (reverse all-to-all,
 *      landing in the send buffer's slab layout);
 *   5. aero_cuda_ep_combine: out[t] = self part + the remote parts in rank
 *      order.
 * All buffers are device memory, 16-byte aligned; the work is enqueued on the
 * handle's stream and the calls do not synchronise. Rows are n_embd wide, f32
 * or f16 (f16 rows take the tcgen05 GEMM path). A metadata row is
 * aero_cuda_ep_meta_ld(handle) = 2k + 2 int32: k global expert ids (-1: not
 * owned by the receiver), k weights (f32 bits), the shared gate (f32 bits),
 * padding. 0 / -1 with the reason in aero_cuda_moe_last_error(handle). */
#define AERO_EP_ROWS_F32 0
#define AERO_EP_ROWS_F16 1
int aero_cuda_ep_meta_ld(void* handle);
/* rank_expert_begin: host array of n_ranks + 1 ascending expert ids from 0 to
 * n_expert; this handle must hold [begin[rank], begin[rank+1]). send_rows /
 * send_meta hold n_ranks * slab_rows rows; slab_rows >= T. counts: n_ranks + 1
 * int32 (counts[n_ranks] = total real rows); pos: (T, n_ranks) int32, the send
 * row of each (token, remote rank) in the slab layout, or -1. */
int aero_cuda_ep_dispatch(void* handle, const float* x, int T, int n_ranks, int rank,
                          const int32_t* rank_expert_begin, int row_dtype, void* self_rows,
                          int32_t* self_meta, void* send_rows, int32_t* send_meta, int slab_rows,
                          int32_t* counts, int32_t* pos);
/* rows (R, n_embd) with metadata (R, meta_ld); the first n_shared rows take the
 * shared expert with their metadata's gate. out (R, n_embd) in out_dtype: f32,
 * or f16 (halves the return exchange; needs the GEMM path, i.e. f16 rows). */
int aero_cuda_ep_expert_block(void* handle, const void* rows, int row_dtype, const int32_t* meta,
                              int R, int n_shared, void* out, int out_dtype);
/* self_out (T, n_embd): rows [0, T) of the expert block's output; back
 * (n_ranks * slab_rows, n_embd): the returned rows in the send slabs' layout;
 * both in parts_dtype (AERO_EP_ROWS_*). out (T, n_embd) f32. */
int aero_cuda_ep_combine(void* handle, const void* self_out, const void* back, int parts_dtype,
                         const int32_t* pos, int T, int n_ranks, int rank, float* out);
/* Metadata ids received since the last call that named an expert this handle
 * does not hold (they were skipped). Synchronises the handle's stream. */
int aero_cuda_ep_bad_ids(void* handle);

/* Expert parallel over peer memory: the same step without a collective
 * library. Each rank allocates an exchange window (rows, metadata and returned
 * partials for n_ranks slabs of slab_rows rows, plus step flags) that the other
 * ranks map through CUDA IPC; the dispatch kernel stores the rows straight into
 * the owners' windows over NVLink, the owners' return kernel stores the partial
 * outputs straight back, and kernels wait for the peers' step flags (bounded
 * waits; a wait that gives up is reported by aero_cuda_ep_peer_status). Needs
 * one GPU per rank with peer access between them. Protocol:
 *   aero_cuda_ep_peer_open on every rank -> all-gather the AERO_EP_IPC_BYTES
 *   handles (rank order) -> aero_cuda_ep_peer_connect -> a host barrier ->
 *   steps (aero_cuda_ep_peer_step, every rank the same number of times, T = 0
 *   allowed) -> synchronise, host barrier -> aero_cuda_ep_peer_close. */
#define AERO_EP_IPC_BYTES 128
int aero_cuda_ep_peer_open(void* handle, int n_ranks, int rank, const int32_t* rank_expert_begin,
                           int slab_rows, int row_dtype, void* ipc_out);
/* ipc_all: n_ranks blobs of AERO_EP_IPC_BYTES bytes (as written by
 * aero_cuda_ep_peer_open), in rank order. Each blob carries its rank's window
 * layout (n_ranks, slab_rows, row type, row width, k, n_expert, window size and
 * a hash of the expert table); connect is refused, before any peer window is
 * mapped, when any rank's layout differs from this rank's, and when two ranks
 * share a GPU. */
int aero_cuda_ep_peer_connect(void* handle, const void* ipc_all);
/* x (T, n_embd) f32 device, T <= slab_rows -> out (T, n_embd) f32 device;
 * enqueued on the handle's stream. A step refused on one rank (or a rank that
 * stops stepping) leaves the other ranks' waits to give up after the handle's
 * peer wait limit (AERO_CUDA_OPT_PEER_WAIT_MS, 5 s by default); their
 * aero_cuda_ep_peer_status then reports it, their outputs are not valid, and
 * once the host has seen the code (a status read, or the next step's entry)
 * every later step is refused with the code in the error message, until the
 * exchange is closed (aero_cuda_ep_peer_close) and opened again. */
int aero_cuda_ep_peer_step(void* handle, const float* x, int T, float* out);
/* 0, or the code of the first wait that gave up (21 rows, 22 returns);
 * synchronises the handle's stream. */
int aero_cuda_ep_peer_status(void* handle);
/* Rows sent to / received from each rank in the last step (host arrays of
 * n_ranks; synchronises). */
int aero_cuda_ep_peer_counts(void* handle, int32_t* sent, int32_t* received);
/* Phase timing (on != 0; synchronises each step); ms (7 doubles or NULL): mean
 * device time per phase since the last read (route, plan, pack, rows wait +
 * unpack, experts, return, combine). Returns the number of steps averaged. */
int aero_cuda_ep_peer_profile(void* handle, int on, double* ms);
/* Unmaps the peers' windows and frees this rank's (call after a host barrier
 * that follows every rank's last step). */
int aero_cuda_ep_peer_close(void* handle);

/* Run the handle's work on this cudaStream_t (NULL: the handle's own stream). */
int aero_cuda_moe_set_stream(void* handle, void* stream);
/* Layer geometry: out[0..7] = n_embd, n_expert, n_expert_used, ffn_len,
 * ffn_len_shared, has_shared, expert dtype, norm_topk_prob. */
int aero_cuda_moe_info(void* handle, int32_t* out8);
/* Last error of a handle, or of the handle-free calls when handle is NULL. */
const char* aero_cuda_moe_last_error(void* handle);
/* JSON record: calls, tokens, device bytes by class, last call device time. */
int aero_cuda_moe_stats(void* handle, char* buf, int len);
int aero_cuda_device_count(void);

/* ---------------------------------------------------------------- guard
 * Device memory guard (src/memory_guard.cpp, include/aero/memory_guard.hpp):
 * classes 0 weights-resident, 1 weights-cache, 2 kv-cache, 3 scratch,
 * 4 runtime; -1 in aero_cuda_guard_committed means the total. */
void aero_cuda_guard_set_budget(size_t bytes);
size_t aero_cuda_guard_budget(void);
size_t aero_cuda_guard_committed(int cls);
size_t aero_cuda_guard_headroom(void);
int aero_cuda_guard_try_reserve(size_t bytes, int cls);
void aero_cuda_guard_release(size_t bytes, int cls);
int aero_cuda_guard_admit_plan(size_t planned, char* why, int why_len);
typedef size_t (*aero_cuda_evict_fn)(void* ctx, size_t need);
void aero_cuda_guard_set_evictor(aero_cuda_evict_fn fn, void* ctx);
void aero_cuda_guard_fail_nth_alloc(long n);
size_t aero_cuda_guard_own_footprint(int device);
size_t aero_cuda_guard_device_free(int device);
int aero_cuda_guard_preflight(int device, size_t headroom);
typedef void (*aero_cuda_breach_fn)(void* ctx, size_t footprint, size_t budget);
void aero_cuda_guard_set_on_breach(aero_cuda_breach_fn fn, void* ctx);
int aero_cuda_guard_exceeded(void);
size_t aero_cuda_guard_peak_footprint(void);
void aero_cuda_guard_reset_exceeded(void);
void aero_cuda_guard_start_monitor(int device, unsigned interval_ms);
void aero_cuda_guard_stop_monitor(void);
/* LoadGate (src/memory_guard.cpp:314-378). */
void* aero_cuda_loadgate_open(size_t planned, int device);
void aero_cuda_loadgate_close(void* gate);
void aero_cuda_loadgate_set_pause_ms(void* gate, unsigned ms);
int aero_cuda_loadgate_next_chunk(void* gate, size_t chunk, int cls);
int aero_cuda_loadgate_pause_and_check(void* gate);
int aero_cuda_loadgate_ok(void* gate);
int aero_cuda_loadgate_done(void* gate);
size_t aero_cuda_loadgate_taken(void* gate);
size_t aero_cuda_loadgate_reserved(void* gate);
size_t aero_cuda_loadgate_remaining(void* gate);
int aero_cuda_loadgate_reason(void* gate, char* buf, int len);

#ifdef __cplusplus
}
#endif

#endif /* AERO_CUDA_MOE_H */
