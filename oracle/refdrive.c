/*
 * Driver for the reference's own MoE block — TEST INFRASTRUCTURE ONLY.
 *
 * Links against oracle/_ref/libaero_ssm.so, which the Makefile beside this file
 * builds from the reference's src/ssm.cpp, src/moe.cpp and src/kernels.cpp with
 * the reference's own flags. It supplies the fetch callback that
 * aero_moe_ffn_block (src/moe.cpp:122-161) calls for every routed expert: the
 * callback copies a full fp32 expert matrix out of a per-call cache that the
 * reference's own dequantiser (aero_dequant_ref, src/kernels.cpp:591-606) fills
 * once per selected expert, the way engine/model.py:651-678 caches experts.
 * Token shards run on POSIX threads; aero_moe_ffn_block keeps no global state.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef int (*aero_moe_fetch_fn)(void* ctx, int which, int expert, float* out);
int aero_moe_route(const float* logits, int n_expert, int k, int norm_topk_prob,
                   int64_t* idx_out, float* w_out);
int aero_moe_ffn_block(const float* h, const float* router_logits, int T, int n_embd,
                       int n_expert, int n_expert_used, int ffn_len, int norm_topk_prob,
                       int has_shared, const float* shexp_gate_inp, const float* shexp_gate,
                       const float* shexp_up, const float* shexp_down,
                       aero_moe_fetch_fn fetch, void* ctx, float* out);
int aero_dequant_ref(int t, const uint8_t* raw, int64_t raw_len, float* out, int64_t n_values);
int64_t aero_dtype_block_bytes(int t);
int64_t aero_dtype_block_values(int t);

typedef struct {
    float** mats[3]; /* per expert fp32 gate / up / down */
    size_t n_floats;
} cache_t;

static int fetch_cb(void* ctx, int which, int expert, float* out) {
    cache_t* c = (cache_t*)ctx;
    if (which < 0 || which > 2 || !c->mats[which][expert]) return 1;
    memcpy(out, c->mats[which][expert], c->n_floats * sizeof(float));
    return 0;
}

typedef struct {
    const float *h, *logits;
    int T, d, E, k, F, norm, has_shared;
    const float *sgi, *sg, *su, *sd;
    cache_t* cache;
    float* out;
    int rc;
} shard_t;

static void* shard_worker(void* a) {
    shard_t* s = (shard_t*)a;
    s->rc = aero_moe_ffn_block(s->h, s->logits, s->T, s->d, s->E, s->k, s->F, s->norm,
                               s->has_shared, s->sgi, s->sg, s->su, s->sd, fetch_cb, s->cache,
                               s->out);
    return NULL;
}

typedef struct {
    int dtype;
    const uint8_t* src[3];
    int64_t ebytes;
    int64_t nvals;
    cache_t* cache;
    const int* list;
    int n, tid, nth, fail;
} deq_t;

static void* deq_worker(void* a) {
    deq_t* j = (deq_t*)a;
    for (int i = j->tid; i < j->n; i += j->nth) {
        const int e = j->list[i];
        for (int w = 0; w < 3; ++w)
            if (aero_dequant_ref(j->dtype, j->src[w] + (int64_t)e * j->ebytes, j->ebytes,
                                 j->cache->mats[w][e], j->nvals) != 1)
                j->fail = 1;
    }
    return NULL;
}

/* One reference MoE block call over quantised experts: route (to find the
 * selected experts), dequantise each selected expert once, then run
 * aero_moe_ffn_block on `nthreads` token shards. The shared expert is passed as
 * fp32 (the reference ABI takes it dequantised, engine/moe.py:192-197) and
 * shares ffn_len with the routed experts, as src/moe.cpp:156-159 requires.
 * Returns 0 ok, -1 on any refusal. */
int refdrive_block(const float* h, const float* logits, int T, int d, int E, int k, int F,
                   int norm, int dtype, const uint8_t* gate, const uint8_t* up,
                   const uint8_t* down, int has_shared, const float* sgi, const float* sg,
                   const float* su, const float* sd, int nthreads, float* out) {
    if (k <= 0 || k > E) return -1;
    if (nthreads < 1) nthreads = 1;
    const int64_t bv = aero_dtype_block_values(dtype), bb = aero_dtype_block_bytes(dtype);
    if (bv <= 0 || d % bv || F % bv) return -1;
    const int64_t ebytes = (int64_t)F * (d / bv) * bb; /* gate/up (F,d) and down (d,F) */
    const size_t nf = (size_t)F * d;

    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)k);
    float* w = (float*)malloc(sizeof(float) * (size_t)k);
    cache_t cache;
    cache.n_floats = nf;
    for (int m = 0; m < 3; ++m) cache.mats[m] = (float**)calloc((size_t)E, sizeof(float*));
    int* list = (int*)malloc(sizeof(int) * (size_t)E);
    int n = 0;
    for (int t = 0; t < T; ++t) {
        aero_moe_route(logits + (size_t)t * E, E, k, norm, idx, w);
        for (int i = 0; i < k; ++i) {
            const int e = (int)idx[i];
            if (!cache.mats[0][e]) {
                for (int m = 0; m < 3; ++m) cache.mats[m][e] = (float*)malloc(nf * sizeof(float));
                list[n++] = e;
            }
        }
    }
    int rc = 0;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    deq_t* dj = (deq_t*)calloc((size_t)nthreads, sizeof(deq_t));
    for (int i = 0; i < nthreads; ++i) {
        dj[i] = (deq_t){dtype, {gate, up, down}, ebytes, (int64_t)nf, &cache, list, n, i,
                        nthreads, 0};
        pthread_create(&th[i], NULL, deq_worker, &dj[i]);
    }
    for (int i = 0; i < nthreads; ++i) {
        pthread_join(th[i], NULL);
        if (dj[i].fail) rc = -1;
    }
    if (rc == 0) {
        shard_t* sj = (shard_t*)calloc((size_t)nthreads, sizeof(shard_t));
        const int per = (T + nthreads - 1) / nthreads;
        int used = 0;
        for (int i = 0; i < nthreads; ++i) {
            const int t0 = i * per;
            if (t0 >= T) break;
            const int tn = (t0 + per > T ? T : t0 + per) - t0;
            sj[i] = (shard_t){h + (size_t)t0 * d, logits + (size_t)t0 * E, tn, d, E, k, F,
                              norm, has_shared, sgi, sg, su, sd, &cache,
                              out + (size_t)t0 * d, 0};
            pthread_create(&th[i], NULL, shard_worker, &sj[i]);
            used++;
        }
        for (int i = 0; i < used; ++i) {
            pthread_join(th[i], NULL);
            if (sj[i].rc != 0) rc = -1;
        }
        free(sj);
    }
    free(th);
    free(dj);
    for (int m = 0; m < 3; ++m) {
        for (int e = 0; e < E; ++e) free(cache.mats[m][e]);
        free(cache.mats[m]);
    }
    free(list);
    free(idx);
    free(w);
    return rc;
}
