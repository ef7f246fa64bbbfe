/*
 * CPU restatement of Aero's MoE FFN path — TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity oracle for the CUDA library in aero_b200/. Only the
 * tests, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it,
 * and only as the checker: it is never the thing measured or shipped.
 *
 * Every function restates the reference algorithm it names (paths are within
 * the Aero project):
 *   f16 decode              src/kernels.cpp:29-52
 *   Q4_K scale unpack       src/kernels.cpp:65-73, engine/quant.py:142-156
 *   dequant Q8_0 / Q4_K     src/kernels.cpp:337-373, engine/quant.py:133-181
 *   top-k route             src/moe.cpp:26-66
 *   expert accumulation     src/moe.cpp:68-88
 *   shared expert           src/moe.cpp:90-120
 *   block                   src/moe.cpp:122-161, with the per-call dequant cache
 *                           of engine/model.py:651-678
 *   router projection       engine/model.py:665-666 (h @ W_r^T)
 * The dispatch permutation has no reference counterpart; orc_dispatch is the
 * host reference sort that defines it: pairs ordered by (expert, token, slot).
 *
 * Built with plain gcc, no -ffast-math, so float arithmetic is IEEE and in
 * program order.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define DT_F32 0
#define DT_Q8_0 8
#define DT_Q4_K 12

/* ---------------------------------------------------------------- fp16 */
static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            /* subnormal: shift the mantissa up until its leading one reaches bit 10 */
            uint32_t e = 113, m = mant;
            while ((m & 0x400u) == 0) { m <<= 1; --e; }
            bits = sign | (e << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (ex == 0x1Fu) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

static void q4k_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 63u;
        *m = q[j + 4] & 63u;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0Fu) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

int64_t orc_block_bytes(int dtype) {
    return dtype == DT_Q8_0 ? 34 : dtype == DT_Q4_K ? 144 : dtype == DT_F32 ? 4 : 0;
}
int64_t orc_block_values(int dtype) {
    return dtype == DT_Q8_0 ? 32 : dtype == DT_Q4_K ? 256 : dtype == DT_F32 ? 1 : 0;
}

/* Dequantise n values. Returns 1 on success, 0 on refusal (unknown type, n not a
 * whole number of blocks, or raw_len too short) — the refusal convention of
 * aero_dequant_ref. */
int orc_dequant(int dtype, const uint8_t* raw, int64_t raw_len, float* out, int64_t n) {
    const int64_t bv = orc_block_values(dtype), bb = orc_block_bytes(dtype);
    if (bv <= 0 || n % bv) return 0;
    const int64_t nb = n / bv;
    if (raw_len < nb * bb) return 0;
    if (dtype == DT_F32) {
        memcpy(out, raw, (size_t)n * 4);
        return 1;
    }
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = raw + b * bb;
        float* o = out + b * bv;
        if (dtype == DT_Q8_0) {
            const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const int8_t* q = (const int8_t*)(blk + 2);
            for (int i = 0; i < 32; ++i) o[i] = d * (float)q[i];
        } else {
            const float d = f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            const float dmin = f16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
            const uint8_t* sc = blk + 4;
            const uint8_t* qs = blk + 16;
            for (int g = 0; g < 4; ++g) {
                uint8_t s1, m1, s2, m2;
                q4k_scale_min(2 * g, sc, &s1, &m1);
                q4k_scale_min(2 * g + 1, sc, &s2, &m2);
                const float f1 = d * (float)s1, g1 = dmin * (float)m1;
                const float f2 = d * (float)s2, g2 = dmin * (float)m2;
                for (int i = 0; i < 32; ++i) {
                    const uint8_t byte = qs[32 * g + i];
                    o[64 * g + i] = f1 * (float)(byte & 0x0F) - g1;
                    o[64 * g + 32 + i] = f2 * (float)(byte >> 4) - g2;
                }
            }
        }
    }
    return 1;
}

/* ------------------------------------------------------------------ route */
static const float* g_sort_logits;
static int cmp_desc_lowidx(const void* a, const void* b) {
    const int ia = *(const int*)a, ib = *(const int*)b;
    const float la = g_sort_logits[ia], lb = g_sort_logits[ib];
    if (la != lb) return la > lb ? -1 : 1;
    return ia < ib ? -1 : (ia > ib);
}

static int route_one(const float* lg, int E, int k, int norm, int64_t* idx, float* w, int* order) {
    if (k <= 0 || k > E) return -1;
    /* Selection by repeated scan: strictly greater logit wins, equal logits keep
     * the earlier (lower) index — the comparator of src/moe.cpp:35-39. */
    unsigned char* taken = (unsigned char*)calloc((size_t)E, 1);
    for (int i = 0; i < k; ++i) {
        int best = -1;
        for (int e = 0; e < E; ++e) {
            if (taken[e]) continue;
            if (best < 0 || lg[e] > lg[best]) best = e;
        }
        order[i] = best;
        taken[best] = 1;
    }
    free(taken);
    for (int i = 0; i < k; ++i) idx[i] = order[i];
    if (norm) {
        float m = lg[order[0]];
        for (int i = 1; i < k; ++i) m = fmaxf(m, lg[order[i]]);
        float sum = 0.0f;
        for (int i = 0; i < k; ++i) {
            const float e = expf(lg[order[i]] - m);
            w[i] = e;
            sum += e;
        }
        for (int i = 0; i < k; ++i) w[i] /= sum;
    } else {
        float m = lg[0];
        for (int i = 1; i < E; ++i) m = fmaxf(m, lg[i]);
        double den = 0.0;
        for (int i = 0; i < E; ++i) den += (double)expf(lg[i] - m);
        for (int i = 0; i < k; ++i) w[i] = (float)((double)expf(lg[order[i]] - m) / den);
    }
    return 0;
}

/* Batched top-k routing over T rows of logits (T, E). 0 ok, -1 refusal. */
int orc_route(const float* logits, int T, int E, int k, int norm, int64_t* idx, float* w) {
    if (k <= 0 || k > E) return -1;
    int* order = (int*)malloc(sizeof(int) * (size_t)k);
    for (int t = 0; t < T; ++t)
        route_one(logits + (size_t)t * E, E, k, norm, idx + (size_t)t * k, w + (size_t)t * k, order);
    free(order);
    return 0;
}

/* Full descending order with ties to the lower index (used by tests to
 * cross-check the scan selection above on large E). */
void orc_argsort_desc(const float* lg, int E, int32_t* order) {
    int* o = (int*)malloc(sizeof(int) * (size_t)E);
    for (int i = 0; i < E; ++i) o[i] = i;
    g_sort_logits = lg;
    qsort(o, (size_t)E, sizeof(int), cmp_desc_lowidx);
    for (int i = 0; i < E; ++i) order[i] = o[i];
    free(o);
}

/* ------------------------------------------------------- expert arithmetic */
static float silu_f(float x) { return x / (1.0f + expf(-x)); }
static float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }

/* acc += wt * down @ (silu(gate @ h) * (up @ h)); sequential fp32 dot order. */
void orc_expert_accum(const float* h, int d, const float* gate, const float* up,
                      const float* down, int F, float wt, float* acc) {
    float* act = (float*)malloc(sizeof(float) * (size_t)F);
    for (int j = 0; j < F; ++j) {
        const float* gj = gate + (size_t)j * d;
        const float* uj = up + (size_t)j * d;
        float g = 0.0f, u = 0.0f;
        for (int c = 0; c < d; ++c) {
            g += h[c] * gj[c];
            u += h[c] * uj[c];
        }
        act[j] = silu_f(g) * u;
    }
    for (int e = 0; e < d; ++e) {
        const float* de = down + (size_t)e * F;
        float s = 0.0f;
        for (int j = 0; j < F; ++j) s += act[j] * de[j];
        acc[e] += wt * s;
    }
    free(act);
}

/* out[t] += sigmoid(h_t . gate_inp) * down @ (silu(gate @ h_t) * (up @ h_t)). */
void orc_shared_accum(const float* h, int T, int d, const float* gate_inp,
                      const float* gate, const float* up, const float* down, int F, float* out) {
    for (int t = 0; t < T; ++t) {
        const float* ht = h + (size_t)t * d;
        float gi = 0.0f;
        for (int c = 0; c < d; ++c) gi += ht[c] * gate_inp[c];
        const float sg = sigmoid_f(gi);
        float* tmp = (float*)calloc((size_t)d, sizeof(float));
        orc_expert_accum(ht, d, gate, up, down, F, 1.0f, tmp);
        /* the reference adds sgate * s per element; tmp holds 1.0f * s exactly */
        for (int e = 0; e < d; ++e) out[(size_t)t * d + e] += sg * tmp[e];
        free(tmp);
    }
}

/* Router projection logits[t][e] = h_t . W_r[e] (+ bias[e]); sequential fp32,
 * or f64 accumulation when f64acc is set (used to tell which side of a near-tie
 * a reduction-order difference falls on). */
void orc_router_logits(const float* h, int T, int d, const float* W, int E,
                       const float* bias, int f64acc, float* out) {
    for (int t = 0; t < T; ++t) {
        const float* ht = h + (size_t)t * d;
        for (int e = 0; e < E; ++e) {
            const float* we = W + (size_t)e * d;
            float v;
            if (f64acc) {
                double s = 0.0;
                for (int c = 0; c < d; ++c) s += (double)ht[c] * (double)we[c];
                v = (float)s;
            } else {
                float s = 0.0f;
                for (int c = 0; c < d; ++c) s += ht[c] * we[c];
                v = s;
            }
            if (bias) v += bias[e];
            out[(size_t)t * E + e] = v;
        }
    }
}

/* --------------------------------------------------------------- dispatch */
/* Counting sort of the T*k (token, slot) pairs by expert; within an expert by
 * token then slot (= by pair index p = t*k + s). offsets has E+1 entries;
 * perm[offsets[e] .. offsets[e+1]) lists the pair indices routed to e. */
void orc_dispatch(const int64_t* idx, int T, int k, int E, int32_t* offsets, int32_t* perm) {
    const int P = T * k;
    int32_t* cnt = (int32_t*)calloc((size_t)E + 1, sizeof(int32_t));
    for (int p = 0; p < P; ++p) cnt[idx[p]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + cnt[e];
    for (int e = 0; e < E; ++e) cnt[e] = offsets[e];
    for (int p = 0; p < P; ++p) perm[cnt[idx[p]]++] = p;
    free(cnt);
}

/* -------------------------------------------------------------- the block */
typedef struct {
    int dtype;
    const uint8_t* data; /* GGUF bytes of the whole (E, rows, cols) tensor */
    int rows, cols;
} orc_mat;

static int64_t mat_expert_bytes(const orc_mat* m) {
    return (int64_t)m->rows * ((int64_t)m->cols / orc_block_values(m->dtype)) *
           orc_block_bytes(m->dtype);
}

static int dequant_expert(const orc_mat* m, int e, float* out) {
    const int64_t eb = mat_expert_bytes(m);
    return orc_dequant(m->dtype, m->data + (int64_t)e * eb, eb, out, (int64_t)m->rows * m->cols);
}

typedef struct {
    const float* h;
    const int64_t* idx;
    const float* w;
    float** cache_g;
    float** cache_u;
    float** cache_d;
    int d, k, F, t0, t1;
    float* out;
} accum_job;

static void* accum_worker(void* arg) {
    accum_job* j = (accum_job*)arg;
    for (int t = j->t0; t < j->t1; ++t) {
        float* acc = j->out + (size_t)t * j->d;
        for (int c = 0; c < j->d; ++c) acc[c] = 0.0f;
        for (int i = 0; i < j->k; ++i) {
            const int e = (int)j->idx[(size_t)t * j->k + i];
            orc_expert_accum(j->h + (size_t)t * j->d, j->d, j->cache_g[e], j->cache_u[e],
                             j->cache_d[e], j->F, j->w[(size_t)t * j->k + i], acc);
        }
    }
    return NULL;
}

typedef struct {
    const orc_mat *g, *u, *dn;
    float** cg;
    float** cu;
    float** cd;
    const int* list;
    int n, tid, nthreads;
    int fail;
} deq_job;

static void* deq_worker(void* arg) {
    deq_job* j = (deq_job*)arg;
    for (int i = j->tid; i < j->n; i += j->nthreads) {
        const int e = j->list[i];
        if (!dequant_expert(j->g, e, j->cg[e]) || !dequant_expert(j->u, e, j->cu[e]) ||
            !dequant_expert(j->dn, e, j->cd[e]))
            j->fail = 1;
    }
    return NULL;
}

/* MoE block over quantised experts, following src/moe.cpp:122-161 with the
 * engine/model.py:651-678 per-call cache (each selected expert is dequantised
 * once per call). gate/up are (E, F, d), down is (E, d, F). The shared expert
 * (sh_* with its own width Fs) is optional. `nthreads` splits dequant and the
 * per-token accumulation across POSIX threads; per-token arithmetic is
 * unchanged, so the result does not depend on nthreads.
 * Returns 0 ok, -1 refusal. */
int orc_moe_block_q(const float* h, const float* router_logits, int T, int d, int E, int k,
                    int F, int norm, int dtype, const uint8_t* gate, const uint8_t* up,
                    const uint8_t* down, int has_shared, const float* sh_gate_inp,
                    int sh_dtype, const uint8_t* sh_gate, const uint8_t* sh_up,
                    const uint8_t* sh_down, int Fs, int nthreads, float* out) {
    if (k <= 0 || k > E || T < 0) return -1;
    if (nthreads < 1) nthreads = 1;
    int64_t* idx = (int64_t*)malloc(sizeof(int64_t) * (size_t)T * k + 8);
    float* w = (float*)malloc(sizeof(float) * (size_t)T * k + 8);
    if (orc_route(router_logits, T, E, k, norm, idx, w) != 0) { free(idx); free(w); return -1; }

    orc_mat mg = {dtype, gate, F, d}, mu = {dtype, up, F, d}, md = {dtype, down, d, F};
    float** cg = (float**)calloc((size_t)E, sizeof(float*));
    float** cu = (float**)calloc((size_t)E, sizeof(float*));
    float** cd = (float**)calloc((size_t)E, sizeof(float*));
    int* list = (int*)malloc(sizeof(int) * (size_t)E);
    int n = 0;
    for (int p = 0; p < T * k; ++p) {
        const int e = (int)idx[p];
        if (!cg[e]) {
            cg[e] = (float*)malloc(sizeof(float) * (size_t)F * d);
            cu[e] = (float*)malloc(sizeof(float) * (size_t)F * d);
            cd[e] = (float*)malloc(sizeof(float) * (size_t)F * d);
            list[n++] = e;
        }
    }
    int rc = 0;
    {
        pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
        deq_job* jobs = (deq_job*)calloc((size_t)nthreads, sizeof(deq_job));
        for (int i = 0; i < nthreads; ++i) {
            jobs[i] = (deq_job){&mg, &mu, &md, cg, cu, cd, list, n, i, nthreads, 0};
            pthread_create(&th[i], NULL, deq_worker, &jobs[i]);
        }
        for (int i = 0; i < nthreads; ++i) {
            pthread_join(th[i], NULL);
            if (jobs[i].fail) rc = -1;
        }
        free(th);
        free(jobs);
    }
    if (rc == 0) {
        pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
        accum_job* jobs = (accum_job*)calloc((size_t)nthreads, sizeof(accum_job));
        const int per = (T + nthreads - 1) / nthreads;
        for (int i = 0; i < nthreads; ++i) {
            int t0 = i * per, t1 = t0 + per;
            if (t0 > T) t0 = T;
            if (t1 > T) t1 = T;
            jobs[i] = (accum_job){h, idx, w, cg, cu, cd, d, k, F, t0, t1, out};
            pthread_create(&th[i], NULL, accum_worker, &jobs[i]);
        }
        for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
        free(th);
        free(jobs);
    }
    if (rc == 0 && has_shared && sh_gate_inp) {
        float* g = (float*)malloc(sizeof(float) * (size_t)Fs * d);
        float* u = (float*)malloc(sizeof(float) * (size_t)Fs * d);
        float* dn = (float*)malloc(sizeof(float) * (size_t)Fs * d);
        const int64_t gb = (int64_t)Fs * (d / orc_block_values(sh_dtype)) * orc_block_bytes(sh_dtype);
        if (!orc_dequant(sh_dtype, sh_gate, gb, g, (int64_t)Fs * d) ||
            !orc_dequant(sh_dtype, sh_up, gb, u, (int64_t)Fs * d) ||
            !orc_dequant(sh_dtype, sh_down, gb, dn, (int64_t)Fs * d))
            rc = -1;
        else
            orc_shared_accum(h, T, d, sh_gate_inp, g, u, dn, Fs, out);
        free(g);
        free(u);
        free(dn);
    }
    for (int e = 0; e < E; ++e) {
        free(cg[e]);
        free(cu[e]);
        free(cd[e]);
    }
    free(cg);
    free(cu);
    free(cd);
    free(list);
    free(idx);
    free(w);
    return rc;
}
