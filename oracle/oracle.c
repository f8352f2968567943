/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY: fp64 CPU restatement of the WISP
 * routed-expert FFN hot path. Imported by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg as the checker; never by the product.
 *
 * Each function cites the reference code (file:line within the reference
 * project) whose algorithm it restates. The restatement is pinned against
 * the reference's golden vectors and against the reference's own compiled
 * CPU functions in tests/test_oracle.py.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* IEEE binary16 decode (normal, subnormal, inf/nan). The reference's host
 * converter is csrc/core/wisp_engine.c:53-79. */
float orc_f16_to_f32(uint16_t h) {
    int sign = h >> 15;
    int exp = (h >> 10) & 0x1f;
    int man = h & 0x3ff;
    double v;
    if (exp == 0)
        v = ldexp((double)man, -24);
    else if (exp == 31)
        v = man ? NAN : INFINITY;
    else
        v = ldexp((double)(man | 0x400), exp - 25);
    return (float)(sign ? -v : v);
}

float orc_bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint32_t rd32(const uint8_t* p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}
static uint64_t rd64(const uint8_t* p) {
    uint64_t v;
    memcpy(&v, p, 8);
    return v;
}

/* Header: 6 x u32 (magic, version, layer, expert, group_size, n_mats) then
 * 3 x {u32 rows, u32 cols, u64 packed, u64 scales, u64 zeros}; blobs follow
 * at byte 120 in matrix order, each matrix packed|scales|zeros.
 * Reference: csrc/core/wisp_engine.h:214-236, csrc/core/wisp_engine.c:268-303,
 * wisp/converter/partitioner.py:10-24. */
int orc_parse_header(const void* blob, size_t size, OrcMeta* m) {
    const uint8_t* b = (const uint8_t*)blob;
    if (!b || size < 120) return 6;
    if (rd32(b) != 0x57455850u || rd32(b + 4) != 1u || rd32(b + 20) != 3u)
        return 6;
    m->group_size = (int32_t)rd32(b + 16);
    uint64_t off = 120;
    for (int i = 0; i < 3; i++) {
        const uint8_t* mh = b + 24 + 32 * i;
        m->rows[i] = (int32_t)rd32(mh);
        m->cols[i] = (int32_t)rd32(mh + 4);
        m->packed_off[i] = (int64_t)off;
        off += rd64(mh + 8);
        m->scales_off[i] = (int64_t)off;
        off += rd64(mh + 16);
        m->zeros_off[i] = (int64_t)off;
        off += rd64(mh + 24);
    }
    m->total_bytes = (int64_t)off;
    return off > size ? 6 : 0;
}

/* value = (nibble - 8) * scale + zero; the low nibble holds the even index;
 * group = flattened index / gs. Reference: csrc/cuda/expert_loader.cu:35-42,
 * wisp/converter/quantizer.py:89-105. */
double orc_dequant(const OrcMat* w, int64_t i, int gs) {
    uint8_t byte = w->packed[i >> 1];
    int nib = (i & 1) ? (byte >> 4) : (byte & 0x0f);
    int64_t g = i / gs;
    double s = orc_f16_to_f32(w->scales[g]);
    double z = w->zeros ? orc_f16_to_f32(w->zeros[g]) : 0.0;
    return (double)(nib - 8) * s + z;
}

void orc_dequant_n(const OrcMat* w, int64_t n, int gs, float* out) {
    for (int64_t i = 0; i < n; i++) out[i] = (float)orc_dequant(w, i, gs);
}

/* Row-wise dot products; scale/zero are fetched once per group run. */
void orc_gemv_int4(const OrcMat* w, int gs, const double* x, double* y) {
    const int64_t cols = w->cols;
    for (int r = 0; r < w->rows; r++) {
        int64_t i = (int64_t)r * cols, end = i + cols;
        double acc = 0.0;
        while (i < end) {
            int64_t g = i / gs;
            int64_t gend = (g + 1) * (int64_t)gs;
            if (gend > end) gend = end;
            double s = orc_f16_to_f32(w->scales[g]);
            double z = w->zeros ? orc_f16_to_f32(w->zeros[g]) : 0.0;
            double qsum = 0.0, xsum = 0.0;
            for (; i < gend; i++) {
                uint8_t byte = w->packed[i >> 1];
                int nib = (i & 1) ? (byte >> 4) : (byte & 0x0f);
                double xv = x[i - (int64_t)r * cols];
                qsum += (double)(nib - 8) * xv;
                xsum += xv;
            }
            acc += s * qsum + z * xsum;
        }
        y[r] = acc;
    }
}

static double silu(double g) { return g / (1.0 + exp(-g)); }

/* gate -> up -> silu(gate)*up -> down -> acc += weight*y.
 * Reference: csrc/core/wisp_engine.c:1535-1561 and :677-690. */
void orc_expert_ffn(const OrcExpert* e, int gs, const double* x, double* acc,
                    double weight) {
    const int inter = e->mat[0].rows, hidden = e->mat[2].rows;
    double* g = (double*)malloc(sizeof(double) * (size_t)inter);
    double* u = (double*)malloc(sizeof(double) * (size_t)inter);
    double* y = (double*)malloc(sizeof(double) * (size_t)hidden);
    orc_gemv_int4(&e->mat[0], gs, x, g);
    orc_gemv_int4(&e->mat[1], gs, x, u);
    for (int i = 0; i < inter; i++) g[i] = silu(g[i]) * u[i];
    orc_gemv_int4(&e->mat[2], gs, g, y);
    for (int m = 0; m < hidden; m++) acc[m] += weight * y[m];
    free(g);
    free(u);
    free(y);
}

static double wval(const void* W, int wtype, size_t i) {
    if (wtype == 0) return ((const float*)W)[i];
    if (wtype == 1) return orc_f16_to_f32(((const uint16_t*)W)[i]);
    return orc_bf16_to_f32(((const uint16_t*)W)[i]);
}

/* Reference: csrc/cuda/router.cu:29-60 (GEMV + bias) and the CPU twin's
 * cpu_gemv_f16 + bias at csrc/core/wisp_engine.c:786-790. */
void orc_router_logits(const void* W, int wtype, const double* bias,
                       const double* x, int T, int E, int M, double* logits) {
    int t;
#pragma omp parallel for schedule(static)
    for (t = 0; t < T; t++) {
        const double* xt = x + (size_t)t * M;
        for (int e = 0; e < E; e++) {
            double acc = 0.0;
            for (int m = 0; m < M; m++)
                acc += wval(W, wtype, (size_t)e * M + m) * xt[m];
            logits[(size_t)t * E + e] = acc + (bias ? bias[e] : 0.0);
        }
    }
}

/* k rounds of "best untaken value, strictly greater wins" -- the lower index
 * keeps a tie. Returns the value of the next-best untaken entry (or -inf). */
static double argmax_rounds(const double* v, const char* allowed, int n, int k,
                            int* idx, double* val) {
    char* taken = (char*)calloc((size_t)n, 1);
    for (int r = 0; r < k; r++) {
        int best = -1;
        double bv = -INFINITY;
        for (int e = 0; e < n; e++) {
            if (taken[e] || (allowed && !allowed[e])) continue;
            if (best < 0 || v[e] > bv) {
                bv = v[e];
                best = e;
            }
        }
        idx[r] = best;
        val[r] = bv;
        if (best >= 0) taken[best] = 1;
    }
    double next = -INFINITY;
    for (int e = 0; e < n; e++)
        if (!taken[e] && (!allowed || allowed[e]) && v[e] > next) next = v[e];
    free(taken);
    return next;
}

/* Reference: csrc/core/wisp_engine.c:782-818 and csrc/cuda/router.cu:67-138.
 * margin is the logit gap between the k-th pick and the best non-pick. */
void orc_topk_softmax(const double* logits, int E, int k, int* idx, double* w,
                      double* margin) {
    double mx = -INFINITY;
    for (int e = 0; e < E; e++)
        if (logits[e] > mx) mx = logits[e];
    double* p = (double*)malloc(sizeof(double) * (size_t)E);
    double den = 0.0;
    for (int e = 0; e < E; e++) {
        p[e] = exp(logits[e] - mx);
        den += p[e];
    }
    for (int e = 0; e < E; e++) p[e] /= den;
    double* lv = (double*)malloc(sizeof(double) * (size_t)k);
    double nextl = argmax_rounds(logits, NULL, E, k, idx, lv);
    double wsum = 0.0;
    for (int r = 0; r < k; r++) {
        w[r] = idx[r] >= 0 ? p[idx[r]] : 0.0;
        wsum += w[r];
    }
    if (wsum > 0.0)
        for (int r = 0; r < k; r++) w[r] /= wsum;
    if (margin) *margin = (k < E) ? lv[k - 1] - nextl : INFINITY;
    free(lv);
    free(p);
}

void orc_topk_sigmoid_grouped(const double* logits, int E, int n_groups,
                              int topk_groups, int k, double scaling, int* idx,
                              double* w, double* margin) {
    const int gsz = E / n_groups;
    double* s = (double*)malloc(sizeof(double) * (size_t)E);
    double* gscore = (double*)malloc(sizeof(double) * (size_t)n_groups);
    for (int e = 0; e < E; e++) s[e] = 1.0 / (1.0 + exp(-logits[e]));
    for (int g = 0; g < n_groups; g++) {
        double a = -INFINITY, b = -INFINITY; /* top-2 of the group */
        for (int j = 0; j < gsz; j++) {
            double v = s[g * gsz + j];
            if (v > a) {
                b = a;
                a = v;
            } else if (v > b) {
                b = v;
            }
        }
        gscore[g] = a + (gsz > 1 ? b : 0.0);
    }
    int* gidx = (int*)malloc(sizeof(int) * (size_t)topk_groups);
    double* gval = (double*)malloc(sizeof(double) * (size_t)topk_groups);
    double gnext = argmax_rounds(gscore, NULL, n_groups, topk_groups, gidx, gval);
    char* allowed = (char*)calloc((size_t)E, 1);
    for (int r = 0; r < topk_groups; r++)
        for (int j = 0; j < gsz; j++) allowed[gidx[r] * gsz + j] = 1;
    double* sv = (double*)malloc(sizeof(double) * (size_t)k);
    double snext = argmax_rounds(s, allowed, E, k, idx, sv);
    double ssum = 0.0;
    for (int r = 0; r < k; r++) ssum += sv[r];
    for (int r = 0; r < k; r++) w[r] = sv[r] / ssum * scaling;
    if (margin) {
        double mg = (topk_groups < n_groups) ? gval[topk_groups - 1] - gnext
                                             : INFINITY;
        double me = sv[k - 1] - snext;
        *margin = mg < me ? mg : me;
    }
    free(sv);
    free(allowed);
    free(gval);
    free(gidx);
    free(gscore);
    free(s);
}

/* Reference: the per-token composition of run_moe's CPU branch,
 * csrc/core/wisp_engine.c:1563-1645 (shared expert with weight 1.0, then
 * each selected routed expert with its renormalised weight). */
void orc_moe_tokens(int M, int gs, const double* x, int k, const int* idx,
                    const double* w, const OrcExpert* experts,
                    const OrcExpert* shared, const int* tok, int ntok,
                    double* out) {
    int j;
#pragma omp parallel for schedule(dynamic, 1)
    for (j = 0; j < ntok; j++) {
        const int t = tok[j];
        const double* xt = x + (size_t)t * M;
        double* o = out + (size_t)j * M;
        for (int m = 0; m < M; m++) o[m] = 0.0;
        if (shared) orc_expert_ffn(shared, gs, xt, o, 1.0);
        for (int r = 0; r < k; r++) {
            int e = idx[(size_t)t * k + r];
            if (e < 0) continue;
            orc_expert_ffn(&experts[e], gs, xt, o, w[(size_t)t * k + r]);
        }
    }
}
