/*
 * oracle.c -- CPU fp64 restatement of the reference's attention and Gated
 * DeltaNet math.  TEST INFRASTRUCTURE ONLY (see oracle.h): the product
 * library never links it and never falls back to it.
 *
 * Threads: a small pthread parallel-for over independent work items
 * ((b, h, row block) for attention, (b, h) for GDN).  Results do not depend
 * on the thread count: every output element is produced by one item.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* parallel-for                                                              */
/* ------------------------------------------------------------------------ */
typedef void (*item_fn)(void* ctx, long item, void* scratch);

typedef struct {
    item_fn fn;
    void* ctx;
    long n_items;
    long next;
    size_t scratch_bytes;
    pthread_mutex_t mu;
    int failed;
} pfor_t;

static void* pfor_worker(void* arg) {
    pfor_t* p = (pfor_t*)arg;
    void* scratch = p->scratch_bytes ? malloc(p->scratch_bytes) : NULL;
    if (p->scratch_bytes && !scratch) {
        pthread_mutex_lock(&p->mu);
        p->failed = 1;
        pthread_mutex_unlock(&p->mu);
        return NULL;
    }
    for (;;) {
        pthread_mutex_lock(&p->mu);
        long it = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (it >= p->n_items) break;
        p->fn(p->ctx, it, scratch);
    }
    free(scratch);
    return NULL;
}

int orc_default_threads(void) {
    cpu_set_t set;
    if (sched_getaffinity(0, sizeof(set), &set) == 0) {
        int n = CPU_COUNT(&set);
        if (n > 0) return n;
    }
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static int parallel_for(long n_items, int nthreads, size_t scratch_bytes,
                        item_fn fn, void* ctx) {
    if (nthreads <= 0) nthreads = orc_default_threads();
    if (nthreads > n_items) nthreads = (int)(n_items > 0 ? n_items : 1);
    pfor_t p;
    p.fn = fn;
    p.ctx = ctx;
    p.n_items = n_items;
    p.next = 0;
    p.scratch_bytes = scratch_bytes;
    p.failed = 0;
    pthread_mutex_init(&p.mu, NULL);
    if (nthreads == 1) {
        pfor_worker(&p);
    } else {
        pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
        if (!th) return -1;
        for (int i = 0; i < nthreads; ++i) pthread_create(&th[i], NULL, pfor_worker, &p);
        for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
        free(th);
    }
    pthread_mutex_destroy(&p.mu);
    return p.failed ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Attention: naive_attn_kernel, src/attn_sm75.cu:55-94.                     */
/* Same two-pass math (row max, then softmax-weighted V sum); the scores are */
/* computed once per row instead of once per (row, d), which changes only    */
/* the cost, not the result.                                                 */
/* ------------------------------------------------------------------------ */
enum { ATTN_ROWS_PER_ITEM = 16 };

typedef struct {
    const float *Q, *K, *V;
    double* O;
    int B, Hq, Hkv, Sq, Skv, D, causal, nrows;
    const int* rows;
    double scale;
    long row_blocks;
} attn_ctx;

static void attn_item(void* vctx, long item, void* scratch) {
    const attn_ctx* c = (const attn_ctx*)vctx;
    const long bh = item / c->row_blocks;
    const int rb = (int)(item % c->row_blocks);
    const int b = (int)(bh / c->Hq);
    const int h = (int)(bh % c->Hq);
    const int hkv = h / (c->Hq / c->Hkv);
    const int D = c->D;
    const float* Kh = c->K + ((size_t)b * c->Hkv + hkv) * (size_t)c->Skv * D;
    const float* Vh = c->V + ((size_t)b * c->Hkv + hkv) * (size_t)c->Skv * D;
    const float* Qh = c->Q + ((size_t)b * c->Hq + h) * (size_t)c->Sq * D;
    const int n_out = c->rows ? c->nrows : c->Sq;
    double* Oh = c->O + ((size_t)b * c->Hq + h) * (size_t)n_out * D;
    double* s = (double*)scratch;            /* [Skv] scores */
    double* acc = s + c->Skv;                /* [D]          */

    const int r0 = rb * ATTN_ROWS_PER_ITEM;
    int r1 = r0 + ATTN_ROWS_PER_ITEM;
    if (r1 > n_out) r1 = n_out;
    for (int r = r0; r < r1; ++r) {
        const int qi = c->rows ? c->rows[r] : r;
        const float* qrow = Qh + (size_t)qi * D;
        int nvis = c->Skv;
        if (c->causal) {
            long lim = (long)qi + (c->Skv - c->Sq) + 1; /* keys [0, lim) visible */
            if (lim < 0) lim = 0;
            if (lim < nvis) nvis = (int)lim;
        }
        double* orow = Oh + (size_t)r * D;
        if (nvis <= 0) {
            for (int d = 0; d < D; ++d) orow[d] = 0.0;
            continue;
        }
        double m = -INFINITY;
        for (int j = 0; j < nvis; ++j) {
            const float* krow = Kh + (size_t)j * D;
            double dot = 0.0;
            for (int d = 0; d < D; ++d) dot += (double)qrow[d] * (double)krow[d];
            s[j] = dot * c->scale;
            if (s[j] > m) m = s[j];
        }
        double l = 0.0;
        for (int d = 0; d < D; ++d) acc[d] = 0.0;
        for (int j = 0; j < nvis; ++j) {
            const double p = exp(s[j] - m);
            l += p;
            const float* vrow = Vh + (size_t)j * D;
            for (int d = 0; d < D; ++d) acc[d] += p * (double)vrow[d];
        }
        for (int d = 0; d < D; ++d) orow[d] = acc[d] / l;
    }
}

int orc_attn_fwd(const float* Q, const float* K, const float* V, double* O,
                 int B, int Hq, int Hkv, int Sq, int Skv, int D, double scale,
                 int causal, const int* rows, int nrows, int nthreads) {
    if (!Q || !K || !V || !O || B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 ||
        Skv <= 0 || D <= 0 || Hq % Hkv != 0)
        return -1;
    if (rows) {
        if (nrows <= 0) return -1;
        for (int r = 0; r < nrows; ++r)
            if (rows[r] < 0 || rows[r] >= Sq) return -1;
    }
    attn_ctx c;
    c.Q = Q; c.K = K; c.V = V; c.O = O;
    c.B = B; c.Hq = Hq; c.Hkv = Hkv; c.Sq = Sq; c.Skv = Skv; c.D = D;
    c.causal = causal; c.rows = rows; c.nrows = nrows; c.scale = scale;
    const int n_out = rows ? nrows : Sq;
    c.row_blocks = (n_out + ATTN_ROWS_PER_ITEM - 1) / ATTN_ROWS_PER_ITEM;
    const long items = (long)B * Hq * c.row_blocks;
    return parallel_for(items, nthreads, sizeof(double) * ((size_t)Skv + D), attn_item, &c);
}

/* ------------------------------------------------------------------------ */
/* GDN common                                                                */
/* ------------------------------------------------------------------------ */
typedef struct {
    const float *q, *k, *v, *g_log, *beta;
    double *state, *out;
    int B, T, Hqk, Hv, dk, dv, head_map, C;
    double scale;
    int refsolve;
} gdn_ctx;

static int gdn_qk_head(const gdn_ctx* c, int h) {
    return c->head_map == 0 ? h % c->Hqk : h / (c->Hv / c->Hqk);
}

static int gdn_check(const float* q, const float* k, const float* v,
                     const float* g_log, const float* beta, const double* state,
                     const double* out, int B, int T, int Hqk, int Hv, int dk,
                     int dv, int head_map) {
    if (!q || !k || !v || !g_log || !beta || !state || !out) return -1;
    if (B <= 0 || T < 0 || Hqk <= 0 || Hv <= 0 || dk <= 0 || dv <= 0) return -1;
    if (head_map != 0 && head_map != 1) return -1;
    if (head_map == 1 && Hv % Hqk != 0) return -1;
    return 0;
}

/* src/gdn_sm75.cu:1078-1106, one (b, h) per item. */
static void gdn_rec_item(void* vctx, long item, void* scratch) {
    (void)scratch;
    const gdn_ctx* c = (const gdn_ctx*)vctx;
    const int b = (int)(item / c->Hv);
    const int h = (int)(item % c->Hv);
    const int hq = gdn_qk_head(c, h);
    const int dk = c->dk, dv = c->dv;
    double* S = c->state + ((size_t)b * c->Hv + h) * (size_t)dv * dk;
    for (int t = 0; t < c->T; ++t) {
        const size_t bt = (size_t)b * c->T + t;
        const float* qt = c->q + (bt * c->Hqk + hq) * dk;
        const float* kt = c->k + (bt * c->Hqk + hq) * dk;
        const float* vt = c->v + (bt * c->Hv + h) * dv;
        const double g = exp((double)c->g_log[bt * c->Hv + h]);
        const double be = (double)c->beta[bt * c->Hv + h];
        double* ot = c->out + (bt * c->Hv + h) * dv;
        for (int col = 0; col < dv; ++col) {
            double* Sc = S + (size_t)col * dk;
            double kv = 0.0;
            for (int i = 0; i < dk; ++i) kv += Sc[i] * (double)kt[i];
            const double d = ((double)vt[col] - g * kv) * be;
            double o = 0.0;
            for (int i = 0; i < dk; ++i) {
                Sc[i] = g * Sc[i] + (double)kt[i] * d;
                o += Sc[i] * (double)qt[i];
            }
            ot[col] = o * c->scale;
        }
    }
}

int orc_gdn_recurrent(const float* q, const float* k, const float* v,
                      const float* g_log, const float* beta, double* state,
                      double* out, int B, int T, int Hqk, int Hv, int dk, int dv,
                      int head_map, double scale, int nthreads) {
    if (gdn_check(q, k, v, g_log, beta, state, out, B, T, Hqk, Hv, dk, dv, head_map))
        return -1;
    gdn_ctx c;
    memset(&c, 0, sizeof(c));
    c.q = q; c.k = k; c.v = v; c.g_log = g_log; c.beta = beta;
    c.state = state; c.out = out;
    c.B = B; c.T = T; c.Hqk = Hqk; c.Hv = Hv; c.dk = dk; c.dv = dv;
    c.head_map = head_map; c.scale = scale;
    return parallel_for((long)B * Hv, nthreads, 0, gdn_rec_item, &c);
}

/* ------------------------------------------------------------------------ */
/* GDN chunked (WY/UT) algebra, src/gdn_sm75.cu:1109-1244, generic chunk C.  */
/*                                                                           */
/* Row-major token notation used here (the reference stores the same C x C  */
/* matrices column-major, A[i + j*CS]):                                      */
/*   gcs[t] = sum_{s<=t} g_log[s]                                            */
/*   A[t][s] = beta_t (k_t.k_s) e^{gcs_t - gcs_s}, s < t   (strictly lower)  */
/*   Tm = (I + A)^-1 by forward substitution                                 */
/*   U = Tm diag(beta) V,  W = Tm diag(beta e^{gcs}) K                       */
/*   Vn = U - W S^T                       (the chunk's delta-rule residuals) */
/*   o_t = scale (e^{gcs_t} S q_t + sum_{s<=t} (q_t.k_s) e^{gcs_t-gcs_s} Vn_s)*/
/*   S  <- e^{gcs_last} S + sum_t e^{gcs_last - gcs_t} Vn_t k_t^T            */
/* Padded tokens past T carry g_log = 0, beta = 0 and zero q/k/v, as in the  */
/* reference (src/gdn_sm75.cu:1125-1137).                                    */
/* ------------------------------------------------------------------------ */
static void gdn_chunk_item(void* vctx, long item, void* scratch) {
    const gdn_ctx* c = (const gdn_ctx*)vctx;
    const int b = (int)(item / c->Hv);
    const int h = (int)(item % c->Hv);
    const int hq = gdn_qk_head(c, h);
    const int dk = c->dk, dv = c->dv, C = c->C;
    double* S = c->state + ((size_t)b * c->Hv + h) * (size_t)dv * dk;

    double* qc = (double*)scratch;           /* [C][dk] */
    double* kc = qc + (size_t)C * dk;        /* [C][dk] */
    double* vc = kc + (size_t)C * dk;        /* [C][dv] */
    double* gcs = vc + (size_t)C * dv;       /* [C]     */
    double* bt = gcs + C;                    /* [C]     */
    double* A = bt + C;                      /* [C][C]  */
    double* Tm = A + (size_t)C * C;          /* [C][C]  */
    double* U = Tm + (size_t)C * C;          /* [C][dv] */
    double* W = U + (size_t)C * dv;          /* [C][dk] */
    double* Vn = W + (size_t)C * dk;         /* [C][dv] */
    double* X = Vn + (size_t)C * dv;         /* [C][C] (refsolve) */

    const int nch = (c->T + C - 1) / C;
    for (int ch = 0; ch < nch; ++ch) {
        const int t0 = ch * C;
        double acc = 0.0;
        for (int t = 0; t < C; ++t) {
            const int tt = t0 + t;
            double gl = 0.0, be = 0.0;
            if (tt < c->T) {
                const size_t bt_i = (size_t)b * c->T + tt;
                const float* qt = c->q + (bt_i * c->Hqk + hq) * dk;
                const float* kt = c->k + (bt_i * c->Hqk + hq) * dk;
                const float* vt = c->v + (bt_i * c->Hv + h) * dv;
                for (int i = 0; i < dk; ++i) {
                    qc[(size_t)t * dk + i] = qt[i];
                    kc[(size_t)t * dk + i] = kt[i];
                }
                for (int i = 0; i < dv; ++i) vc[(size_t)t * dv + i] = vt[i];
                gl = c->g_log[bt_i * c->Hv + h];
                be = c->beta[bt_i * c->Hv + h];
            } else {
                for (int i = 0; i < dk; ++i) qc[(size_t)t * dk + i] = kc[(size_t)t * dk + i] = 0.0;
                for (int i = 0; i < dv; ++i) vc[(size_t)t * dv + i] = 0.0;
            }
            acc += gl;
            gcs[t] = acc;
            bt[t] = be;
        }
        /* A, strictly lower */
        for (int t = 0; t < C; ++t)
            for (int s = 0; s < C; ++s) {
                double a = 0.0;
                if (s < t) {
                    double dot = 0.0;
                    for (int i = 0; i < dk; ++i) dot += kc[(size_t)t * dk + i] * kc[(size_t)s * dk + i];
                    a = bt[t] * dot * exp(gcs[t] - gcs[s]);
                }
                A[(size_t)t * C + s] = a;
            }
        if (!c->refsolve) {
            /* Tm = (I + A)^-1, forward substitution column by column */
            for (int col = 0; col < C; ++col)
                for (int t = 0; t < C; ++t) {
                    double x = (t == col) ? 1.0 : 0.0;
                    for (int s = col; s < t; ++s) x -= A[(size_t)t * C + s] * Tm[(size_t)s * C + col];
                    Tm[(size_t)t * C + col] = (t < col) ? 0.0 : x;
                }
        } else {
            /* The reference's loop (src/gdn_sm75.cu:1160-1180), stated in the
             * row-major notation above: with kb(i,j) = A[j][i] for i < j,
             *   X(r,cj) = -[r<cj] kb(r,cj) - sum_{p<r} kb(p,r) X(p,cj)
             *   attn(i,t) = X(i,t) + [i==t],  used as Tm[t][i] = attn(i,t). */
            for (int cj = 0; cj < C; ++cj)
                for (int r = 0; r < C; ++r) {
                    double sum = 0.0;
                    for (int p = 0; p < r; ++p) sum += A[(size_t)r * C + p] * X[(size_t)p * C + cj];
                    const double rhs = (r < cj) ? -A[(size_t)cj * C + r] : 0.0;
                    X[(size_t)r * C + cj] = rhs - sum;
                }
            for (int i = 0; i < C; ++i)
                for (int t = 0; t < C; ++t)
                    Tm[(size_t)t * C + i] = X[(size_t)i * C + t] + (i == t ? 1.0 : 0.0);
        }
        /* U = Tm diag(beta) V ; W = Tm diag(beta e^gcs) K */
        for (int t = 0; t < C; ++t) {
            for (int i = 0; i < dv; ++i) U[(size_t)t * dv + i] = 0.0;
            for (int i = 0; i < dk; ++i) W[(size_t)t * dk + i] = 0.0;
            for (int s = 0; s < C; ++s) {
                const double ts = Tm[(size_t)t * C + s];
                if (ts == 0.0) continue;
                const double fu = ts * bt[s];
                const double fw = fu * exp(gcs[s]);
                for (int i = 0; i < dv; ++i) U[(size_t)t * dv + i] += fu * vc[(size_t)s * dv + i];
                for (int i = 0; i < dk; ++i) W[(size_t)t * dk + i] += fw * kc[(size_t)s * dk + i];
            }
        }
        /* Vn = U - W S^T */
        for (int t = 0; t < C; ++t)
            for (int col = 0; col < dv; ++col) {
                const double* Sc = S + (size_t)col * dk;
                double ws = 0.0;
                for (int i = 0; i < dk; ++i) ws += W[(size_t)t * dk + i] * Sc[i];
                Vn[(size_t)t * dv + col] = U[(size_t)t * dv + col] - ws;
            }
        /* outputs */
        for (int t = 0; t < C; ++t) {
            const int tt = t0 + t;
            if (tt >= c->T) continue;
            const double eg = exp(gcs[t]);
            double* ot = c->out + (((size_t)b * c->T + tt) * c->Hv + h) * dv;
            for (int col = 0; col < dv; ++col) {
                const double* Sc = S + (size_t)col * dk;
                double sq = 0.0;
                for (int i = 0; i < dk; ++i) sq += Sc[i] * qc[(size_t)t * dk + i];
                double intra = 0.0;
                for (int s = 0; s <= t; ++s) {
                    double qk = 0.0;
                    for (int i = 0; i < dk; ++i) qk += qc[(size_t)t * dk + i] * kc[(size_t)s * dk + i];
                    intra += qk * exp(gcs[t] - gcs[s]) * Vn[(size_t)s * dv + col];
                }
                ot[col] = (eg * sq + intra) * c->scale;
            }
        }
        /* state */
        const double glast = gcs[C - 1];
        const double egl = exp(glast);
        for (int col = 0; col < dv; ++col) {
            double* Sc = S + (size_t)col * dk;
            for (int i = 0; i < dk; ++i) Sc[i] *= egl;
            for (int t = 0; t < C; ++t) {
                const double f = Vn[(size_t)t * dv + col] * exp(glast - gcs[t]);
                if (f == 0.0) continue;
                for (int i = 0; i < dk; ++i) Sc[i] += f * kc[(size_t)t * dk + i];
            }
        }
    }
}

static int gdn_chunked_common(const float* q, const float* k, const float* v,
                              const float* g_log, const float* beta, double* state,
                              double* out, int B, int T, int Hqk, int Hv, int dk,
                              int dv, int head_map, double scale, int C,
                              int nthreads, int refsolve) {
    if (gdn_check(q, k, v, g_log, beta, state, out, B, T, Hqk, Hv, dk, dv, head_map))
        return -1;
    if (C <= 0) return -1;
    gdn_ctx c;
    memset(&c, 0, sizeof(c));
    c.q = q; c.k = k; c.v = v; c.g_log = g_log; c.beta = beta;
    c.state = state; c.out = out;
    c.B = B; c.T = T; c.Hqk = Hqk; c.Hv = Hv; c.dk = dk; c.dv = dv;
    c.head_map = head_map; c.scale = scale; c.C = C; c.refsolve = refsolve;
    const size_t scratch = sizeof(double) *
        ((size_t)C * dk * 3 + (size_t)C * dv * 3 + 2 * (size_t)C + 3 * (size_t)C * C);
    return parallel_for((long)B * Hv, nthreads, scratch, gdn_chunk_item, &c);
}

int orc_gdn_chunked(const float* q, const float* k, const float* v,
                    const float* g_log, const float* beta, double* state,
                    double* out, int B, int T, int Hqk, int Hv, int dk, int dv,
                    int head_map, double scale, int C, int nthreads) {
    return gdn_chunked_common(q, k, v, g_log, beta, state, out, B, T, Hqk, Hv, dk,
                              dv, head_map, scale, C, nthreads, 0);
}

int orc_gdn_chunked_refsolve(const float* q, const float* k, const float* v,
                             const float* g_log, const float* beta, double* state,
                             double* out, int B, int T, int Hqk, int Hv, int dk,
                             int dv, int head_map, double scale, int C,
                             int nthreads) {
    return gdn_chunked_common(q, k, v, g_log, beta, state, out, B, T, Hqk, Hv, dk,
                              dv, head_map, scale, C, nthreads, 1);
}
