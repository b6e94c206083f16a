/*
 * CPU oracle for the fused sequence-loss path (CTC, RNN-T, TDT), forward + backward.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the parity tests, the
 * smoke check and the bench's CPU-baseline leg compare the CUDA path against.
 * Nothing in the shipped library links or calls it.
 *
 * It is a plain-C, double-precision restatement of the reference's maths:
 *   CTC   : src/asr/loss/csrc/ctc.cu:55-212 (alpha over the 2S+1 extended labels,
 *           beta fused with d loss / d logits); torch F.ctc_loss semantics.
 *   RNN-T : tests/loss/rnnt_reference.py:44-259 (dense joint, edge log-probs,
 *           alpha, beta, posterior gradients) with the kernel conventions of
 *           src/asr/loss/csrc/rnnt.cu:128-317 (NEG=-1e30 finite sentinel,
 *           terminal blank).
 *   TDT   : tests/loss/tdt_reference.py:50-356 with src/asr/loss/csrc/tdt.cu:142-500
 *           (durations, sigma under-normalisation, exact landing at
 *           (in_lens, tgt_lens), blank never takes duration 0, the d=0 token
 *           chain uses the first zero duration only).
 *
 * Only valid lattice nodes (t < in_lens[b], u <= tgt_lens[b]) are visited;
 * padded nodes carry exactly zero gradient in the reference, so they stay zero
 * here. Utterances are independent and are spread over pthreads; the weight
 * gradients are accumulated per worker and summed at the end.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define NEG (-1e30)

/* log(exp(a)+exp(b)), -inf safe (ctc.cu:38-43, rnnt.cu:44-49 semantics). */
static double lae(double a, double b) {
    double m = a > b ? a : b;
    if (isinf(m) && m < 0) return -INFINITY;
    return m + log1p(exp(-fabs(a - b)));
}

/* ------------------------------------------------------------------ threading */

typedef void (*utt_fn)(void* ctx, int b, int worker);

typedef struct {
    utt_fn fn;
    void* ctx;
    int B;
    int next;
    pthread_mutex_t mu;
} pool_t;

typedef struct {
    pool_t* pool;
    int worker;
} worker_t;

static void* pool_main(void* p) {
    worker_t* w = (worker_t*)p;
    pool_t* pool = w->pool;
    for (;;) {
        pthread_mutex_lock(&pool->mu);
        int b = pool->next++;
        pthread_mutex_unlock(&pool->mu);
        if (b >= pool->B) break;
        pool->fn(pool->ctx, b, w->worker);
    }
    return NULL;
}

/* Runs fn(ctx, b, worker) for every b in [0, B) on nthreads workers. */
static void run_pool(utt_fn fn, void* ctx, int B, int nthreads) {
    if (nthreads <= 1 || B <= 1) {
        for (int b = 0; b < B; ++b) fn(ctx, b, 0);
        return;
    }
    pool_t pool;
    pool.fn = fn;
    pool.ctx = ctx;
    pool.B = B;
    pool.next = 0;
    pthread_mutex_init(&pool.mu, NULL);
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    worker_t* ws = (worker_t*)calloc((size_t)nthreads, sizeof(worker_t));
    for (int i = 0; i < nthreads; ++i) {
        ws[i].pool = &pool;
        ws[i].worker = i;
        pthread_create(&th[i], NULL, pool_main, &ws[i]);
    }
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    pthread_mutex_destroy(&pool.mu);
    free(th);
    free(ws);
}

/* ================================================================== CTC */

typedef struct {
    const float* log_probs; /* (B, T, V) */
    const int32_t* targets; /* (B, S) */
    const int32_t* in_lens;
    const int32_t* tgt_lens;
    const float* grad_loss; /* (B,) or NULL (backward skipped) */
    int B, T, V, S, zero_infinity;
    double* loss;        /* (B,) */
    double* grad_logits; /* (B, T, V) or NULL */
} ctc_ctx;

static void ctc_utt(void* vctx, int b, int worker) {
    (void)worker;
    ctc_ctx* c = (ctc_ctx*)vctx;
    const int T = c->T, V = c->V, S = c->S;
    const int Tb = c->in_lens[b];
    const int Sb = c->tgt_lens[b];
    const int L = 2 * Sb + 1;
    const float* lp = c->log_probs + (size_t)b * T * V;
    const int32_t* y = c->targets + (size_t)b * S;
    double* alpha = (double*)malloc(sizeof(double) * (size_t)Tb * L);
    double* beta = (double*)malloc(sizeof(double) * (size_t)Tb * L);
#define LBL(s) (((s) % 2 == 0) ? 0 : y[(s) / 2])
    /* alpha: ctc.cu:66-104 */
    for (int s = 0; s < L; ++s) alpha[s] = (s <= 1) ? (double)lp[LBL(s)] : -INFINITY;
    for (int t = 1; t < Tb; ++t) {
        for (int s = 0; s < L; ++s) {
            double acc = alpha[(size_t)(t - 1) * L + s];
            if (s > 0) acc = lae(acc, alpha[(size_t)(t - 1) * L + s - 1]);
            int skip = (s % 2 == 1) && (s / 2 > 0) && (y[s / 2] != y[s / 2 - 1]);
            if (skip) acc = lae(acc, alpha[(size_t)(t - 1) * L + s - 2]);
            alpha[(size_t)t * L + s] = acc + (double)lp[(size_t)t * V + LBL(s)];
        }
    }
    double logZ;
    if (L == 1)
        logZ = alpha[(size_t)(Tb - 1) * L];
    else
        logZ = lae(alpha[(size_t)(Tb - 1) * L + L - 2], alpha[(size_t)(Tb - 1) * L + L - 1]);
    double loss = -logZ;
    if (c->zero_infinity && !isfinite(loss)) loss = 0.0;
    c->loss[b] = loss;
    if (c->grad_logits) {
        double* g = c->grad_logits + (size_t)b * T * V;
        for (size_t i = 0; i < (size_t)T * V; ++i) g[i] = 0.0;
        if (!(c->zero_infinity && !isfinite(logZ))) {
            /* beta excludes the emission at t (ctc.cu:137-205) */
            for (int s = 0; s < L; ++s) beta[(size_t)(Tb - 1) * L + s] = -INFINITY;
            beta[(size_t)(Tb - 1) * L + L - 1] = 0.0;
            if (L >= 2) beta[(size_t)(Tb - 1) * L + L - 2] = 0.0;
            for (int t = Tb - 1; t > 0; --t) {
                for (int s = 0; s < L; ++s) {
                    double acc = beta[(size_t)t * L + s] + (double)lp[(size_t)t * V + LBL(s)];
                    if (s < L - 1) acc = lae(acc, beta[(size_t)t * L + s + 1] + (double)lp[(size_t)t * V + LBL(s + 1)]);
                    int skip = (s % 2 == 1) && (s / 2 < Sb - 1) && (y[s / 2] != y[s / 2 + 1]);
                    if (s < L - 2 && skip) acc = lae(acc, beta[(size_t)t * L + s + 2] + (double)lp[(size_t)t * V + LBL(s + 2)]);
                    beta[(size_t)(t - 1) * L + s] = acc;
                }
            }
            const double gl = (double)c->grad_loss[b];
            for (int t = 0; t < Tb; ++t) {
                double* gr = g + (size_t)t * V;
                for (int s = 0; s < L; ++s) gr[LBL(s)] += exp(alpha[(size_t)t * L + s] + beta[(size_t)t * L + s] - logZ);
                for (int v = 0; v < V; ++v) gr[v] = gl * (exp((double)lp[(size_t)t * V + v]) - gr[v]);
            }
        }
    }
#undef LBL
    free(alpha);
    free(beta);
}

/* Per-utterance CTC loss (-log Z, zero_infinity applied) and, when grad_logits is
 * non-NULL, d loss / d logits for log_probs = log_softmax(logits). */
void oracle_ctc(const float* log_probs, const int32_t* targets, const int32_t* in_lens, const int32_t* tgt_lens,
                const float* grad_loss, int B, int T, int V, int S, int zero_infinity, double* loss,
                double* grad_logits, int nthreads) {
    ctc_ctx c = {log_probs, targets, in_lens, tgt_lens, grad_loss, B, T, V, S, zero_infinity, loss, grad_logits};
    run_pool(ctc_utt, &c, B, nthreads);
}

/* ============================================================ transducers */

/* One context for RNN-T (n_dur == 0) and TDT (n_dur > 0). */
typedef struct {
    const float* enc;   /* (B, T, d) */
    const float* dec;   /* (B, U, d) */
    const float* W;     /* (V, d) */
    const float* W_dur; /* (n_dur, d) or NULL */
    const int32_t* targets;
    const int32_t* in_lens;
    const int32_t* tgt_lens;
    const int32_t* durations; /* (n_dur,) */
    const float* grad_loss;   /* (B,) or NULL */
    int B, T, U, V, d, S, n_dur, blank;
    double sigma;
    double* loss;     /* (B,) */
    double* log_prob; /* (B,) */
    double* d_enc;    /* (B, T, d) or NULL */
    double* d_dec;    /* (B, U, d) */
    double* dW_w;     /* (workers, V, d) per-worker partials */
    double* dWd_w;    /* (workers, n_dur, d) */
} tr_ctx;

/* Dense joint for one node: hidden = tanh(enc+dec) (rnnt_reference.py:54-58),
 * token log-softmax (and duration log-softmax for TDT, tdt_reference.py:62-66). */
static void joint_node(const tr_ctx* c, int b, int t, int u, double* h, double* lt, double* ld, double* lse_t,
                       double* lse_d) {
    const int d = c->d, V = c->V, Dn = c->n_dur;
    const float* e = c->enc + ((size_t)b * c->T + t) * d;
    const float* p = c->dec + ((size_t)b * c->U + u) * d;
    for (int k = 0; k < d; ++k) h[k] = tanh((double)e[k] + (double)p[k]);
    double m = -INFINITY;
    for (int v = 0; v < V; ++v) {
        const float* w = c->W + (size_t)v * d;
        double acc = 0.0;
        for (int k = 0; k < d; ++k) acc += h[k] * (double)w[k];
        lt[v] = acc;
        if (acc > m) m = acc;
    }
    double s = 0.0;
    for (int v = 0; v < V; ++v) s += exp(lt[v] - m);
    *lse_t = m + log(s);
    if (Dn > 0) {
        double md = -INFINITY;
        for (int j = 0; j < Dn; ++j) {
            const float* w = c->W_dur + (size_t)j * d;
            double acc = 0.0;
            for (int k = 0; k < d; ++k) acc += h[k] * (double)w[k];
            ld[j] = acc;
            if (acc > md) md = acc;
        }
        double sd = 0.0;
        for (int j = 0; j < Dn; ++j) sd += exp(ld[j] - md);
        *lse_d = md + log(sd);
    }
}

/* Per-utterance scratch shared by the row-parallel phases. */
typedef struct {
    tr_ctx* c;
    int b, Tb, Ub, zk;
    const int32_t* y;
    double *lpb, *lpy, *lpd, *alpha, *beta, logZ;
    double* dW_w;   /* (workers, V, d) */
    double* dWd_w;  /* (workers, n_dur, d) */
    double* ddec_w; /* (workers, Ub, d) */
} utt_t;

#define A(t, u) alpha[(size_t)(t) * Ub + (u)]
#define Bt(t, u) beta[(size_t)(t) * Ub + (u)]
#define NI(t, u) ((size_t)(t) * Ub + (u))

/* Phase 1 (parallel over frames): edge log-probs of row t (rnnt.cu:148-152, tdt.cu:162-187). */
static void edge_row(void* vu, int t, int worker) {
    (void)worker;
    utt_t* s = (utt_t*)vu;
    tr_ctx* c = s->c;
    const int Ub = s->Ub, Dn = c->n_dur, V = c->V;
    double* h = (double*)malloc(sizeof(double) * c->d);
    double* lt = (double*)malloc(sizeof(double) * V);
    double* ld = (double*)malloc(sizeof(double) * (Dn > 0 ? Dn : 1));
    for (int u = 0; u < Ub; ++u) {
        double lse_t, lse_d = 0.0;
        joint_node(c, s->b, t, u, h, lt, ld, &lse_t, &lse_d);
        const size_t n = NI(t, u);
        const int yy = (u < Ub - 1) ? s->y[u] : -1;
        s->lpb[n] = lt[c->blank] - lse_t - c->sigma;
        s->lpy[n] = (yy >= 0) ? lt[yy] - lse_t - c->sigma : NEG;
        for (int j = 0; j < Dn; ++j) s->lpd[n * Dn + j] = ld[j] - lse_d;
    }
    free(h);
    free(lt);
    free(ld);
}

/* Phase 2 (serial): alpha, beta, log Z. */
static void recursions(utt_t* s) {
    tr_ctx* c = s->c;
    const int Tb = s->Tb, Ub = s->Ub, Dn = c->n_dur, zk = s->zk;
    double *alpha = s->alpha, *beta = s->beta, *lpb = s->lpb, *lpy = s->lpy, *lpd = s->lpd;
    if (Dn == 0) {
        /* rnnt_reference.py:94-129 */
        for (int t = 0; t < Tb; ++t)
            for (int u = 0; u < Ub; ++u) {
                if (t == 0 && u == 0) {
                    A(0, 0) = 0.0;
                    continue;
                }
                double th = (t > 0) ? A(t - 1, u) + lpb[NI(t - 1, u)] : NEG;
                double tv = (u > 0) ? A(t, u - 1) + lpy[NI(t, u - 1)] : NEG;
                A(t, u) = lae(th, tv);
            }
        s->logZ = A(Tb - 1, Ub - 1) + lpb[NI(Tb - 1, Ub - 1)];
        /* rnnt_reference.py:132-178 */
        for (int t = Tb - 1; t >= 0; --t)
            for (int u = Ub - 1; u >= 0; --u) {
                const int is_term = (t == Tb - 1) && (u == Ub - 1);
                double bl = is_term ? lpb[NI(t, u)] : ((t < Tb - 1) ? lpb[NI(t, u)] + Bt(t + 1, u) : NEG);
                double lb = (u < Ub - 1) ? lpy[NI(t, u)] + Bt(t, u + 1) : NEG;
                Bt(t, u) = lae(bl, lb);
            }
        return;
    }
    /* tdt_reference.py:109-177 (alpha), tdt.cu:212-289 */
    for (int t = 0; t <= Tb; ++t)
        for (int u = 0; u < Ub; ++u) {
            double acc = (t == 0 && u == 0) ? 0.0 : NEG;
            for (int j = 0; j < Dn; ++j) {
                const int dd = c->durations[j];
                if (dd < 1) continue;
                const int src = t - dd;
                if (src < 0 || src >= Tb) continue;
                acc = lae(acc, A(src, u) + lpb[NI(src, u)] + lpd[NI(src, u) * Dn + j]);
                if (u >= 1) acc = lae(acc, A(src, u - 1) + lpy[NI(src, u - 1)] + lpd[NI(src, u - 1) * Dn + j]);
            }
            if (zk >= 0 && t < Tb && u >= 1) acc = lae(acc, A(t, u - 1) + lpy[NI(t, u - 1)] + lpd[NI(t, u - 1) * Dn + zk]);
            A(t, u) = acc;
        }
    s->logZ = A(Tb, Ub - 1);
    /* tdt_reference.py:180-248 (beta), tdt.cu:326-398 */
    for (int u = 0; u < Ub; ++u) Bt(Tb, u) = (u == Ub - 1) ? 0.0 : NEG;
    for (int t = Tb - 1; t >= 0; --t)
        for (int u = Ub - 1; u >= 0; --u) {
            double acc = NEG;
            for (int j = 0; j < Dn; ++j) {
                const int dd = c->durations[j];
                if (dd < 1) continue;
                const int nt = t + dd;
                if (nt > Tb) continue;
                acc = lae(acc, lpb[NI(t, u)] + lpd[NI(t, u) * Dn + j] + Bt(nt, u));
                if (u < Ub - 1) acc = lae(acc, lpy[NI(t, u)] + lpd[NI(t, u) * Dn + j] + Bt(nt, u + 1));
            }
            if (zk >= 0 && u < Ub - 1) acc = lae(acc, lpy[NI(t, u)] + lpd[NI(t, u) * Dn + zk] + Bt(t, u + 1));
            Bt(t, u) = acc;
        }
}

/* Phase 3 (parallel over frames): posteriors and gradients of row t. d_enc row t
 * belongs to this call alone; d_dec and the weight gradients go to per-worker partials. */
static void grad_row(void* vu, int t, int worker) {
    utt_t* s = (utt_t*)vu;
    tr_ctx* c = s->c;
    const int d = c->d, V = c->V, Dn = c->n_dur, Tb = s->Tb, Ub = s->Ub;
    const int tdt = Dn > 0;
    const double logZ = s->logZ;
    const double gl = (double)c->grad_loss[s->b];
    double *alpha = s->alpha, *beta = s->beta, *lpb = s->lpb, *lpy = s->lpy, *lpd = s->lpd;
    double* h = (double*)malloc(sizeof(double) * d);
    double* lt = (double*)malloc(sizeof(double) * V);
    double* ld = (double*)malloc(sizeof(double) * (Dn > 0 ? Dn : 1));
    double* gt = (double*)malloc(sizeof(double) * V);
    double* gh = (double*)malloc(sizeof(double) * d);
    double* gb = (double*)malloc(sizeof(double) * (Dn > 0 ? Dn : 1));
    double* gk = (double*)malloc(sizeof(double) * (Dn > 0 ? Dn : 1));
    double* dW = s->dW_w + (size_t)worker * V * d;
    double* dWd = tdt ? s->dWd_w + (size_t)worker * Dn * d : NULL;
    double* ddec = s->ddec_w + (size_t)worker * Ub * d;
    double* de = c->d_enc + ((size_t)s->b * c->T + t) * d;
    for (int u = 0; u < Ub; ++u) {
        const size_t n = NI(t, u);
        const double a = A(t, u);
        double bp = 0.0, tp = 0.0;
        if (!tdt) {
            /* rnnt.cu:286-303, rnnt_reference.py:223-235 */
            const int is_term = (t == Tb - 1) && (u == Ub - 1);
            if (is_term)
                bp = exp(a + lpb[n] - logZ);
            else if (t < Tb - 1)
                bp = exp(a + lpb[n] + Bt(t + 1, u) - logZ);
            if (u < Ub - 1) tp = exp(a + lpy[n] + Bt(t, u + 1) - logZ);
        } else {
            /* tdt.cu:400-426, tdt_reference.py:302-325 */
            for (int j = 0; j < Dn; ++j) {
                const int dd = c->durations[j];
                const int nt = t + dd;
                double g_b = 0.0, g_t = 0.0;
                if (nt <= Tb) {
                    if (dd >= 1) g_b = exp(a + lpb[n] + lpd[n * Dn + j] + Bt(nt, u) - logZ);
                    if (u < Ub - 1) g_t = exp(a + lpy[n] + lpd[n * Dn + j] + Bt(nt, u + 1) - logZ);
                }
                bp += g_b;
                tp += g_t;
                gb[j] = -(g_b + g_t); /* d loss / d log_P_dur[j] */
            }
        }
        if (bp == 0.0 && tp == 0.0) continue; /* every gradient of this node is zero */
        double lse_t, lse_d = 0.0;
        joint_node(c, s->b, t, u, h, lt, ld, &lse_t, &lse_d);
        const int yy = (u < Ub - 1) ? s->y[u] : -1;
        /* token head: g = gl*(softmax*(bp+tp) - bp[v=blank] - tp[v=y]) (rnnt.cu:189-194) */
        for (int v = 0; v < V; ++v) {
            double g = gl * exp(lt[v] - lse_t) * (bp + tp);
            if (v == c->blank) g -= gl * bp;
            if (v == yy) g -= gl * tp;
            gt[v] = g;
        }
        /* duration head: g = gl*(g_in - softmax*sum(g_in)) (tdt.cu:499) */
        if (tdt) {
            double gsum = 0.0;
            for (int j = 0; j < Dn; ++j) gsum += gb[j];
            for (int j = 0; j < Dn; ++j) gk[j] = gl * (gb[j] - exp(ld[j] - lse_d) * gsum);
        }
        for (int k = 0; k < d; ++k) gh[k] = 0.0;
        for (int v = 0; v < V; ++v) {
            const double g = gt[v];
            if (g == 0.0) continue;
            const float* w = c->W + (size_t)v * d;
            double* dw = dW + (size_t)v * d;
            for (int k = 0; k < d; ++k) {
                gh[k] += g * (double)w[k];
                dw[k] += g * h[k];
            }
        }
        for (int j = 0; j < Dn; ++j) {
            const double g = gk[j];
            const float* w = c->W_dur + (size_t)j * d;
            double* dw = dWd + (size_t)j * d;
            for (int k = 0; k < d; ++k) {
                gh[k] += g * (double)w[k];
                dw[k] += g * h[k];
            }
        }
        double* dd2 = ddec + (size_t)u * d;
        for (int k = 0; k < d; ++k) {
            const double gp = gh[k] * (1.0 - h[k] * h[k]);
            de[k] += gp;
            dd2[k] += gp;
        }
    }
    free(h);
    free(lt);
    free(ld);
    free(gt);
    free(gh);
    free(gb);
    free(gk);
}

#undef A
#undef Bt
#undef NI

/* Utterances run one after another; inside an utterance the joint network and
 * the gradients are spread over `workers` threads by frame. */
static void run_transducer(tr_ctx* c, double* dW, double* dW_dur, int nthreads) {
    const int workers = nthreads < 1 ? 1 : nthreads;
    const int grads = c->d_enc != NULL;
    double* dW_w = NULL;
    double* dWd_w = NULL;
    if (grads) {
        memset(c->d_enc, 0, sizeof(double) * (size_t)c->B * c->T * c->d);
        memset(c->d_dec, 0, sizeof(double) * (size_t)c->B * c->U * c->d);
        dW_w = (double*)calloc((size_t)workers * c->V * c->d, sizeof(double));
        dWd_w = c->n_dur > 0 ? (double*)calloc((size_t)workers * c->n_dur * c->d, sizeof(double)) : NULL;
    }
    for (int b = 0; b < c->B; ++b) {
        utt_t s;
        memset(&s, 0, sizeof(s));
        s.c = c;
        s.b = b;
        s.Tb = c->in_lens[b];
        s.Ub = c->tgt_lens[b] + 1;
        s.y = c->targets + (size_t)b * c->S;
        s.zk = -1;
        for (int j = 0; j < c->n_dur; ++j)
            if (c->durations[j] == 0) {
                s.zk = j; /* first zero duration (tdt_reference.py:134-135) */
                break;
            }
        const size_t nn = (size_t)s.Tb * s.Ub;
        const int TR = c->n_dur > 0 ? s.Tb + 1 : s.Tb; /* TDT uses the (T_b+1)-frame grid */
        s.lpb = (double*)malloc(sizeof(double) * nn);
        s.lpy = (double*)malloc(sizeof(double) * nn);
        s.lpd = c->n_dur > 0 ? (double*)malloc(sizeof(double) * nn * c->n_dur) : NULL;
        s.alpha = (double*)malloc(sizeof(double) * (size_t)TR * s.Ub);
        s.beta = (double*)malloc(sizeof(double) * (size_t)TR * s.Ub);
        run_pool(edge_row, &s, s.Tb, workers);
        recursions(&s);
        c->log_prob[b] = s.logZ;
        c->loss[b] = -s.logZ;
        if (grads) {
            s.dW_w = dW_w;
            s.dWd_w = dWd_w;
            s.ddec_w = (double*)calloc((size_t)workers * s.Ub * c->d, sizeof(double));
            run_pool(grad_row, &s, s.Tb, workers);
            double* dd = c->d_dec + (size_t)b * c->U * c->d;
            for (int w = 0; w < workers; ++w)
                for (size_t i = 0; i < (size_t)s.Ub * c->d; ++i) dd[i] += s.ddec_w[(size_t)w * s.Ub * c->d + i];
            free(s.ddec_w);
        }
        free(s.lpb);
        free(s.lpy);
        free(s.lpd);
        free(s.alpha);
        free(s.beta);
    }
    if (grads) {
        const size_t nw = (size_t)c->V * c->d;
        for (size_t i = 0; i < nw; ++i) {
            double acc = 0.0;
            for (int w = 0; w < workers; ++w) acc += dW_w[(size_t)w * nw + i];
            dW[i] = acc;
        }
        if (c->n_dur > 0) {
            const size_t nd = (size_t)c->n_dur * c->d;
            for (size_t i = 0; i < nd; ++i) {
                double acc = 0.0;
                for (int w = 0; w < workers; ++w) acc += dWd_w[(size_t)w * nd + i];
                dW_dur[i] = acc;
            }
        }
        free(dW_w);
        free(dWd_w);
    }
}

/* RNN-T: loss = -log P(y|x) and log_prob per utterance; with grad_loss non-NULL
 * also d_enc (B,T,d), d_dec (B,U,d), dW (V,d). */
void oracle_rnnt(const float* enc, const float* dec, const float* W, const int32_t* targets, const int32_t* in_lens,
                 const int32_t* tgt_lens, const float* grad_loss, int B, int T, int U, int V, int d, int S, int blank,
                 double* loss, double* log_prob, double* d_enc, double* d_dec, double* dW, int nthreads) {
    tr_ctx c;
    memset(&c, 0, sizeof(c));
    c.enc = enc;
    c.dec = dec;
    c.W = W;
    c.targets = targets;
    c.in_lens = in_lens;
    c.tgt_lens = tgt_lens;
    c.grad_loss = grad_loss;
    c.B = B;
    c.T = T;
    c.U = U;
    c.V = V;
    c.d = d;
    c.S = S;
    c.blank = blank;
    c.loss = loss;
    c.log_prob = log_prob;
    c.d_enc = grad_loss ? d_enc : NULL;
    c.d_dec = d_dec;
    run_transducer(&c, dW, NULL, nthreads);
}

/* TDT: as oracle_rnnt plus the duration head (W_dur, durations) and sigma. */
void oracle_tdt(const float* enc, const float* dec, const float* W, const float* W_dur, const int32_t* targets,
                const int32_t* in_lens, const int32_t* tgt_lens, const int32_t* durations, int n_dur, double sigma,
                const float* grad_loss, int B, int T, int U, int V, int d, int S, int blank, double* loss,
                double* log_prob, double* d_enc, double* d_dec, double* dW, double* dW_dur, int nthreads) {
    tr_ctx c;
    memset(&c, 0, sizeof(c));
    c.enc = enc;
    c.dec = dec;
    c.W = W;
    c.W_dur = W_dur;
    c.targets = targets;
    c.in_lens = in_lens;
    c.tgt_lens = tgt_lens;
    c.durations = durations;
    c.grad_loss = grad_loss;
    c.B = B;
    c.T = T;
    c.U = U;
    c.V = V;
    c.d = d;
    c.S = S;
    c.n_dur = n_dur;
    c.blank = blank;
    c.sigma = sigma;
    c.loss = loss;
    c.log_prob = log_prob;
    c.d_enc = grad_loss ? d_enc : NULL;
    c.d_dec = d_dec;
    run_transducer(&c, dW, dW_dur, nthreads);
}
