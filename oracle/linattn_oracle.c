/*
 * ORACLE — test infrastructure only. Nothing in the product links or calls
 * this file; only the tests, the smoke check and the CPU-baseline leg of
 * bench.py load it, and only as the checker.
 *
 * A float64 CPU restatement of the reference's causal ELU+1 linear-attention
 * scan, forward and backward, one (batch, head) sequence at a time:
 *
 *   phi(x)  = x + 1 (x > 0) else exp(x)
 *   S_t     = gamma_t * S_{t-1} + phi(k_t) v_t^T          (d x e)
 *   z_t     = gamma_t * z_{t-1} + phi(k_t)                 (d)
 *   unnormalised: o_t = phi(q_t)^T S_t
 *   normalised:   o_t = (s phi(q_t))^T S_t / max((s phi(q_t))^T z_t, clamp)
 *
 * Reference behaviour restated here (paths relative to the reference tree):
 *   - feature map and its derivative: python/subq_audio/autograd.py:15-28,
 *     src/kernels/attention_backward.cpp:22-32.
 *   - unnormalised engine recurrence with a scalar decay and the subnormal
 *     flush of the state: src/kernels/attention_forward.cpp:42-58,153-169,
 *     include/kernels.hpp:21-26.
 *   - normalised scan with D^-1/2 query scale, running denominator, clamp
 *     1e-5, per-token log-decay, padding mask that zeroes phi(k), v and the
 *     log-decay of pad tokens and the output of pad tokens:
 *     python/subq_audio/autograd.py:292-376 (mask at :336-341, clamp :367).
 *   - backward: chunk-boundary checkpoints (64 tokens) then a reverse adjoint
 *     per chunk with recomputation, exactly the structure of
 *     src/kernels/attention_backward.cpp:88-231 (Gamma_t recursion :183-190,
 *     dQ :192-201, dV :203-210, dK :212-220, d_gamma :222-228), extended by
 *     the quotient rule of python/subq_audio/autograd.py:497-499 (the
 *     analytic form, which ignores the clamp exactly as the reference does)
 *     and the per-token log-decay gradient d/dlog(gamma_t) = gamma_t <G_t, S_{t-1}>.
 *
 * The normaliser is handled by augmenting V with a column equal to the mask
 * (V' = [V*m | m]), so S' = [S | z]; this is algebraically the reference's
 * separate denominator scan (autograd.py:359-365).
 */
#include <float.h>
#include <pthread.h>
#include <stdatomic.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_CHUNK 64

static double phi_val(double x) { return x > 0.0 ? x + 1.0 : exp(x); }
static double phi_prime(double x) { return x > 0.0 ? 1.0 : exp(x); }

double oracle_phi(double x) { return phi_val(x); }
double oracle_phi_prime(double x) { return phi_prime(x); }

static double flush(double s, int ftz) {
    return (ftz && fabs(s) < (double)FLT_MIN) ? 0.0 : s;
}

/* Token-level inputs shared by forward and backward. */
typedef struct {
    long N, d, e;
    const double *q, *k, *v;      /* [N,d], [N,d], [N,e] */
    const double *log_gamma;      /* [N] or NULL (gamma == 1) */
    const double *mask;           /* [N] or NULL (all valid) */
    int normalize;
    double scale, clamp_min;
    int ftz;
} seq_t;

static double mask_at(const seq_t* s, long t) { return s->mask ? s->mask[t] : 1.0; }
static double lg_at(const seq_t* s, long t) {
    if (!s->log_gamma) return 0.0;
    return mask_at(s, t) > 0.0 ? s->log_gamma[t] : 0.0;
}

/* One recurrence step on the augmented state S' [d][ep]. */
static void step_state(const seq_t* s, long t, double* Sp, long ep, double* kbuf, double* vbuf) {
    const long d = s->d, e = s->e;
    const double m = mask_at(s, t);
    const double g = exp(lg_at(s, t));
    for (long i = 0; i < d; ++i) kbuf[i] = phi_val(s->k[t * d + i]) * m;
    for (long j = 0; j < e; ++j) vbuf[j] = s->v[t * e + j] * m;
    if (ep > e) vbuf[e] = m;
    for (long i = 0; i < d; ++i)
        for (long j = 0; j < ep; ++j)
            Sp[i * ep + j] = flush(g * Sp[i * ep + j] + kbuf[i] * vbuf[j], s->ftz);
}

static void load_state(const seq_t* s, double* Sp, long ep, const double* S0, const double* z0) {
    const long d = s->d, e = s->e;
    memset(Sp, 0, sizeof(double) * d * ep);
    if (S0)
        for (long i = 0; i < d; ++i)
            for (long j = 0; j < e; ++j) Sp[i * ep + j] = S0[i * e + j];
    if (ep > e && z0)
        for (long i = 0; i < d; ++i) Sp[i * ep + e] = z0[i];
}

static void query_row(const seq_t* s, long t, double* qbuf) {
    for (long i = 0; i < s->d; ++i) qbuf[i] = phi_val(s->q[t * s->d + i]) * s->scale;
}

/* o = q~^T S' : numerator in o[0..e), denominator (if any) in o[e]. */
static void read_out(const seq_t* s, const double* Sp, long ep, const double* qbuf, double* o) {
    for (long j = 0; j < ep; ++j) {
        double acc = 0.0;
        for (long i = 0; i < s->d; ++i) acc += qbuf[i] * Sp[i * ep + j];
        o[j] = acc;
    }
}

static void forward_seq(const seq_t* s, const double* S0, const double* z0, double* out,
                        double* S_out, double* z_out, double* den_out) {
    const long d = s->d, e = s->e, ep = e + (s->normalize ? 1 : 0);
    double* Sp = (double*)malloc(sizeof(double) * d * ep);
    double* kbuf = (double*)malloc(sizeof(double) * d);
    double* qbuf = (double*)malloc(sizeof(double) * d);
    double* vbuf = (double*)malloc(sizeof(double) * ep);
    double* o = (double*)malloc(sizeof(double) * ep);
    load_state(s, Sp, ep, S0, z0);
    for (long t = 0; t < s->N; ++t) {
        step_state(s, t, Sp, ep, kbuf, vbuf);
        query_row(s, t, qbuf);
        read_out(s, Sp, ep, qbuf, o);
        const double m = mask_at(s, t);
        if (s->normalize) {
            const double zc = o[e] > s->clamp_min ? o[e] : s->clamp_min;
            for (long j = 0; j < e; ++j) out[t * e + j] = o[j] / zc * m;
            if (den_out) den_out[t] = zc;
        } else {
            for (long j = 0; j < e; ++j) out[t * e + j] = o[j] * m;
            if (den_out) den_out[t] = 1.0;
        }
    }
    if (S_out)
        for (long i = 0; i < d; ++i)
            for (long j = 0; j < e; ++j) S_out[i * e + j] = Sp[i * ep + j];
    if (z_out)
        for (long i = 0; i < d; ++i) z_out[i] = s->normalize ? Sp[i * ep + e] : 0.0;
    free(Sp); free(kbuf); free(qbuf); free(vbuf); free(o);
}

static void backward_seq(const seq_t* s, const double* S0, const double* z0, const double* dO,
                         double* dq, double* dk, double* dv, double* dlg) {
    const long N = s->N, d = s->d, e = s->e, ep = e + (s->normalize ? 1 : 0);
    const long C = ORACLE_CHUNK;
    const long nchunks = (N + C - 1) / C;
    const long SS = d * ep;
    double* ckpt = (double*)malloc(sizeof(double) * SS * (nchunks + 1));
    double* chunkS = (double*)malloc(sizeof(double) * SS * C);
    double* Sp = (double*)malloc(sizeof(double) * SS);
    double* G = (double*)calloc((size_t)SS, sizeof(double));
    double* kbuf = (double*)malloc(sizeof(double) * d);
    double* qbuf = (double*)malloc(sizeof(double) * d);
    double* vbuf = (double*)malloc(sizeof(double) * ep);
    double* o = (double*)malloc(sizeof(double) * ep);
    double* dOp = (double*)malloc(sizeof(double) * ep);

    /* Pass 1: state at every chunk boundary. */
    load_state(s, Sp, ep, S0, z0);
    double* S_init = (double*)malloc(sizeof(double) * SS);
    memcpy(S_init, Sp, sizeof(double) * SS);
    for (long c = 0; c < nchunks; ++c) {
        memcpy(ckpt + c * SS, Sp, sizeof(double) * SS);
        const long t1 = (c + 1) * C < N ? (c + 1) * C : N;
        for (long t = c * C; t < t1; ++t) step_state(s, t, Sp, ep, kbuf, vbuf);
    }

    /* Pass 2: reverse adjoint, one chunk at a time, states recomputed. */
    double g_next = 1.0; /* gamma_{t+1}, applied to G before adding token t */
    for (long c = nchunks - 1; c >= 0; --c) {
        const long t0 = c * C;
        const long t1 = (c + 1) * C < N ? (c + 1) * C : N;
        memcpy(Sp, ckpt + c * SS, sizeof(double) * SS);
        for (long t = t0; t < t1; ++t) {
            step_state(s, t, Sp, ep, kbuf, vbuf);
            memcpy(chunkS + (t - t0) * SS, Sp, sizeof(double) * SS);
        }
        for (long t = t1 - 1; t >= t0; --t) {
            const double* St = chunkS + (t - t0) * SS;
            const double* Sprev = (t > t0) ? chunkS + (t - 1 - t0) * SS : ckpt + c * SS;
            const double m = mask_at(s, t);
            const double lg = lg_at(s, t);
            query_row(s, t, qbuf);
            for (long i = 0; i < d; ++i) kbuf[i] = phi_val(s->k[t * d + i]) * m;
            for (long j = 0; j < e; ++j) vbuf[j] = s->v[t * e + j] * m;
            if (ep > e) vbuf[e] = m;

            /* Upstream gradient on the augmented output (quotient rule). */
            if (s->normalize) {
                read_out(s, St, ep, qbuf, o);
                const double zc = o[e] > s->clamp_min ? o[e] : s->clamp_min;
                double dot = 0.0;
                for (long j = 0; j < e; ++j) {
                    const double g = dO[t * e + j] * m;
                    dOp[j] = g / zc;
                    dot += g * o[j];
                }
                dOp[e] = -dot / (zc * zc);
            } else {
                for (long j = 0; j < e; ++j) dOp[j] = dO[t * e + j] * m;
            }

            /* G_t = gamma_{t+1} G_{t+1} + q~_t dO'_t^T */
            for (long i = 0; i < d; ++i)
                for (long j = 0; j < ep; ++j) G[i * ep + j] = g_next * G[i * ep + j] + qbuf[i] * dOp[j];
            g_next = exp(lg);

            /* dq~_t = S_t dO'_t */
            for (long i = 0; i < d; ++i) {
                double acc = 0.0;
                for (long j = 0; j < ep; ++j) acc += St[i * ep + j] * dOp[j];
                dq[t * d + i] = acc * s->scale * phi_prime(s->q[t * d + i]) * m;
            }
            /* dk~_t = G_t v'_t */
            for (long i = 0; i < d; ++i) {
                double acc = 0.0;
                for (long j = 0; j < ep; ++j) acc += G[i * ep + j] * vbuf[j];
                dk[t * d + i] = acc * phi_prime(s->k[t * d + i]) * m;
            }
            /* dv_t = (G_t^T phi(k_t))[0:e] */
            for (long j = 0; j < e; ++j) {
                double acc = 0.0;
                for (long i = 0; i < d; ++i) acc += G[i * ep + j] * kbuf[i];
                dv[t * e + j] = acc * m;
            }
            /* dL/dlog(gamma_t) = gamma_t <G_t, S_{t-1}>; pads carry a constant 0 log-decay. */
            if (dlg) {
                double acc = 0.0;
                for (long x = 0; x < SS; ++x) acc += G[x] * Sprev[x];
                dlg[t] = (m > 0.0) ? exp(lg) * acc : 0.0;
            }
        }
    }
    free(ckpt); free(chunkS); free(Sp); free(G); free(kbuf); free(qbuf); free(vbuf);
    free(o); free(dOp); free(S_init);
}

static seq_t make_seq(long b, long N, long d, long e, const double* q, const double* k,
                      const double* v, const double* log_gamma, const double* mask, int normalize,
                      double scale, double clamp_min, int ftz) {
    seq_t s;
    s.N = N; s.d = d; s.e = e;
    s.q = q + b * N * d; s.k = k + b * N * d; s.v = v + b * N * e;
    s.log_gamma = log_gamma ? log_gamma + b * N : NULL;
    s.mask = mask ? mask + b * N : NULL;
    s.normalize = normalize; s.scale = scale; s.clamp_min = clamp_min; s.ftz = ftz;
    return s;
}

/* All arrays are C-contiguous float64; BH sequences are independent.
 * q,k [BH,N,d]; v,out [BH,N,e]; log_gamma, mask, den_out [BH,N];
 * S0, S_out [BH,d,e]; z0, z_out [BH,d]. Optional pointers may be NULL. */
/* Sequences are independent: a small pthread pool walks them with an atomic
 * cursor (the oracle's only concession to speed). */
typedef struct {
    int backward;
    long BH, N, d, e;
    const double *q, *k, *v, *log_gamma, *mask, *S0, *z0, *dO;
    int normalize, ftz;
    double scale, clamp_min;
    double *out, *S_out, *z_out, *den_out, *dq, *dk, *dv, *dlg;
    atomic_long next;
} job_t;

static void* worker(void* arg) {
    job_t* j = (job_t*)arg;
    for (;;) {
        const long b = atomic_fetch_add(&j->next, 1);
        if (b >= j->BH) break;
        const long N = j->N, d = j->d, e = j->e;
        seq_t s = make_seq(b, N, d, e, j->q, j->k, j->v, j->log_gamma, j->mask, j->normalize,
                           j->scale, j->clamp_min, j->ftz);
        const double* S0 = j->S0 ? j->S0 + b * d * e : NULL;
        const double* z0 = j->z0 ? j->z0 + b * d : NULL;
        if (!j->backward) {
            forward_seq(&s, S0, z0, j->out + b * N * e, j->S_out ? j->S_out + b * d * e : NULL,
                        j->z_out ? j->z_out + b * d : NULL, j->den_out ? j->den_out + b * N : NULL);
        } else {
            backward_seq(&s, S0, z0, j->dO + b * N * e, j->dq + b * N * d, j->dk + b * N * d,
                         j->dv + b * N * e, j->dlg ? j->dlg + b * N : NULL);
        }
    }
    return NULL;
}

static void run_job(job_t* j, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > j->BH) nthreads = (int)(j->BH > 0 ? j->BH : 1);
    atomic_init(&j->next, 0);
    pthread_t th[256];
    int started = 0;
    for (int i = 1; i < nthreads; ++i)
        if (pthread_create(&th[started], NULL, worker, j) == 0) ++started;
    worker(j);
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
}

/* All arrays are C-contiguous float64; BH sequences are independent.
 * q,k [BH,N,d]; v,out [BH,N,e]; log_gamma, mask, den_out [BH,N];
 * S0, S_out [BH,d,e]; z0, z_out [BH,d]. Optional pointers may be NULL. */
int oracle_forward(long BH, long N, long d, long e, const double* q, const double* k,
                   const double* v, const double* log_gamma, const double* mask, int normalize,
                   double scale, double clamp_min, const double* S0, const double* z0, double* out,
                   double* S_out, double* z_out, double* den_out, int ftz, int nthreads) {
    if (BH < 0 || N < 0 || d <= 0 || e <= 0) return 1;
    job_t j;
    memset(&j, 0, sizeof(j));
    j.backward = 0; j.BH = BH; j.N = N; j.d = d; j.e = e;
    j.q = q; j.k = k; j.v = v; j.log_gamma = log_gamma; j.mask = mask; j.S0 = S0; j.z0 = z0;
    j.normalize = normalize; j.ftz = ftz; j.scale = scale; j.clamp_min = clamp_min;
    j.out = out; j.S_out = S_out; j.z_out = z_out; j.den_out = den_out;
    run_job(&j, nthreads);
    return 0;
}

/* dO [BH,N,e] -> dq,dk [BH,N,d], dv [BH,N,e], dlog_gamma [BH,N] (may be NULL). */
int oracle_backward(long BH, long N, long d, long e, const double* q, const double* k,
                    const double* v, const double* log_gamma, const double* mask, int normalize,
                    double scale, double clamp_min, const double* S0, const double* z0,
                    const double* dO, double* dq, double* dk, double* dv, double* dlog_gamma,
                    int ftz, int nthreads) {
    if (BH < 0 || N < 0 || d <= 0 || e <= 0) return 1;
    job_t j;
    memset(&j, 0, sizeof(j));
    j.backward = 1; j.BH = BH; j.N = N; j.d = d; j.e = e;
    j.q = q; j.k = k; j.v = v; j.log_gamma = log_gamma; j.mask = mask; j.S0 = S0; j.z0 = z0;
    j.dO = dO; j.normalize = normalize; j.ftz = ftz; j.scale = scale; j.clamp_min = clamp_min;
    j.dq = dq; j.dk = dk; j.dv = dv; j.dlg = dlog_gamma;
    run_job(&j, nthreads);
    return 0;
}
