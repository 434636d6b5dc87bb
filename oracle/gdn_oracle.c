/*
 * CPU oracle for the gated delta rule, in C: TEST INFRASTRUCTURE ONLY.
 *
 * Used by the tests (large-size parity) and by bench.py's cpu_baseline / --impl reference legs as
 * the timed CPU restatement of the reference. Never linked into the product library.
 *
 * Restates soreRNN sore/model/gdn_ref.py:11-22 (per token: decay, delta update, readout) with the
 * GVA mapping of sore/model/gdn.py:171-174 and the F.normalize of gdn.py:177, in fp32 like the
 * reference (gdn_ref.py:45-47). The backward is the reverse-mode recurrence documented in
 * oracle/gdn_oracle.py (gdn_backward); states S_{t-1} are recomputed per block of BLK tokens from
 * block-start checkpoints so memory stays O(T/BLK * dk * dv) per (sequence, head).
 * Work is split over (sequence, head) pairs with OpenMP.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define BLK 64
#define L2_EPS 1e-12f

typedef struct {
    int64_t bos, eos;  /* token range in the flattened [B*T] axis */
    int64_t n;         /* sequence index */
} seq_t;

static int make_seqs(int64_t B, int64_t T, const int64_t* cu, int64_t N, seq_t* out) {
    if (cu) {
        for (int64_t i = 0; i < N; ++i) { out[i].bos = cu[i]; out[i].eos = cu[i + 1]; out[i].n = i; }
        return (int)N;
    }
    for (int64_t b = 0; b < B; ++b) { out[b].bos = b * T; out[b].eos = (b + 1) * T; out[b].n = b; }
    return (int)B;
}

static void norm_vec(const float* x, float* y, int d, int l2, float* inv_out) {
    if (!l2) { memcpy(y, x, sizeof(float) * d); if (inv_out) *inv_out = 1.f; return; }
    double s = 0; for (int i = 0; i < d; ++i) s += (double)x[i] * x[i];
    float n = (float)sqrt(s); float nn = n > L2_EPS ? n : L2_EPS;
    for (int i = 0; i < d; ++i) y[i] = x[i] / nn;
    if (inv_out) *inv_out = nn;
}

/* one token of the recurrence on S [dk][dv]; writes o (if not NULL) */
static void step(float* S, const float* qn, const float* kn, const float* v, float g, float beta,
                 float scale, int dk, int dv, float* delta_tmp, float* o) {
    float gam = expf(g);
    for (int i = 0; i < dk * dv; ++i) S[i] *= gam;
    for (int j = 0; j < dv; ++j) delta_tmp[j] = 0.f;
    for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) delta_tmp[j] += S[i * dv + j] * kn[i];
    for (int j = 0; j < dv; ++j) delta_tmp[j] = (v[j] - delta_tmp[j]) * beta;
    for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) S[i * dv + j] += kn[i] * delta_tmp[j];
    if (o) {
        for (int j = 0; j < dv; ++j) o[j] = 0.f;
        for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) o[j] += scale * qn[i] * S[i * dv + j];
    }
}

/* q,k [B*T, H, dk]; v,o [B*T, HV, dv]; g,beta [B*T, HV]; h0/ht [N, HV, dk, dv] (either may be NULL) */
void oracle_gdn_fwd(const float* q, const float* k, const float* v, const float* g, const float* beta,
                    int64_t B, int64_t T, int64_t H, int64_t HV, int64_t dk, int64_t dv,
                    const int64_t* cu, int64_t N, float scale, int l2norm, const float* h0,
                    float* o, float* ht, int nthreads) {
    seq_t* seqs = (seq_t*)malloc(sizeof(seq_t) * (cu ? N : B));
    int ns = make_seqs(B, T, cu, N, seqs);
    int64_t rep = HV / H;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t w = 0; w < (int64_t)ns * HV; ++w) {
        seq_t sq = seqs[w / HV]; int64_t hv = w % HV, hq = hv / rep;
        float* S = (float*)calloc(dk * dv, sizeof(float));
        float *qn = (float*)malloc(sizeof(float) * dk), *kn = (float*)malloc(sizeof(float) * dk);
        float* tmp = (float*)malloc(sizeof(float) * dv);
        if (h0) memcpy(S, h0 + (sq.n * HV + hv) * dk * dv, sizeof(float) * dk * dv);
        for (int64_t t = sq.bos; t < sq.eos; ++t) {
            norm_vec(q + (t * H + hq) * dk, qn, dk, l2norm, NULL);
            norm_vec(k + (t * H + hq) * dk, kn, dk, l2norm, NULL);
            step(S, qn, kn, v + (t * HV + hv) * dv, g[t * HV + hv], beta[t * HV + hv], scale, dk, dv, tmp,
                 o + (t * HV + hv) * dv);
        }
        if (ht) memcpy(ht + (sq.n * HV + hv) * dk * dv, S, sizeof(float) * dk * dv);
        free(S); free(qn); free(kn); free(tmp);
    }
    free(seqs);
}

/* Gradients: dq, dk [B*T, H, dk] are ACCUMULATED over the HV/H value heads (caller zeroes them). */
void oracle_gdn_bwd(const float* q, const float* k, const float* v, const float* g, const float* beta,
                    const float* dout, int64_t B, int64_t T, int64_t H, int64_t HV, int64_t dk, int64_t dv,
                    const int64_t* cu, int64_t N, float scale, int l2norm, const float* h0, const float* dht,
                    float* dq, float* dkk, float* dvv, float* dg, float* dbeta, float* dh0, int nthreads) {
    seq_t* seqs = (seq_t*)malloc(sizeof(seq_t) * (cu ? N : B));
    int ns = make_seqs(B, T, cu, N, seqs);
    int64_t rep = HV / H;
    int64_t SZ = dk * dv;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t w = 0; w < (int64_t)ns * HV; ++w) {
        seq_t sq = seqs[w / HV]; int64_t hv = w % HV, hq = hv / rep;
        int64_t L = sq.eos - sq.bos, nb = (L + BLK - 1) / BLK;
        float* ck = (float*)calloc((nb > 0 ? nb : 1) * SZ, sizeof(float)); /* block-start states */
        float* st = (float*)malloc(sizeof(float) * BLK * SZ);              /* S_{t-1} inside a block */
        float *S = (float*)calloc(SZ, sizeof(float)), *dH = (float*)calloc(SZ, sizeof(float));
        float *Sd = (float*)malloc(sizeof(float) * SZ);
        float *qn = (float*)malloc(sizeof(float) * dk), *kn = (float*)malloc(sizeof(float) * dk);
        float *tmp = (float*)malloc(sizeof(float) * dv), *delta = (float*)malloc(sizeof(float) * dv);
        float *u = (float*)malloc(sizeof(float) * dv), *dd = (float*)malloc(sizeof(float) * dv);
        float *gq = (float*)malloc(sizeof(float) * dk), *gk = (float*)malloc(sizeof(float) * dk);
        if (h0) memcpy(S, h0 + (sq.n * HV + hv) * SZ, sizeof(float) * SZ);
        for (int64_t b = 0; b < nb; ++b) {
            memcpy(ck + b * SZ, S, sizeof(float) * SZ);
            for (int64_t t = sq.bos + b * BLK; t < sq.bos + (b + 1) * BLK && t < sq.eos; ++t) {
                norm_vec(k + (t * H + hq) * dk, kn, dk, l2norm, NULL);
                step(S, kn, kn, v + (t * HV + hv) * dv, g[t * HV + hv], beta[t * HV + hv], scale, dk, dv, tmp, NULL);
            }
        }
        if (dht) memcpy(dH, dht + (sq.n * HV + hv) * SZ, sizeof(float) * SZ);
        for (int64_t b = nb - 1; b >= 0; --b) {
            int64_t t0 = sq.bos + b * BLK, t1 = t0 + BLK < sq.eos ? t0 + BLK : sq.eos;
            memcpy(S, ck + b * SZ, sizeof(float) * SZ);
            for (int64_t t = t0; t < t1; ++t) {
                memcpy(st + (t - t0) * SZ, S, sizeof(float) * SZ);
                norm_vec(k + (t * H + hq) * dk, kn, dk, l2norm, NULL);
                step(S, kn, kn, v + (t * HV + hv) * dv, g[t * HV + hv], beta[t * HV + hv], scale, dk, dv, tmp, NULL);
            }
            for (int64_t t = t1 - 1; t >= t0; --t) {
                float qnrm, knrm;
                norm_vec(q + (t * H + hq) * dk, qn, dk, l2norm, &qnrm);
                norm_vec(k + (t * H + hq) * dk, kn, dk, l2norm, &knrm);
                const float* vt = v + (t * HV + hv) * dv;
                const float* dot = dout + (t * HV + hv) * dv;
                float gam = expf(g[t * HV + hv]), bt = beta[t * HV + hv];
                const float* Sp = st + (t - t0) * SZ;
                for (int64_t i = 0; i < SZ; ++i) Sd[i] = Sp[i] * gam;
                for (int j = 0; j < dv; ++j) u[j] = 0.f;
                for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) u[j] += Sd[i * dv + j] * kn[i];
                for (int j = 0; j < dv; ++j) { u[j] = vt[j] - u[j]; delta[j] = u[j] * bt; }
                for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) dH[i * dv + j] += scale * qn[i] * dot[j];
                for (int i = 0; i < dk; ++i) {  /* dq = scale * S_t do, S_t = Sd + k delta^T */
                    float a = 0.f, c = 0.f, e = 0.f;
                    for (int j = 0; j < dv; ++j) {
                        a += (Sd[i * dv + j] + kn[i] * delta[j]) * dot[j];
                        c += dH[i * dv + j] * delta[j];
                    }
                    gq[i] = scale * a; gk[i] = c; (void)e;
                }
                for (int j = 0; j < dv; ++j) dd[j] = 0.f;
                for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) dd[j] += dH[i * dv + j] * kn[i];
                for (int i = 0; i < dk; ++i) {
                    float a = 0.f;
                    for (int j = 0; j < dv; ++j) a += Sd[i * dv + j] * dd[j];
                    gk[i] -= bt * a;
                }
                float db = 0.f, dgs = 0.f;
                for (int j = 0; j < dv; ++j) { dvv[(t * HV + hv) * dv + j] = bt * dd[j]; db += dd[j] * u[j]; }
                for (int i = 0; i < dk; ++i) for (int j = 0; j < dv; ++j) {
                    float x = dH[i * dv + j] - bt * kn[i] * dd[j];
                    dgs += x * Sd[i * dv + j];
                    dH[i * dv + j] = x * gam;
                }
                dbeta[t * HV + hv] = db; dg[t * HV + hv] = dgs;
                if (l2norm) {  /* chain rule through x / max(||x||, eps) */
                    float sq_ = 0.f, sk = 0.f;
                    for (int i = 0; i < dk; ++i) { sq_ += qn[i] * gq[i]; sk += kn[i] * gk[i]; }
                    for (int i = 0; i < dk; ++i) {
                        gq[i] = (gq[i] - qn[i] * sq_ * (qnrm > L2_EPS)) / qnrm;
                        gk[i] = (gk[i] - kn[i] * sk * (knrm > L2_EPS)) / knrm;
                    }
                }
#ifdef _OPENMP
                /* value heads sharing one q/k head may run on other threads */
                for (int i = 0; i < dk; ++i) {
#pragma omp atomic
                    dq[(t * H + hq) * dk + i] += gq[i];
#pragma omp atomic
                    dkk[(t * H + hq) * dk + i] += gk[i];
                }
#else
                for (int i = 0; i < dk; ++i) { dq[(t * H + hq) * dk + i] += gq[i]; dkk[(t * H + hq) * dk + i] += gk[i]; }
#endif
            }
        }
        if (dh0) memcpy(dh0 + (sq.n * HV + hv) * SZ, dH, sizeof(float) * SZ);
        free(ck); free(st); free(S); free(dH); free(Sd); free(qn); free(kn); free(tmp); free(delta);
        free(u); free(dd); free(gq); free(gk);
    }
    free(seqs);
}

/* one decode token: q,k [N,H,dk], v [N,HV,dv], g,beta [N,HV], state [N,HV,dk,dv] in place, o [N,HV,dv] */
void oracle_gdn_decode(const float* q, const float* k, const float* v, const float* g, const float* beta,
                       int64_t N, int64_t H, int64_t HV, int64_t dk, int64_t dv, float scale, int l2norm,
                       float* state, float* o, int nthreads) {
    int64_t rep = HV / H;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int64_t w = 0; w < N * HV; ++w) {
        int64_t n = w / HV, hv = w % HV, hq = hv / rep;
        float qn[1024], kn[1024], tmp[1024];
        if (dk > 1024 || dv > 1024) continue;
        norm_vec(q + (n * H + hq) * dk, qn, dk, l2norm, NULL);
        norm_vec(k + (n * H + hq) * dk, kn, dk, l2norm, NULL);
        step(state + w * dk * dv, qn, kn, v + w * dv, g[w], beta[w], scale, dk, dv, tmp, o + w * dv);
    }
}
