/*
 * TEST INFRASTRUCTURE ONLY.  CPU restatement of the reference SGSA forward,
 * used as the parity checker by tests/, by __graft_entry__.smoke() and as the
 * timed CPU baseline in bench.py.  The shipped library never links or calls it.
 *
 * Parity status: pinned.  tests/golden/make_golden.py runs the reference's own
 * Python code (naive_recurrent_sgsa, SparseRetriever._masked_topk and
 * TopKSparseKVReuseAttention) on seeded inputs and commits the outputs; the CPU
 * test suite checks these functions against those fixtures.
 *
 * Layout conventions follow the reference:
 *   q, k, v, sparse_k, sparse_v, out : [B, T, H, D]      (float32)
 *   beta, gamma, alpha               : [B, T, H]         (float32)
 *   state                            : [B, H, D, D]      (float32, S[d][e])
 *   indexer q/k                      : [B, T, H, DI]
 *   top-k indices                    : [B, H, T, K] int32, ascending, -1 padded
 * All arithmetic is carried in double precision.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/*
 * Token-by-token SGSA recurrence.
 * Follows modelings/sgsa_ops/naive.py:39-55: the decayed base state
 * gamma_t * S feeds both the local write (k, v, beta) and the optional sparse
 * write (sparse_k, sparse_v, alpha); the readout is o_t = S_t^T q_t with no
 * query scale.  Only heads [h0, h1) are processed (h1 <= 0 means all), which
 * lets the CPU baseline time a bounded sample.
 */
void oracle_sgsa_recurrent(const float *q, const float *k, const float *v,
                           const float *beta, const float *gamma,
                           const float *sk, const float *sv, const float *alpha,
                           const float *init_state, float *out, float *final_state,
                           int B, int T, int H, int D, int h0, int h1) {
    if (h1 <= 0 || h1 > H) h1 = H;
    const int has_sparse = (sk && sv && alpha);
    const int nbh = B * (h1 - h0);
#pragma omp parallel for schedule(dynamic, 1)
    for (int bh = 0; bh < nbh; ++bh) {
        const int b = bh / (h1 - h0);
        const int h = h0 + bh % (h1 - h0);
        double *S = (double *)malloc(sizeof(double) * D * D);
        double *pl = (double *)malloc(sizeof(double) * D);
        double *ps = (double *)malloc(sizeof(double) * D);
        if (init_state) {
            const float *s0 = init_state + ((size_t)b * H + h) * D * D;
            for (int i = 0; i < D * D; ++i) S[i] = s0[i];
        } else {
            memset(S, 0, sizeof(double) * D * D);
        }
        for (int t = 0; t < T; ++t) {
            const size_t row = (((size_t)b * T + t) * H + h);
            const float *kt = k + row * D, *vt = v + row * D, *qt = q + row * D;
            const double g = gamma[row], bt = beta[row];
            for (int i = 0; i < D * D; ++i) S[i] *= g;
            /* predicted = base^T k : pl[e] = sum_d S[d][e] k[d] */
            for (int e = 0; e < D; ++e) pl[e] = 0.0;
            for (int d = 0; d < D; ++d) {
                const double kd = kt[d];
                const double *Sd = S + (size_t)d * D;
                for (int e = 0; e < D; ++e) pl[e] += Sd[e] * kd;
            }
            if (has_sparse) {
                const float *skt = sk + row * D;
                for (int e = 0; e < D; ++e) ps[e] = 0.0;
                for (int d = 0; d < D; ++d) {
                    const double kd = skt[d];
                    const double *Sd = S + (size_t)d * D;
                    for (int e = 0; e < D; ++e) ps[e] += Sd[e] * kd;
                }
            }
            for (int e = 0; e < D; ++e) pl[e] = (vt[e] - pl[e]) * bt;
            if (has_sparse) {
                const float *svt = sv + row * D;
                const double al = alpha[row];
                for (int e = 0; e < D; ++e) ps[e] = (svt[e] - ps[e]) * al;
            }
            for (int d = 0; d < D; ++d) {
                double *Sd = S + (size_t)d * D;
                const double kd = kt[d];
                for (int e = 0; e < D; ++e) Sd[e] += kd * pl[e];
                if (has_sparse) {
                    const double skd = sk[row * D + d];
                    for (int e = 0; e < D; ++e) Sd[e] += skd * ps[e];
                }
            }
            float *ot = out + row * D;
            for (int e = 0; e < D; ++e) {
                double acc = 0.0;
                for (int d = 0; d < D; ++d) acc += S[(size_t)d * D + e] * qt[d];
                ot[e] = (float)acc;
            }
        }
        if (final_state) {
            float *sf = final_state + ((size_t)b * H + h) * D * D;
            for (int i = 0; i < D * D; ++i) sf[i] = (float)S[i];
        }
        free(S);
        free(pl);
        free(ps);
    }
}

/* Descending score, ties to the lower index: the stable order that the
 * reference's torch.topk calls (modelings/modeling_sgsa.py:155-164,
 * modelings/hybrid_dense_delta_topk.py:349) produce on distinct scores. */
typedef struct {
    double s;
    int j;
} scored_t;

static int cmp_scored(const void *a, const void *b) {
    const scored_t *x = (const scored_t *)a, *y = (const scored_t *)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    return (x->j > y->j) - (x->j < y->j);
}

static int cmp_int(const void *a, const void *b) {
    int x = *(const int *)a, y = *(const int *)b;
    return (x > y) - (x < y);
}

/*
 * Row-wise top-k over given scores.  Row r considers columns [0, valid[r]) and
 * keeps min(K, valid[r]) of them; output indices are sorted ascending and the
 * remaining slots hold -1.  Scores are compared as given (float32), so this is
 * the exact reference for a device select run on the same score matrix.
 */
void oracle_topk_select_f32(const float *scores, const int *valid, int R, int S, int K,
                            int32_t *idx_out) {
#pragma omp parallel
    {
        scored_t *buf = (scored_t *)malloc(sizeof(scored_t) * (S > 0 ? S : 1));
        int *sel = (int *)malloc(sizeof(int) * (K > 0 ? K : 1));
#pragma omp for schedule(dynamic, 16)
        for (int r = 0; r < R; ++r) {
            const int n = valid[r] < S ? valid[r] : S;
            const float *row = scores + (size_t)r * S;
            for (int j = 0; j < n; ++j) {
                buf[j].s = row[j];
                buf[j].j = j;
            }
            qsort(buf, n, sizeof(scored_t), cmp_scored);
            const int m = n < K ? n : K;
            for (int i = 0; i < m; ++i) sel[i] = buf[i].j;
            qsort(sel, m, sizeof(int), cmp_int);
            int32_t *o = idx_out + (size_t)r * K;
            for (int i = 0; i < K; ++i) o[i] = i < m ? sel[i] : -1;
        }
        free(buf);
        free(sel);
    }
}

/*
 * Causal per-head indexer: s_tj = iq_t . ik_j (j <= t), keep top-min(K, t+1)
 * by score with ties to the lowest j, self included.  Mirrors the per-head
 * selection of modelings/hybrid_dense_delta_topk.py:344-349 and
 * modelings/modeling_sgsa.py:144-165 with the indexer vectors in place of the
 * attention q/k.  Optionally writes the K-th largest score of each row to
 * kth_score (for near-tie analysis in tests).  Queries t in [t0, t1) only.
 */
void oracle_indexer_topk(const float *iq, const float *ik, int B, int T, int H, int DI, int K,
                         int t0, int t1, int32_t *idx_out, double *kth_score) {
    if (t1 <= 0 || t1 > T) t1 = T;
    const int nq = t1 - t0;
#pragma omp parallel
    {
        scored_t *buf = (scored_t *)malloc(sizeof(scored_t) * (T > 0 ? T : 1));
        int *sel = (int *)malloc(sizeof(int) * (K > 0 ? K : 1));
#pragma omp for collapse(2) schedule(dynamic, 8)
        for (int bh = 0; bh < B * H; ++bh) {
            for (int tt = 0; tt < nq; ++tt) {
                const int b = bh / H, h = bh % H, t = t0 + tt;
                const float *qv = iq + (((size_t)b * T + t) * H + h) * DI;
                const int n = t + 1;
                for (int j = 0; j < n; ++j) {
                    const float *kv = ik + (((size_t)b * T + j) * H + h) * DI;
                    double acc = 0.0;
                    for (int d = 0; d < DI; ++d) acc += (double)qv[d] * (double)kv[d];
                    buf[j].s = acc;
                    buf[j].j = j;
                }
                qsort(buf, n, sizeof(scored_t), cmp_scored);
                const int m = n < K ? n : K;
                if (kth_score) kth_score[((size_t)bh) * nq + tt] = buf[m - 1].s;
                for (int i = 0; i < m; ++i) sel[i] = buf[i].j;
                qsort(sel, m, sizeof(int), cmp_int);
                int32_t *o = idx_out + (((size_t)bh) * nq + tt) * K;
                for (int i = 0; i < K; ++i) o[i] = i < m ? sel[i] : -1;
            }
        }
        free(buf);
        free(sel);
    }
}

/*
 * Sparse attention over the selected rows followed by the gate.
 * o_s,t = sum_{j in I_t} softmax_j(q_t . k_j * scale) v_j in double
 * (modelings/hybrid_dense_delta_topk.py:343-356), then
 * out = m * o_s + (1 - m) * o_delta (modelings/hybrid_dense_delta_topk.py:389-390).
 * mix is [B,T,H,D] when mix_per_channel != 0, else [B,T,H].  Index rows are
 * [B,H,T,K] for queries [t0, t1); entries < 0 are skipped.  o_delta/mix may be
 * NULL, in which case out = o_s.
 */
void oracle_sparse_attn_mix(const float *q, const float *k, const float *v, const int32_t *idx,
                            const float *o_delta, const float *mix, float *out, int B, int T,
                            int H, int D, int K, double scale, int mix_per_channel, int t0,
                            int t1) {
    if (t1 <= 0 || t1 > T) t1 = T;
    const int nq = t1 - t0;
#pragma omp parallel
    {
        double *p = (double *)malloc(sizeof(double) * (K > 0 ? K : 1));
        double *acc = (double *)malloc(sizeof(double) * D);
#pragma omp for collapse(2) schedule(dynamic, 8)
        for (int bh = 0; bh < B * H; ++bh) {
            for (int tt = 0; tt < nq; ++tt) {
                const int b = bh / H, h = bh % H, t = t0 + tt;
                const size_t row = (((size_t)b * T + t) * H + h);
                const float *qv = q + row * D;
                const int32_t *ix = idx + (((size_t)bh) * nq + tt) * K;
                double mx = -INFINITY;
                for (int i = 0; i < K; ++i) {
                    p[i] = -INFINITY;
                    if (ix[i] < 0) continue;
                    const float *kv = k + (((size_t)b * T + ix[i]) * H + h) * D;
                    double s = 0.0;
                    for (int d = 0; d < D; ++d) s += (double)qv[d] * (double)kv[d];
                    p[i] = s * scale;
                    if (p[i] > mx) mx = p[i];
                }
                double den = 0.0;
                for (int i = 0; i < K; ++i) {
                    p[i] = (ix[i] < 0) ? 0.0 : exp(p[i] - mx);
                    den += p[i];
                }
                for (int d = 0; d < D; ++d) acc[d] = 0.0;
                for (int i = 0; i < K; ++i) {
                    if (ix[i] < 0) continue;
                    const float *vv = v + (((size_t)b * T + ix[i]) * H + h) * D;
                    const double w = p[i] / den;
                    for (int d = 0; d < D; ++d) acc[d] += w * vv[d];
                }
                float *ot = out + (((size_t)b * nq + tt) * H + h) * D;
                for (int d = 0; d < D; ++d) {
                    double o = acc[d];
                    if (o_delta && mix) {
                        const double m = mix_per_channel ? mix[row * D + d] : mix[row];
                        o = m * o + (1.0 - m) * o_delta[row * D + d];
                    }
                    ot[d] = (float)o;
                }
            }
        }
        free(p);
        free(acc);
    }
}
