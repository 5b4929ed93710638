/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle of the vesper-b200 hot path.
 *
 * Plain C, float64 throughout, written from the mathematics of mstampfli/vesper-preview's
 * pure-PyTorch reference path. Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline legs may load this library, and only as the checker (or as the timed CPU port of
 * the reference); nothing in the vesper_b200 package links or calls it.
 *
 * Parity pin: tests/test_oracle_golden.py checks every function here against golden vectors
 * that tests/golden/make_golden.py produced by running the reference itself (float64, CPU),
 * plus the reference's hand-derived two-token known-answer test.
 *
 * Functions and the reference code each one restates (paths inside the reference project):
 *   vo_delta_scan_fwd / vo_delta_scan_bwd   vesper/recurrence.py:118-163 (delta_update,
 *       delta_scan_step: token-serial form; tests pin it equal to delta_scan_chunked
 *       :166-217) and the analytic gradient autograd takes through it.
 *   vo_keys_fwd / vo_keys_bwd               vesper/column.py:255-289 (RecurrentSublayer.keys:
 *       causal depthwise filter with history, then normalize_keys recurrence.py:91-115 per
 *       head; the normalisation's max-abs scale is detached, clamp_min passes gradient at and
 *       above a squared norm of one).
 *   vo_rms_fwd / vo_rms_bwd                 vesper/column.py:159-188 (RMSNorm.forward, scale-safe,
 *       eps inside the root, scale detached) and kernels/norm_triton.py:47-82 (its gradient).
 *   vo_window_attn_fwd / vo_window_attn_bwd vesper/attention.py:340-407 (attend: softmax over
 *       the last `window` positions of cache+chunk, scale 1/sqrt(dk), GQA head h -> h / groups)
 *       and kernels/window_attn.py:27-39.
 *
 * State layout follows the reference: H[i][j], i the key index, j the value index, read as
 * o = H^T q after the token's own write.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define VO_CKPT 64 /* tokens between saved states in the backward's recomputation */
#define VO_MAX_D 256 /* the largest head width the scan accepts (kernels/delta_scan.py:41) */

/* ------------------------------------------------------------------------------------------ */
/* delta rule, token-serial                                                                     */
/* ------------------------------------------------------------------------------------------ */

/* index helpers for [B, T, H, D] and [B, T, H] */
#define IX4(b, t, h, i) ((((int64_t)(b) * T + (t)) * H + (h)) * D + (i))
#define IX3(b, t, h) (((int64_t)(b) * T + (t)) * H + (h))

/* One token: r = v - H^T k; H += beta k r^T; o = H^T q (recurrence.py:118-163). */
static void step_fwd(int D, double *S, const double *q, const double *k, const double *v,
                     double beta, double *o) {
    double r[VO_MAX_D];
    for (int j = 0; j < D; ++j) r[j] = v[j];
    for (int i = 0; i < D; ++i) {
        double ki = k[i];
        for (int j = 0; j < D; ++j) r[j] -= S[i * D + j] * ki;
    }
    for (int i = 0; i < D; ++i) {
        double bk = beta * k[i];
        for (int j = 0; j < D; ++j) S[i * D + j] += bk * r[j];
    }
    if (o) {
        for (int j = 0; j < D; ++j) o[j] = 0.0;
        for (int i = 0; i < D; ++i) {
            double qi = q[i];
            for (int j = 0; j < D; ++j) o[j] += S[i * D + j] * qi;
        }
    }
}

/* Forward over all tokens. q,k,v,o [B,T,H,D]; beta [B,T,H]; s0, sn [B,H,D,D]. */
void vo_delta_scan_fwd(int B, int T, int H, int D, const double *q, const double *k,
                       const double *v, const double *beta, const double *s0, double *o,
                       double *sn) {
#pragma omp parallel for schedule(dynamic, 1)
    for (int bh = 0; bh < B * H; ++bh) {
        int b = bh / H, h = bh % H;
        double *S = sn + (int64_t)bh * D * D;
        memcpy(S, s0 + (int64_t)bh * D * D, sizeof(double) * D * D);
        for (int t = 0; t < T; ++t)
            step_fwd(D, S, q + IX4(b, t, h, 0), k + IX4(b, t, h, 0), v + IX4(b, t, h, 0),
                     beta[IX3(b, t, h)], o + IX4(b, t, h, 0));
    }
}

/*
 * Backward of vo_delta_scan_fwd for the loss sum(o * dout) + sum(sn * dsn).
 * With S_t = S_{t-1} + beta k r^T, r = v - S_{t-1}^T k, o_t = S_t^T q and G = dL/dS_t:
 *   G += q dout_t^T;  dq = S_t dout_t;  dr = beta G^T k;  dv = dr;  dbeta = k^T G r;
 *   dk = beta G r - S_{t-1} dr;  dL/dS_{t-1} = G - k dr^T.
 * States are recomputed forward from checkpoints every VO_CKPT tokens.
 */
void vo_delta_scan_bwd(int B, int T, int H, int D, const double *q, const double *k,
                       const double *v, const double *beta, const double *s0,
                       const double *dout, const double *dsn, double *dq, double *dk,
                       double *dv, double *dbeta, double *ds0) {
    int segs = (T + VO_CKPT - 1) / VO_CKPT;
#pragma omp parallel for schedule(dynamic, 1)
    for (int bh = 0; bh < B * H; ++bh) {
        int b = bh / H, h = bh % H;
        int64_t dd = (int64_t)D * D;
        double *ck = (double *)malloc(sizeof(double) * dd * (segs + 1));
        double *seg = (double *)malloc(sizeof(double) * dd * (VO_CKPT + 1));
        double *G = (double *)malloc(sizeof(double) * dd);
        double *r = (double *)malloc(sizeof(double) * D);
        double *dr = (double *)malloc(sizeof(double) * D);
        double *gr = (double *)malloc(sizeof(double) * D);
        memcpy(ck, s0 + bh * dd, sizeof(double) * dd);
        for (int s = 0; s < segs; ++s) {
            memcpy(ck + (s + 1) * dd, ck + s * dd, sizeof(double) * dd);
            int t1 = (s + 1) * VO_CKPT < T ? (s + 1) * VO_CKPT : T;
            for (int t = s * VO_CKPT; t < t1; ++t)
                step_fwd(D, ck + (s + 1) * dd, NULL, k + IX4(b, t, h, 0), v + IX4(b, t, h, 0),
                         beta[IX3(b, t, h)], NULL);
        }
        memcpy(G, dsn + bh * dd, sizeof(double) * dd);
        for (int s = segs - 1; s >= 0; --s) {
            int t0 = s * VO_CKPT;
            int t1 = (s + 1) * VO_CKPT < T ? (s + 1) * VO_CKPT : T;
            memcpy(seg, ck + s * dd, sizeof(double) * dd); /* seg[0] = S_{t0-1} */
            for (int t = t0; t < t1; ++t) {
                memcpy(seg + (t - t0 + 1) * dd, seg + (t - t0) * dd, sizeof(double) * dd);
                step_fwd(D, seg + (t - t0 + 1) * dd, NULL, k + IX4(b, t, h, 0),
                         v + IX4(b, t, h, 0), beta[IX3(b, t, h)], NULL);
            }
            for (int t = t1 - 1; t >= t0; --t) {
                const double *St = seg + (t - t0 + 1) * dd;
                const double *Sp = seg + (t - t0) * dd;
                const double *qt = q + IX4(b, t, h, 0), *kt = k + IX4(b, t, h, 0);
                const double *vt = v + IX4(b, t, h, 0), *gt = dout + IX4(b, t, h, 0);
                double bt = beta[IX3(b, t, h)];
                for (int i = 0; i < D; ++i)
                    for (int j = 0; j < D; ++j) G[i * D + j] += qt[i] * gt[j];
                for (int i = 0; i < D; ++i) {
                    double acc = 0.0;
                    for (int j = 0; j < D; ++j) acc += St[i * D + j] * gt[j];
                    dq[IX4(b, t, h, i)] = acc;
                }
                for (int j = 0; j < D; ++j) {
                    double acc = 0.0;
                    for (int i = 0; i < D; ++i) acc += Sp[i * D + j] * kt[i];
                    r[j] = vt[j] - acc;
                }
                for (int j = 0; j < D; ++j) {
                    double acc = 0.0;
                    for (int i = 0; i < D; ++i) acc += G[i * D + j] * kt[i];
                    dr[j] = bt * acc;
                    dv[IX4(b, t, h, j)] = dr[j];
                }
                double db = 0.0;
                for (int i = 0; i < D; ++i) {
                    double acc = 0.0;
                    for (int j = 0; j < D; ++j) acc += G[i * D + j] * r[j];
                    gr[i] = acc;
                    db += kt[i] * acc;
                }
                dbeta[IX3(b, t, h)] = db;
                for (int i = 0; i < D; ++i) {
                    double acc = 0.0;
                    for (int j = 0; j < D; ++j) acc += Sp[i * D + j] * dr[j];
                    dk[IX4(b, t, h, i)] = bt * gr[i] - acc;
                }
                for (int i = 0; i < D; ++i)
                    for (int j = 0; j < D; ++j) G[i * D + j] -= kt[i] * dr[j];
            }
        }
        memcpy(ds0 + bh * dd, G, sizeof(double) * dd);
        free(ck);
        free(seg);
        free(G);
        free(r);
        free(dr);
        free(gr);
    }
}

/* ------------------------------------------------------------------------------------------ */
/* causal key filter + normalize_keys                                                           */
/* ------------------------------------------------------------------------------------------ */

/* full[b, p, j] with p in [0, K-1+T): history rows first, then z */
static inline double full_at(const double *z, const double *hist, int T, int W, int K, int b,
                             int p, int j) {
    if (p < K - 1) return hist[((int64_t)b * (K - 1) + p) * W + j];
    return z[((int64_t)b * T + (p - (K - 1))) * W + j];
}

/* u[b,t,j] = sum_r taps[r,j] full[b, t + K-1 - r, j] */
static void conv_row(const double *z, const double *hist, const double *taps, int T, int W,
                     int K, int b, int t, double *u) {
    for (int j = 0; j < W; ++j) {
        double acc = 0.0;
        for (int r = 0; r < K; ++r) acc += taps[(int64_t)r * W + j] * full_at(z, hist, T, W, K, b, t + K - 1 - r, j);
        u[j] = acc;
    }
}

/* normalize_keys on one head vector (recurrence.py:91-115); returns scale, den, sq. */
static void norm_keys_vec(const double *u, int n, double floor_, double *out, double *scale_o,
                          double *den_o, double *sq_o) {
    double amax = 0.0;
    for (int i = 0; i < n; ++i) amax = fmax(amax, fabs(u[i]));
    double scale = fmax(amax, floor_);
    double sq = 0.0;
    for (int i = 0; i < n; ++i) {
        double s = u[i] / scale;
        sq += s * s;
    }
    double den = sqrt(fmax(sq, 1.0));
    for (int i = 0; i < n; ++i) out[i] = (u[i] / scale) / den;
    if (scale_o) *scale_o = scale;
    if (den_o) *den_o = den;
    if (sq_o) *sq_o = sq;
}

/* keys [B,T,W] (viewed [B,T,heads,W/heads]) from z [B,T,W], hist [B,K-1,W], taps [K,W]. */
void vo_keys_fwd(int B, int T, int W, int heads, int K, const double *z, const double *hist,
                 const double *taps, double floor_, double *keys) {
    int hd = W / heads;
#pragma omp parallel for schedule(static)
    for (int64_t bt = 0; bt < (int64_t)B * T; ++bt) {
        int b = (int)(bt / T), t = (int)(bt % T);
        double *u = (double *)malloc(sizeof(double) * W);
        conv_row(z, hist, taps, T, W, K, b, t, u);
        for (int h = 0; h < heads; ++h)
            norm_keys_vec(u + h * hd, hd, floor_, keys + bt * W + h * hd, NULL, NULL, NULL);
        free(u);
    }
}

/* gradients of sum(keys * gk): dz [B,T,W], dhist [B,K-1,W], dtaps [K,W]. */
void vo_keys_bwd(int B, int T, int W, int heads, int K, const double *z, const double *hist,
                 const double *taps, double floor_, const double *gk, double *dz,
                 double *dhist, double *dtaps) {
    int hd = W / heads;
    int64_t rows = (int64_t)B * T;
    double *du = (double *)malloc(sizeof(double) * (rows * W + 1));
#pragma omp parallel for schedule(static)
    for (int64_t bt = 0; bt < rows; ++bt) {
        int b = (int)(bt / T), t = (int)(bt % T);
        double *u = (double *)malloc(sizeof(double) * W);
        double *kk = (double *)malloc(sizeof(double) * W);
        conv_row(z, hist, taps, T, W, K, b, t, u);
        for (int h = 0; h < heads; ++h) {
            double scale, den, sq;
            norm_keys_vec(u + h * hd, hd, floor_, kk + h * hd, &scale, &den, &sq);
            const double *g = gk + bt * W + h * hd;
            double dot = 0.0;
            for (int i = 0; i < hd; ++i) dot += g[i] * (u[h * hd + i] / scale);
            for (int i = 0; i < hd; ++i) {
                double s = u[h * hd + i] / scale;
                double through = sq >= 1.0 ? s * dot / (den * den * den) : 0.0;
                du[bt * W + h * hd + i] = (g[i] / den - through) / scale;
            }
        }
        free(u);
        free(kk);
    }
    memset(dtaps, 0, sizeof(double) * K * W);
    if (dhist) memset(dhist, 0, sizeof(double) * (int64_t)B * (K - 1) * W);
#pragma omp parallel for schedule(static)
    for (int j = 0; j < W; ++j) {
        for (int b = 0; b < B; ++b) {
            for (int p = 0; p < K - 1 + T; ++p) {
                /* full position p feeds u[t] with t = p - (K-1) + r, r in [0,K) */
                double acc = 0.0;
                for (int r = 0; r < K; ++r) {
                    int t = p - (K - 1) + r;
                    if (t < 0 || t >= T) continue;
                    acc += taps[(int64_t)r * W + j] * du[((int64_t)b * T + t) * W + j];
                }
                if (p < K - 1) {
                    if (dhist) dhist[((int64_t)b * (K - 1) + p) * W + j] = acc;
                } else {
                    dz[((int64_t)b * T + (p - (K - 1))) * W + j] = acc;
                }
            }
            for (int t = 0; t < T; ++t)
                for (int r = 0; r < K; ++r)
                    dtaps[(int64_t)r * W + j] += du[((int64_t)b * T + t) * W + j] *
                                                 full_at(z, hist, T, W, K, b, t + K - 1 - r, j);
        }
    }
    free(du);
}

/* ------------------------------------------------------------------------------------------ */
/* RMSNorm                                                                                      */
/* ------------------------------------------------------------------------------------------ */

void vo_rms_fwd(int64_t rows, int W, const double *x, const double *g, double floor_, double eps,
                double *y, double *inv) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const double *xr = x + r * W;
        double amax = 0.0;
        for (int j = 0; j < W; ++j) amax = fmax(amax, fabs(xr[j]));
        double scale = fmax(amax, floor_);
        double ss = 0.0;
        for (int j = 0; j < W; ++j) {
            double s = xr[j] / scale;
            ss += s * s;
        }
        double rms = sqrt(ss / W + eps / (scale * scale));
        for (int j = 0; j < W; ++j) y[r * W + j] = (xr[j] / scale) / rms * g[j];
        if (inv) inv[r] = 1.0 / (scale * rms);
    }
}

void vo_rms_bwd(int64_t rows, int W, const double *x, const double *g, double floor_, double eps,
                const double *dy, double *dx, double *dg) {
    memset(dg, 0, sizeof(double) * W);
    double *inv = (double *)malloc(sizeof(double) * (rows + 1));
    double *tmp = (double *)malloc(sizeof(double) * ((int64_t)rows * W + 1));
    vo_rms_fwd(rows, W, x, g, floor_, eps, tmp, inv);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const double *xr = x + r * W, *dr = dy + r * W;
        double mean = 0.0;
        for (int j = 0; j < W; ++j) mean += dr[j] * g[j] * xr[j] * inv[r];
        mean /= W;
        for (int j = 0; j < W; ++j)
            dx[r * W + j] = inv[r] * (dr[j] * g[j] - xr[j] * inv[r] * mean);
    }
    for (int64_t r = 0; r < rows; ++r)
        for (int j = 0; j < W; ++j) dg[j] += dy[r * W + j] * x[r * W + j] * inv[r];
    free(inv);
    free(tmp);
}

/* ------------------------------------------------------------------------------------------ */
/* windowed attention over cache (m rows) + chunk (n rows)                                      */
/* ------------------------------------------------------------------------------------------ */

/* q [B,n,H,D]; keys, values [B,L,Hkv,D] with L = m + n; o [B,n,H,D]; lse [B,n,H] (optional) */
void vo_window_attn_fwd(int B, int n, int L, int H, int Hkv, int D, int window,
                        const double *q, const double *kk, const double *vv, double *o,
                        double *lse) {
    int m = L - n, groups = H / Hkv;
    double scale = 1.0 / sqrt((double)D);
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < (int64_t)B * n * H; ++idx) {
        int h = (int)(idx % H);
        int i = (int)((idx / H) % n);
        int b = (int)(idx / ((int64_t)H * n));
        int g = h / groups, qi = m + i;
        int lo = qi - window + 1 < 0 ? 0 : qi - window + 1;
        const double *qv = q + idx * D;
        double mx = -INFINITY;
        double *s = (double *)malloc(sizeof(double) * (qi - lo + 1));
        for (int j = lo; j <= qi; ++j) {
            const double *kv = kk + (((int64_t)b * L + j) * Hkv + g) * D;
            double acc = 0.0;
            for (int e = 0; e < D; ++e) acc += qv[e] * kv[e];
            s[j - lo] = acc * scale;
            mx = fmax(mx, s[j - lo]);
        }
        double den = 0.0;
        for (int j = lo; j <= qi; ++j) den += exp(s[j - lo] - mx);
        double *ov = o + idx * D;
        for (int e = 0; e < D; ++e) ov[e] = 0.0;
        for (int j = lo; j <= qi; ++j) {
            double p = exp(s[j - lo] - mx) / den;
            const double *vr = vv + (((int64_t)b * L + j) * Hkv + g) * D;
            for (int e = 0; e < D; ++e) ov[e] += p * vr[e];
        }
        if (lse) lse[idx] = mx + log(den);
        free(s);
    }
}

/* gradients of sum(o * dout): dq [B,n,H,D], dk, dv [B,L,Hkv,D] */
void vo_window_attn_bwd(int B, int n, int L, int H, int Hkv, int D, int window,
                        const double *q, const double *kk, const double *vv, const double *dout,
                        double *dq, double *dk, double *dv) {
    int m = L - n, groups = H / Hkv;
    double scale = 1.0 / sqrt((double)D);
    double *o = (double *)malloc(sizeof(double) * ((int64_t)B * n * H * D + 1));
    double *lse = (double *)malloc(sizeof(double) * ((int64_t)B * n * H + 1));
    vo_window_attn_fwd(B, n, L, H, Hkv, D, window, q, kk, vv, o, lse);
    memset(dk, 0, sizeof(double) * (int64_t)B * L * Hkv * D);
    memset(dv, 0, sizeof(double) * (int64_t)B * L * Hkv * D);
    /* serial over (b, kv head) to keep the dk/dv accumulation race-free and ordered */
#pragma omp parallel for schedule(static)
    for (int bg = 0; bg < B * Hkv; ++bg) {
        int b = bg / Hkv, g = bg % Hkv;
        for (int h = g * groups; h < (g + 1) * groups; ++h) {
            for (int i = 0; i < n; ++i) {
                int64_t idx = ((int64_t)b * n + i) * H + h;
                int qi = m + i;
                int lo = qi - window + 1 < 0 ? 0 : qi - window + 1;
                const double *qv = q + idx * D, *go = dout + idx * D, *ov = o + idx * D;
                double di = 0.0;
                for (int e = 0; e < D; ++e) di += go[e] * ov[e];
                double *dqv = dq + idx * D;
                for (int e = 0; e < D; ++e) dqv[e] = 0.0;
                for (int j = lo; j <= qi; ++j) {
                    const double *kv = kk + (((int64_t)b * L + j) * Hkv + g) * D;
                    const double *vr = vv + (((int64_t)b * L + j) * Hkv + g) * D;
                    double s = 0.0, dp = 0.0;
                    for (int e = 0; e < D; ++e) {
                        s += qv[e] * kv[e];
                        dp += go[e] * vr[e];
                    }
                    double p = exp(s * scale - lse[idx]);
                    double ds = p * (dp - di) * scale;
                    double *dkr = dk + (((int64_t)b * L + j) * Hkv + g) * D;
                    double *dvr = dv + (((int64_t)b * L + j) * Hkv + g) * D;
                    for (int e = 0; e < D; ++e) {
                        dqv[e] += ds * kv[e];
                        dkr[e] += ds * qv[e];
                        dvr[e] += p * go[e];
                    }
                }
            }
        }
    }
    free(o);
    free(lse);
}

int vo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets the OpenMP thread count of every later call (n < 1 leaves it unchanged); returns the
 * count in effect. A launcher such as torchrun exports OMP_NUM_THREADS=1, which a timed CPU
 * baseline must override with the cores the process may actually use. */
int vo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}
