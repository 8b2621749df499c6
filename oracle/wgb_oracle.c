/*
 * wgb_oracle.c -- CPU restatement of WarpGBM's tree-growing hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in warpgbm_b200/csrc.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline leg may load it.  The product never calls it.
 *
 * Every function cites the reference (quantverse/warpgbm v2.2.0) lines whose
 * semantics it restates.  Two histogram flavours exist:
 *   - "reference" (orc_hist_ref): fp32 sums in sample order, one legal order
 *     of the reference's fp32 atomics (warpgbm/cuda/histogram_kernel.cu:36-59);
 *   - "canonical" (orc_hist_q): exact int64 sums of residuals quantised to a
 *     per-tree power-of-two grid.  This is what the CUDA product computes; it
 *     is order-independent, so results are identical at every GPU count.
 *
 * Build: make -C oracle   (gcc -O2 -ffp-contract=off -fopenmp)
 * -ffp-contract=off matters: the split arithmetic of best_split_kernel.cu has
 * to be evaluated with one rounding per operation, like the CUDA product's
 * __fmul_rn/__fdiv_rn/__fadd_rn sequence.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Binning                                                                   */
/* ------------------------------------------------------------------------ */

/* warpgbm/cuda/binner.cu:16-25: bin = number of leading edges e[0..] with
 * x >= e[b]; the scan stops at the first failure, so NaN -> 0. */
void orc_bin_matrix(const float *X, int64_t n, int64_t F, int64_t x_stride,
                    const float *edges, int nedges, int8_t *out,
                    int64_t out_stride)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        for (int64_t f = 0; f < F; ++f) {
            float v = X[i * x_stride + f];
            const float *e = edges + f * nedges;
            int b = 0;
            while (b < nedges && v >= e[b]) ++b;
            out[i * out_stride + f] = (int8_t)b;
        }
    }
}

static int cmp_float_nan_last(const void *pa, const void *pb)
{
    float a = *(const float *)pa, b = *(const float *)pb;
    int na = isnan(a), nb = isnan(b);
    if (na || nb) return na - nb;
    return (a > b) - (a < b);
}

/* torch.quantile(col, q, dim=0), linear interpolation, as called by the
 * reference at warpgbm/core.py:529-534.  Restates the published ATen
 * algorithm: sort (NaN last); rank = q * (n-1) in fp32; any NaN in the column
 * sets every rank to n-1; below = trunc(rank), above = ceil(rank),
 * w = rank - below; lerp(a, b, w) = |w| < 0.5 ? a + w*(b-a)
 *                                             : b - (b-a)*(1-w),
 * each branch with one fused multiply-add (matches torch's CPU and CUDA
 * builds; checked against torch here and on the GPU). */
void orc_quantile_edges(const float *col, int64_t n, int64_t stride,
                        const float *q, int nq, float *out)
{
    float *s = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    int has_nan = 0;
    for (int64_t i = 0; i < n; ++i) {
        s[i] = col[i * stride];
        if (isnan(s[i])) has_nan = 1;
    }
    qsort(s, (size_t)n, sizeof(float), cmp_float_nan_last);
    float last = (float)(n - 1);
    for (int j = 0; j < nq; ++j) {
        float rank = has_nan ? last : q[j] * last;
        int64_t lo = (int64_t)rank;
        int64_t hi = (int64_t)ceilf(rank);
        float w = rank - (float)lo;
        float a = s[lo], b = s[hi];
        float d = b - a;
        out[j] = (fabsf(w) < 0.5f) ? fmaf(w, d, a) : fmaf(-d, 1.0f - w, b);
    }
    free(s);
}

/* Every column of a row-major matrix, parallel over columns (the CPU
 * baseline's binning step; each column as orc_quantile_edges). */
void orc_quantile_edges_matrix(const float *X, int64_t n, int64_t F,
                               int64_t x_stride, const float *q, int nq,
                               float *out)
{
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t f = 0; f < F; ++f)
        orc_quantile_edges(X + f, n, x_stride, q, nq, out + f * nq);
}

/* ------------------------------------------------------------------------ */
/* Histograms                                                                */
/* ------------------------------------------------------------------------ */

/* warpgbm/cuda/histogram_kernel.cu:36-59 (+ launcher :63-104).
 * G[e][j][b] += g[row], H[e][j][b] += 1 for every row in samples (in order),
 * skipping bins outside [0, B).  Accumulates; the caller zero-fills
 * (warpgbm/core.py:544-549).  Parallel over feature blocks: every (e, j, b)
 * cell still sums its rows in sample order, so the result does not depend on
 * the thread count. */
void orc_hist_ref(const int8_t *bins, int64_t stride, const float *g,
                  const int32_t *samples, int64_t n, const int32_t *feats,
                  int k, const int32_t *era, int E, int B, float *G, float *H)
{
    (void)E;
#pragma omp parallel for schedule(dynamic, 1)
    for (int j0 = 0; j0 < k; j0 += 16) {
        int j1 = j0 + 16 < k ? j0 + 16 : k;
        for (int64_t i = 0; i < n; ++i) {
            int64_t row = samples[i];
            const int8_t *r = bins + row * stride;
            float gv = g[row];
            int64_t eb = (int64_t)era[row] * k;
            for (int j = j0; j < j1; ++j) {
                int b = r[feats[j]];
                if (b >= 0 && b < B) {
                    int64_t c = (eb + j) * B + b;
                    G[c] += gv;
                    H[c] += 1.0f;
                }
            }
        }
    }
}

/* Quantisation grid of the canonical histogram: s = 29 - e where
 * max|g| = m * 2^e, m in [0.5, 1) (frexp).  Every |q| = |rint(g*2^s)| <= 2^29,
 * so int64 sums of up to 2^33 rows cannot overflow.  s is clamped so that 2^s
 * and 2^-s are normal floats. */
int orc_quant_shift(float maxabs)
{
    if (!(maxabs > 0.0f) || isinf(maxabs)) return 0;
    int e;
    frexpf(maxabs, &e);
    int s = 29 - e;
    if (s > 126) s = 126;
    if (s < -99) s = -99;
    return s;
}

void orc_quantize(const float *g, int64_t n, int s, int32_t *q)
{
    float sc = ldexpf(1.0f, s);
    for (int64_t i = 0; i < n; ++i) q[i] = (int32_t)lrintf(g[i] * sc);
}

/* Canonical histogram: same cells as orc_hist_ref but exact int64 sums of q
 * and int32 counts, plus one extra slot b == B per (e, j) collecting rows
 * whose bin is negative (pre-binned input may hold them; the reference's
 * kernel skips them, histogram_kernel.cu:41, but they go left at every split,
 * core.py:629, so child totals need them).  Layout [E][k][B+1].
 * Accumulates. */
void orc_hist_q(const int8_t *bins, int64_t stride, const int32_t *q,
                const int32_t *samples, int64_t n, const int32_t *feats, int k,
                const int32_t *era, int E, int B, int64_t *G, int32_t *C)
{
    (void)E;
    int B1 = B + 1;
#pragma omp parallel for schedule(dynamic, 1)
    for (int j0 = 0; j0 < k; j0 += 16) {
        int j1 = j0 + 16 < k ? j0 + 16 : k;
        for (int64_t i = 0; i < n; ++i) {
            int64_t row = samples[i];
            const int8_t *r = bins + row * stride;
            int64_t qv = q[row];
            int64_t eb = (int64_t)era[row] * k;
            for (int j = j0; j < j1; ++j) {
                int b = r[feats[j]];
                int slot = b < 0 ? B : b;
                if (b < B) {
                    int64_t c = (eb + j) * B1 + slot;
                    G[c] += qv;
                    C[c] += 1;
                }
            }
        }
    }
}

/* Canonical dequantisation: G = float(sum) * 2^-s (int64 -> float rounds to
 * nearest, the scaling is exact), H = float(count).  Input [m][B+1], output
 * [m][B] (the negative-bin slot is dropped, as the reference never sees it). */
void orc_hist_dequant(const int64_t *G, const int32_t *C, int64_t m, int B,
                      int s, float *Gf, float *Hf)
{
    float inv = ldexpf(1.0f, -s);
    for (int64_t i = 0; i < m; ++i) {
        for (int b = 0; b < B; ++b) {
            Gf[i * B + b] = (float)G[i * (B + 1) + b] * inv;
            Hf[i * B + b] = (float)C[i * (B + 1) + b];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Split search                                                              */
/* ------------------------------------------------------------------------ */

/* warpgbm/cuda/best_split_kernel.cu:25-53, one (era, feature) at a time.
 * Totals summed sequentially over all B bins, prefix over b < B-1; gain and
 * direction only where both sides hold >= mcw rows, else 0.  eps = L2_reg
 * (core.py:566-575). */
void orc_split(const float *G, const float *H, int E, int k, int B, float mcw,
               float eps, float *gain, float *dir)
{
    for (int64_t ej = 0; ej < (int64_t)E * k; ++ej) {
        const float *g = G + ej * B, *h = H + ej * B;
        float GT = 0.0f, HT = 0.0f;
        for (int b = 0; b < B; ++b) {
            GT += g[b];
            HT += h[b];
        }
        float GL = 0.0f, HL = 0.0f;
        for (int b = 0; b < B - 1; ++b) {
            GL += g[b];
            HL += h[b];
            float GR = GT - GL, HR = HT - HL;
            float gn = 0.0f, dr = 0.0f;
            if (HL >= mcw && HR >= mcw) {
                float t1 = (GL * GL) / (HL + eps);
                float t2 = (GR * GR) / (HR + eps);
                float t3 = (GT * GT) / (HT + eps);
                gn = t1 + t2 - t3;
                float lv = GL / (HL + eps), rv = GR / (HR + eps);
                dr = (lv > rv) ? 1.0f : -1.0f;
            }
            gain[ej * (B - 1) + b] = gn;
            dir[ej * (B - 1) + b] = dr;
        }
    }
}

/* Directional era splitting, warpgbm/core.py:577-594.
 *   E == 1: crit = gain[0]; mask = crit > msg.
 *   E >  1: agree = |mean_e dir|, crit = mean_e gain,
 *           mask = (agree == max(agree)) & (crit > msg); max over all cells.
 * mean_mode 0: sequential fp32 sum over eras, then / E (torch CPU mean);
 * mean_mode 1: sequential fp32 sum over eras, times factor (torch CUDA mean
 *              multiplies by factor = float(k*(B-1)) / float(E*k*(B-1))).
 * Returns the flat index argmax over [k, B-1] (first maximum) or -1. */
int64_t orc_des_pick(const float *gain, const float *dir, int E, int k, int B,
                     float msg, int mean_mode, float factor)
{
    int64_t m = (int64_t)k * (B - 1);
    int64_t best = -1;
    float bestc = 0.0f;
    if (E == 1) {
        for (int64_t i = 0; i < m; ++i) {
            float c = gain[i];
            if (c > msg && (best < 0 || c > bestc)) {
                best = i;
                bestc = c;
            }
        }
        return best;
    }
    float *crit = (float *)malloc(sizeof(float) * (size_t)m);
    float *agree = (float *)malloc(sizeof(float) * (size_t)m);
    float amax = -INFINITY;
    for (int64_t i = 0; i < m; ++i) {
        float sg = 0.0f, sd = 0.0f;
        for (int e = 0; e < E; ++e) {
            sg += gain[(int64_t)e * m + i];
            sd += dir[(int64_t)e * m + i];
        }
        if (mean_mode == 0) {
            crit[i] = sg / (float)E;
            agree[i] = fabsf(sd / (float)E);
        } else {
            crit[i] = sg * factor;
            agree[i] = fabsf(sd * factor);
        }
        if (agree[i] > amax) amax = agree[i];
    }
    for (int64_t i = 0; i < m; ++i) {
        float c = crit[i];
        if (agree[i] == amax && c > msg && (best < 0 || c > bestc)) {
            best = i;
            bestc = c;
        }
    }
    free(crit);
    free(agree);
    return best;
}

/* ------------------------------------------------------------------------ */
/* Prediction                                                                */
/* ------------------------------------------------------------------------ */

/* warpgbm/cuda/predict.cu:17-44 over the flattened forest of
 * core.py:1215-1252 ([T][max_nodes][6]: feat, split_bin, left, right,
 * is_leaf, leaf_value).  Go left iff bin <= split_bin (signed int8).  Trees
 * are summed in tree order: out[i] += lr * leaf (one legal order of the
 * reference's atomics).  Accumulates into out. */
void orc_predict_flat(const int8_t *bins, int64_t n, int64_t stride,
                      const float *forest, int T, int max_nodes, float lr,
                      float *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const int8_t *r = bins + i * stride;
        float acc = out[i];
        for (int t = 0; t < T; ++t) {
            const float *tree = forest + (int64_t)t * max_nodes * 6;
            int node = 0;
            for (;;) {
                const float *nd = tree + node * 6;
                if (nd[4] > 0.5f) {
                    acc += lr * nd[5];
                    break;
                }
                int feat = (int)nd[0];
                int sb = (int)nd[1];
                node = (r[feat] <= sb) ? (int)nd[2] : (int)nd[3];
            }
        }
        out[i] = acc;
    }
}

int orc_num_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int t)
{
#ifdef _OPENMP
    if (t > 0) omp_set_num_threads(t);
#else
    (void)t;
#endif
}
