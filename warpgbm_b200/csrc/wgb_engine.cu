// Level-wise tree engine of warpgbm_b200 (sm_100a).
//
// Replaces the depth-first recursion of the reference (warpgbm/core.py:
// 543-658, 692-744) by one pass per tree level:
//
//   histogram  : all nodes that need a built histogram (root, then the smaller
//                child of every split -- core.py:636-643) in ONE launch over a
//                device-side chunk list; shared-memory privatised cells with
//                packed 64-bit (count << 47 | sum q) atomics, int64 flush;
//   subtract   : sibling = parent - built, exact, in place of the parent;
//   split      : per (node, feature) bin scan with the reference arithmetic
//                (best_split_kernel.cu:25-53) and the directional era rule
//                (core.py:577-594) as an arg-max reduction;
//   partition  : stable on-device partition of the row order (core.py:629-631)
//                with leaf updates of finished rows (core.py:598-621).
//
// No host synchronisation happens inside a tree: level sizes live on the
// device and every grid is sized by a host-known upper bound.
#include <cstdarg>
#include <cstdio>

#include "wgb_common.cuh"

namespace wgb {

static thread_local char g_err[1024];

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

// ====================================================================== //
// tree start                                                             //
// ====================================================================== //

__global__ void k_reset(float *maxabs, long long *rootsum) {
    *maxabs = 0.0f;
    *rootsum = 0;
}

// g = y - pred[:, cls] (regression, core.py:719) and max |g|.
__global__ void k_residual(const float *__restrict__ y, const float *__restrict__ pred, int K,
                           int cls, float *__restrict__ g, long long n, float *maxabs) {
    float m = 0.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v;
        if (y) {
            v = __fsub_rn(y[i], pred[i * K + cls]);
            g[i] = v;
        } else {
            v = g[i];
        }
        m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    __shared__ float sm[32];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (blockDim.x >> 5); ++i) m = fmaxf(m, sm[i]);
        // non-negative floats order like their bit patterns
        atomicMax(reinterpret_cast<int *>(maxabs), __float_as_int(m));
    }
}

__global__ void k_quantize(const float *__restrict__ g, int *__restrict__ qg, long long n,
                           const float *maxabs, int *shift_out, long long *rootsum) {
    int s = quant_shift(*maxabs);
    if (blockIdx.x == 0 && threadIdx.x == 0) *shift_out = s;
    float sc = pow2f(s);
    long long acc = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        int q = __float2int_rn(__fmul_rn(g[i], sc));
        qg[i] = q;
        acc += q;
    }
    acc = warp_sum(acc);
    __shared__ long long sm[32];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (blockDim.x >> 5); ++i) acc += sm[i];
        atomicAdd(reinterpret_cast<unsigned long long *>(rootsum), (unsigned long long)acc);
    }
}

__global__ void k_root(wgb_node *nodes, int *nn, int *nact, int D, long long n_local,
                       long long n_global, const long long *rootsum, const int *shift) {
    wgb_node r;
    r.sumq = *rootsum;
    r.count = n_global;
    r.lsumq = 0;
    r.lcount = 0;
    r.lstart = 0;
    r.lcnt = (int)n_local;
    r.slot = 0;
    r.built = 1;
    r.fpos = -1;
    r.bin = 0;
    r.child = -1;
    r.leaf = canon_leaf(r.sumq, r.count, pow2f(-*shift));
    nodes[0] = r;
    for (int d = 0; d <= D; ++d) {
        nn[d] = d == 0 ? 1 : 0;
        nact[d] = d == 0 ? (int)n_local : 0;
    }
}

// ====================================================================== //
// histogram build                                                        //
// ====================================================================== //

// Chunk list of level d: every built node's local rows cut into HIST_R-row
// pieces.  One block.
__global__ void __launch_bounds__(1024) k_chunk_plan(const wgb_node *__restrict__ lvl,
                                                     const int *nn_d, int4 *chunks,
                                                     int *nchunks, int cap) {
    __shared__ int s_cnt[1024];
    __shared__ int s_off[1025];
    __shared__ int s_base;
    int nnd = *nn_d;
    if (threadIdx.x == 0) s_base = 0;
    __syncthreads();
    for (int b0 = 0; b0 < nnd; b0 += 1024) {
        int i = b0 + threadIdx.x;
        int c = 0;
        if (i < nnd && lvl[i].built) c = (lvl[i].lcnt + HIST_R - 1) / HIST_R;
        s_cnt[threadIdx.x] = c;
        __syncthreads();
        if (threadIdx.x == 0) {
            int acc = s_base;
            for (int t = 0; t < 1024; ++t) {
                s_off[t] = acc;
                acc += s_cnt[t];
            }
            s_off[1024] = acc;
        }
        __syncthreads();
        int lo = s_off[0], hi = s_off[1024];
        for (int c2 = lo + threadIdx.x; c2 < hi; c2 += 1024) {
            // node of chunk c2: last t with s_off[t] <= c2 and s_cnt[t] > 0
            int a = 0, z = 1023;
            while (a < z) {
                int m = (a + z + 1) >> 1;
                if (s_off[m] <= c2) a = m; else z = m - 1;
            }
            while (s_cnt[a] == 0) --a;
            int node = b0 + a;
            int piece = c2 - s_off[a];
            int p0 = lvl[node].lstart + piece * HIST_R;
            int p1 = min(p0 + HIST_R, lvl[node].lstart + lvl[node].lcnt);
            if (c2 < cap) chunks[c2] = make_int4(node, p0, p1, 0);
        }
        __syncthreads();
        if (threadIdx.x == 0) s_base = hi;
        __syncthreads();
    }
    if (threadIdx.x == 0) *nchunks = min(s_base, cap);
}

// One CTA = one chunk (<= HIST_R rows of one node) x one 128-feature tile.
// Lane l of every warp owns features 4l..4l+3 of the tile (one 32-bit load
// per row); shared cells are [era window][slot b][j][lane] u64, so a warp's
// 64-bit atomics touch 32 consecutive words (2 wavefronts, no conflicts).
// Slot b == B collects negative bins; bins >= B are skipped
// (histogram_kernel.cu:41).  When q == nullptr the residual g is quantised
// on the fly with 2^shift (used by the drop-in wgb_compute_histogram3).
template <bool HAS_ERA>
__global__ void __launch_bounds__(HIST_THREADS) k_hist(
    const int8_t *__restrict__ bins, long long S, int F, const int *__restrict__ order,
    const int *__restrict__ q, const float *__restrict__ g, const int *shift,
    const int *__restrict__ era, const int *__restrict__ kpos, int k, int E, int B, int EW,
    const int4 *__restrict__ chunks, const int *nchunks, const wgb_node *__restrict__ lvl,
    long long *__restrict__ hg, int *__restrict__ hc, long long slot_elems, long long nrows) {
    extern __shared__ unsigned long long sh[];  // [EW][B+1][4][32]
    __shared__ int s_kp[HIST_FT];
    __shared__ int s_row[HIST_R];
    __shared__ int s_q[HIST_R];
    __shared__ int s_era[HIST_R];
    __shared__ int s_red[33];

    const int c = blockIdx.x;
    if (c >= *nchunks) return;
    const int f0 = blockIdx.y * HIST_FT;
    int any = 0;
    if (threadIdx.x < HIST_FT) {
        int f = f0 + threadIdx.x;
        int kp = f < F ? kpos[f] : -1;
        s_kp[threadIdx.x] = kp;
        any = kp >= 0;
    }
    if (!__syncthreads_or(any)) return;

    const int4 ch = chunks[c];
    const int cnt = ch.z - ch.y;
    const long long slot = lvl[ch.x].slot;
    float sc = 0.0f;
    if (!q) sc = pow2f(*shift);
    // rows outside [0, nrows) or eras outside [0, E) are skipped (only the
    // drop-in entry point can receive them; the engine never produces them)
    for (int i = threadIdx.x; i < cnt; i += HIST_THREADS) {
        int r = order[ch.y + i];
        bool ok = r >= 0 && r < nrows;
        int e = 0;
        if (HAS_ERA && ok) {
            e = era[r];
            ok = e >= 0 && e < E;
        }
        s_row[i] = ok ? r : -1;
        s_q[i] = ok ? (q ? q[r] : __float2int_rn(__fmul_rn(g[r], sc))) : 0;
        if (HAS_ERA) s_era[i] = ok ? e : INT_MAX;
    }
    __syncthreads();
    const bool aligned4 = (S & 3) == 0;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned vmask = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (s_kp[4 * lane + j] >= 0) vmask |= 1u << j;
    const int B1 = B + 1;
    const int win = B1 * HIST_FT;
    const int8_t *tile = bins + f0 + 4 * lane;

    int e_lo = 0;
    if (HAS_ERA) {
        int m = INT_MAX;
        for (int i = threadIdx.x; i < cnt; i += HIST_THREADS) m = min(m, s_era[i]);
        e_lo = block_min(m, s_red);
        if (e_lo == INT_MAX) return;  // no valid row (uniform)
    }
    for (;;) {
        for (int t = threadIdx.x; t < EW * win; t += HIST_THREADS) sh[t] = 0ull;
        __syncthreads();
        if (vmask) {
            for (int i0 = warp; i0 < cnt; i0 += 32) {
                uint32_t w[4];
                int ew[4];
                bool ok[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    int i = i0 + 8 * u;
                    ok[u] = i < cnt && s_row[i] >= 0;
                    ew[u] = 0;
                    if (HAS_ERA && ok[u]) {
                        int e = s_era[i] - e_lo;
                        ok[u] = e >= 0 && e < EW;
                        ew[u] = e;
                    }
                    w[u] = 0u;
                    if (ok[u]) {
                        const int8_t *src = tile + (long long)s_row[i] * S;
                        if (aligned4) {
                            w[u] = __ldg(reinterpret_cast<const uint32_t *>(src));
                        } else {
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                if ((vmask >> j) & 1u) w[u] |= (uint32_t)(uint8_t)__ldg(src + j) << (8 * j);
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (!ok[u]) continue;
                    unsigned long long pk = PACK_ONE + (unsigned long long)(long long)s_q[i0 + 8 * u];
                    unsigned long long *base = sh + ew[u] * win + lane;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        int b = (int)(int8_t)(w[u] >> (8 * j));
                        if (((vmask >> j) & 1u) && b < B) {
                            int sl = b < 0 ? B : b;
                            atomicAdd(base + (sl * 4 + j) * 32, pk);
                        }
                    }
                }
            }
        }
        __syncthreads();
        for (int t = threadIdx.x; t < EW * win; t += HIST_THREADS) {
            unsigned long long w = sh[t];
            if (w == 0ull) continue;
            long long cntv, gs;
            unpack_cell(w, cntv, gs);
            int ew = t / win, rem = t - ew * win;
            int sl = rem >> 7, jl = rem & 127;
            int fl = 4 * (jl & 31) + (jl >> 5);
            long long idx = slot * slot_elems + ((long long)(e_lo + ew) * k + s_kp[fl]) * B1 + sl;
            atomicAdd(reinterpret_cast<unsigned long long *>(hg + idx), (unsigned long long)gs);
            atomicAdd(hc + idx, (int)cntv);
        }
        if (!HAS_ERA) break;
        int m = INT_MAX;
        for (int i = threadIdx.x; i < cnt; i += HIST_THREADS)
            if (s_era[i] >= e_lo + EW) m = min(m, s_era[i]);
        m = block_min(m, s_red);  // also orders the flush before the next zeroing
        if (m == INT_MAX) break;
        e_lo = m;
    }
}

// sibling = parent - built, in place of the parent's slot (the sibling
// inherits it).  grid.y = pair.
__global__ void k_subtract(const wgb_node *__restrict__ lvl, const int *nn_d, long long *hg, int *hc,
                           long long slot_elems) {
    int p = blockIdx.y;
    if (2 * p + 1 >= *nn_d) return;
    const wgb_node &a = lvl[2 * p], &b = lvl[2 * p + 1];
    long long sb = a.built ? b.slot : a.slot;  // sibling (= parent) slot
    long long bb = a.built ? a.slot : b.slot;  // built slot
    long long *gs = hg + sb * slot_elems;
    const long long *gb = hg + bb * slot_elems;
    int *cs = hc + sb * slot_elems;
    const int *cb = hc + bb * slot_elems;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < slot_elems;
         i += (long long)gridDim.x * blockDim.x) {
        gs[i] -= gb[i];
        cs[i] -= cb[i];
    }
}

// ====================================================================== //
// split search                                                           //
// ====================================================================== //

// One thread = (node, feature position j): every era's bin scan with the
// reference arithmetic; E == 1 takes gain as the criterion, E > 1 the
// sequential fp32 era sum times `factor` (torch's CUDA mean) and the
// agreement |sum dir| (core.py:581-583).  Block arg-max -> cand[node][blk].
template <int NB, bool MULTI>
__global__ void __launch_bounds__(SPLIT_THREADS) k_split(
    const wgb_node *__restrict__ lvl, const int *nn_d, const long long *__restrict__ hg,
    const int *__restrict__ hc, long long slot_elems, int k, int E, int B, const int *shift,
    float mcw, float eps, float msg, float factor, int4 *cand, int nblk) {
    const int n = blockIdx.y;
    if (n >= *nn_d) return;
    const int j = blockIdx.x * SPLIT_THREADS + threadIdx.x;
    const float inv = pow2f(-*shift);
    const int B1 = B + 1, nb = B - 1;
    const long long slot = lvl[n].slot;
    Key best = key_none();
    if (j < k) {
        float cs[MULTI ? NB : 1];
        int ds[MULTI ? NB : 1];
        if (MULTI) {
#pragma unroll
            for (int b = 0; b < (MULTI ? NB : 1); ++b) {
                cs[b] = 0.0f;
                ds[b] = 0;
            }
        }
        for (int e = 0; e < E; ++e) {
            const long long off = slot * slot_elems + ((long long)e * k + j) * B1;
            const long long *gp = hg + off;
            const int *cp = hc + off;
            float GT = 0.0f, HT = 0.0f;
            for (int b = 0; b < B; ++b) {
                GT = __fadd_rn(GT, __fmul_rn(__ll2float_rn(__ldg(gp + b)), inv));
                HT = __fadd_rn(HT, __int2float_rn(__ldg(cp + b)));
            }
            float GL = 0.0f, HL = 0.0f;
#pragma unroll 4
            for (int b = 0; b < nb; ++b) {
                GL = __fadd_rn(GL, __fmul_rn(__ll2float_rn(__ldg(gp + b)), inv));
                HL = __fadd_rn(HL, __int2float_rn(__ldg(cp + b)));
                SplitEval r = eval_split(GL, HL, GT, HT, mcw, eps);
                if (MULTI) {
                    if (b < NB) {
                        cs[b] = __fadd_rn(cs[b], r.gain);
                        ds[b] += (int)r.dir;
                    }
                } else {
                    Key kk{0, r.gain > msg ? r.gain : -INFINITY, j * nb + b};
                    if (key_better(kk, best)) best = kk;
                }
            }
        }
        if (MULTI) {
#pragma unroll
            for (int b = 0; b < (MULTI ? NB : 1); ++b) {
                if (b < nb) {
                    float cr = __fmul_rn(cs[b], factor);
                    Key kk{abs(ds[b]), cr > msg ? cr : -INFINITY, j * nb + b};
                    if (key_better(kk, best)) best = kk;
                }
            }
        }
    }
    best = warp_key_max(best);
    __shared__ Key s_k[SPLIT_THREADS / 32];
    if ((threadIdx.x & 31) == 0) s_k[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < SPLIT_THREADS / 32; ++w)
            if (key_better(s_k[w], best)) best = s_k[w];
        cand[(long long)n * nblk + blockIdx.x] = make_int4(best.A, __float_as_int(best.c), best.idx, 0);
    }
}

// Per node: final arg-max, per-era gain of the chosen split (importance,
// core.py:624-627) and the exact left-child totals (bins <= bin plus the
// negative-bin slot, which always goes left).
__global__ void __launch_bounds__(256) k_split_final(
    wgb_node *__restrict__ lvl, const int *nn_d, const long long *__restrict__ hg,
    const int *__restrict__ hc, long long slot_elems, int k, int E, int B, const int *shift,
    float mcw, float eps, const int4 *__restrict__ cand, int nblk, float *era_gain) {
    const int n = blockIdx.x;
    if (n >= *nn_d) return;
    __shared__ Key s_best;
    __shared__ long long s_c[8], s_g[8];
    if (threadIdx.x == 0) {
        Key best = key_none();
        for (int b = 0; b < nblk; ++b) {
            int4 v = cand[(long long)n * nblk + b];
            Key kk{v.x, __int_as_float(v.y), v.z};
            if (key_better(kk, best)) best = kk;
        }
        s_best = best;
    }
    __syncthreads();
    const Key best = s_best;
    wgb_node &nd = lvl[n];
    if (!(best.c > -INFINITY)) {
        if (threadIdx.x == 0) {
            nd.fpos = -1;
            nd.lsumq = 0;
            nd.lcount = 0;
        }
        return;
    }
    const int nb = B - 1, B1 = B + 1;
    const int fpos = best.idx / nb, bin = best.idx - fpos * nb;
    const float inv = pow2f(-*shift);
    const long long slot = nd.slot;
    long long lc = 0, ls = 0;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const long long off = slot * slot_elems + ((long long)e * k + fpos) * B1;
        const long long *gp = hg + off;
        const int *cp = hc + off;
        float GT = 0.0f, HT = 0.0f, GL = 0.0f, HL = 0.0f;
        for (int b = 0; b < B; ++b) {
            float gv = __fmul_rn(__ll2float_rn(gp[b]), inv);
            float hv = __int2float_rn(cp[b]);
            GT = __fadd_rn(GT, gv);
            HT = __fadd_rn(HT, hv);
            if (b <= bin) {
                GL = __fadd_rn(GL, gv);
                HL = __fadd_rn(HL, hv);
                lc += cp[b];
                ls += gp[b];
            }
        }
        lc += cp[B];
        ls += gp[B];
        era_gain[(long long)n * E + e] = eval_split(GL, HL, GT, HT, mcw, eps).gain;
    }
    lc = warp_sum(lc);
    ls = warp_sum(ls);
    if ((threadIdx.x & 31) == 0) {
        s_c[threadIdx.x >> 5] = lc;
        s_g[threadIdx.x >> 5] = ls;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            lc += s_c[w];
            ls += s_g[w];
        }
        nd.fpos = fpos;
        nd.bin = bin;
        nd.lcount = lc;
        nd.lsumq = ls;
    }
}

// Next level's node records (one block): children of splitting nodes in
// node order, smaller child built (left on ties, core.py:636), the built
// child in a fresh slot 2^d + r, the sibling in the parent's slot.
__global__ void __launch_bounds__(1024) k_plan_next(wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt,
                                                    int *nn, int d, const int *shift) {
    __shared__ int s_f[1024];
    __shared__ int s_base;
    const int nnd = nn[d];
    const float inv = pow2f(-*shift);
    if (threadIdx.x == 0) s_base = 0;
    __syncthreads();
    for (int b0 = 0; b0 < nnd; b0 += 1024) {
        int i = b0 + threadIdx.x;
        int f = (i < nnd && lvl[i].fpos >= 0) ? 1 : 0;
        s_f[threadIdx.x] = f;
        __syncthreads();
        // inclusive scan (Hillis-Steele)
        for (int o = 1; o < 1024; o <<= 1) {
            int v = threadIdx.x >= o ? s_f[threadIdx.x - o] : 0;
            __syncthreads();
            s_f[threadIdx.x] += v;
            __syncthreads();
        }
        int r = s_base + s_f[threadIdx.x] - f;
        if (f) {
            wgb_node &p = lvl[i];
            p.child = 2 * r;
            long long cl = p.lcount, cr = p.count - p.lcount;
            long long sl = p.lsumq, sr = p.sumq - p.lsumq;
            int builtL = cl <= cr;
            int fresh = (1 << d) + r;
            wgb_node L, R;
            L.sumq = sl; L.count = cl; R.sumq = sr; R.count = cr;
            L.lsumq = R.lsumq = 0; L.lcount = R.lcount = 0;
            L.lstart = R.lstart = 0; L.lcnt = R.lcnt = 0;
            L.built = builtL; R.built = !builtL;
            L.slot = builtL ? fresh : p.slot;
            R.slot = builtL ? p.slot : fresh;
            L.fpos = R.fpos = -1; L.bin = R.bin = 0; L.child = R.child = -1;
            L.leaf = canon_leaf(sl, cl, inv);
            R.leaf = canon_leaf(sr, cr, inv);
            nxt[2 * r] = L;
            nxt[2 * r + 1] = R;
        } else if (i < nnd) {
            lvl[i].child = -1;
        }
        __syncthreads();
        if (threadIdx.x == 1023) s_base = r + f;
        __syncthreads();
    }
    if (threadIdx.x == 0) nn[d + 1] = 2 * s_base;
}

// ====================================================================== //
// partition                                                              //
// ====================================================================== //

// flag per position: 1 left, 0 right, 2 node is a leaf; left count per tile.
__global__ void __launch_bounds__(PART_THREADS) k_flags(
    const wgb_node *__restrict__ lvl, const int *nact_d, const int *__restrict__ order,
    const int *__restrict__ posnode, const int8_t *__restrict__ bins, long long S,
    const int *__restrict__ feats, uint8_t *flags, int *tile_cnt) {
    const int nact = *nact_d;
    const long long t0 = (long long)blockIdx.x * PART_TILE;
    int cnt = 0;
    for (int i = threadIdx.x; i < PART_TILE; i += PART_THREADS) {
        long long p = t0 + i;
        if (p >= nact) break;
        int n = posnode ? posnode[p] : 0;
        int fp = lvl[n].fpos;
        uint8_t fl = 2;
        if (fp >= 0) {
            int row = order[p];
            int b = bins[(long long)row * S + feats[fp]];
            fl = b <= lvl[n].bin ? 1 : 0;
            cnt += fl;
        }
        flags[p] = fl;
    }
    cnt = warp_sum(cnt);
    __shared__ int sm[PART_THREADS / 32];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < PART_THREADS / 32; ++w) cnt += sm[w];
        tile_cnt[blockIdx.x] = cnt;
    }
}

// exclusive scan of tile counts (one block)
__global__ void __launch_bounds__(1024) k_scan_tiles(const int *tile_cnt, int *tile_off, int ntiles) {
    __shared__ int s[1024];
    __shared__ int s_base;
    if (threadIdx.x == 0) s_base = 0;
    __syncthreads();
    for (int b0 = 0; b0 < ntiles; b0 += 1024) {
        int i = b0 + threadIdx.x;
        int v = i < ntiles ? tile_cnt[i] : 0;
        s[threadIdx.x] = v;
        __syncthreads();
        for (int o = 1; o < 1024; o <<= 1) {
            int t = threadIdx.x >= o ? s[threadIdx.x - o] : 0;
            __syncthreads();
            s[threadIdx.x] += t;
            __syncthreads();
        }
        if (i < ntiles) tile_off[i] = s_base + s[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == 1023) s_base += s[1023];
        __syncthreads();
    }
    if (threadIdx.x == 0) tile_off[ntiles] = s_base;  // total, for p == end
}

// lefts before position p (p may equal nact)
__device__ __forceinline__ int lefts_before(long long p, const uint8_t *flags, const int *tile_off,
                                            int lane) {
    long long t = p / PART_TILE;
    long long a = t * PART_TILE;
    int c = 0;
    for (long long i = a + lane; i < p; i += 32) c += flags[i] == 1;
    c = warp_sum(c);
    return tile_off[t] + c;
}

// Per splitting node: local left count and the start of its children in the
// next order; children's local segments; next level's active rows.
__global__ void __launch_bounds__(1024) k_node_offsets(wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt,
                                                       const int *nn, int *nact, int d,
                                                       const uint8_t *flags, const int *tile_off,
                                                       int4 *part) {
    const int nnd = nn[d];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int n = warp; n < nnd; n += 32) {
        const wgb_node &nd = lvl[n];
        if (nd.fpos < 0) continue;
        int a = lefts_before(nd.lstart, flags, tile_off, lane);
        int b = lefts_before((long long)nd.lstart + nd.lcnt, flags, tile_off, lane);
        if (lane == 0) part[n] = make_int4(a, 0, b - a, 0);
    }
    __syncthreads();
    __shared__ int s[1024];
    __shared__ int s_base;
    if (threadIdx.x == 0) s_base = 0;
    __syncthreads();
    for (int b0 = 0; b0 < nnd; b0 += 1024) {
        int i = b0 + threadIdx.x;
        int v = (i < nnd && lvl[i].fpos >= 0) ? lvl[i].lcnt : 0;
        s[threadIdx.x] = v;
        __syncthreads();
        for (int o = 1; o < 1024; o <<= 1) {
            int t = threadIdx.x >= o ? s[threadIdx.x - o] : 0;
            __syncthreads();
            s[threadIdx.x] += t;
            __syncthreads();
        }
        if (v > 0 || (i < nnd && lvl[i].fpos >= 0)) {
            int ns = s_base + s[threadIdx.x] - v;
            int4 pr = part[i];
            pr.y = ns;
            part[i] = pr;
            int c = lvl[i].child;
            nxt[c].lstart = ns;
            nxt[c].lcnt = pr.z;
            nxt[c + 1].lstart = ns + pr.z;
            nxt[c + 1].lcnt = v - pr.z;
        }
        __syncthreads();
        if (threadIdx.x == 1023) s_base += s[1023];
        __syncthreads();
    }
    if (threadIdx.x == 0) nact[d + 1] = s_base;
}

// Scatter rows into the next level's order; finished rows get their leaf
// update pred += lr * leaf (core.py:598-621).
__global__ void __launch_bounds__(PART_THREADS) k_scatter(
    const wgb_node *__restrict__ lvl, const int *nact_d, const int *__restrict__ order,
    const int *__restrict__ posnode, const uint8_t *__restrict__ flags,
    const int *__restrict__ tile_off, const int4 *__restrict__ part, int *__restrict__ order_next,
    int *__restrict__ posnode_next, float *__restrict__ pred, int K, int cls, float lr, long long N) {
    constexpr int IPT = PART_TILE / PART_THREADS;  // 8 consecutive positions per thread
    const int nact = *nact_d;
    const long long p0 = (long long)blockIdx.x * PART_TILE + threadIdx.x * IPT;
    uint8_t f[IPT];
    int c = 0;
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        f[u] = (p0 + u < nact) ? flags[p0 + u] : 3;
        c += f[u] == 1;
    }
    // block exclusive scan of c
    __shared__ int sw[PART_THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) sw[warp] = incl;
    __syncthreads();
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += sw[w];
    int lp = tile_off[blockIdx.x] + wbase + incl - c;
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        if (f[u] == 3) break;
        long long p = p0 + u;
        int n = posnode ? posnode[p] : 0;
        const wgb_node &nd = lvl[n];
        int row = order[p];
        if (f[u] == 2) {
            float *pp = pred + (long long)row * K + cls;
            *pp = __fadd_rn(*pp, __fmul_rn(lr, nd.leaf));
        } else {
            int4 pr = part[n];
            int lb = lp - pr.x;  // lefts before p inside the node
            int np;
            int child;
            if (f[u] == 1) {
                np = pr.y + lb;
                child = nd.child;
            } else {
                np = pr.y + pr.z + (int)(p - nd.lstart) - lb;
                child = nd.child + 1;
            }
            if (np >= 0 && np < N) {  // always true for consistent offsets; guards memory
                order_next[np] = row;
                posnode_next[np] = child;
            }
            if (f[u] == 1) ++lp;
        }
    }
}

__global__ void k_finish(const wgb_node *__restrict__ lvl, const int *nact_d, const int *__restrict__ order,
                         const int *__restrict__ posnode, float *__restrict__ pred, int K, int cls,
                         float lr) {
    const int nact = *nact_d;
    for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < nact;
         p += (long long)gridDim.x * blockDim.x) {
        int n = posnode ? posnode[p] : 0;
        int row = order[p];
        float *pp = pred + (long long)row * K + cls;
        *pp = __fadd_rn(*pp, __fmul_rn(lr, lvl[n].leaf));
    }
}

// ====================================================================== //
// host side                                                              //
// ====================================================================== //

static inline long long *LL(int64_t *p) { return reinterpret_cast<long long *>(p); }
static inline wgb_node *level_nodes(const wgb_ws *ws, int d) { return ws->nodes + ((1 << d) - 1); }
static inline const int *level_order(const wgb_ws *ws, int d) {
    return d == 0 ? ws->root_order : ws->order[(d - 1) & 1];
}
static inline const int *level_posnode(const wgb_ws *ws, int d) {
    return d == 0 ? nullptr : ws->posnode[(d - 1) & 1];
}
static inline long long slot_elems(const wgb_ws *ws) { return (long long)ws->E * ws->k * (ws->B + 1); }

static int grid_for(long long n, int threads, int cap = 148 * 16) {
    long long b = (n + threads - 1) / threads;
    if (b < 1) b = 1;
    return (int)(b < cap ? b : cap);
}

size_t hist_smem_bytes(int B, int EW) { return (size_t)EW * (B + 1) * HIST_FT * 8; }

}  // namespace wgb

using namespace wgb;

extern "C" {

const char *wgb_last_error(void) { return wgb::g_err; }
int wgb_version(void) { return 1; }
int32_t wgb_sizeof_node(void) { return (int32_t)sizeof(wgb_node); }
int32_t wgb_sizeof_ws(void) { return (int32_t)sizeof(wgb_ws); }

void wgb_built_slots(int32_t d, int32_t *first, int32_t *count) {
    if (d <= 0) {
        *first = 0;
        *count = 1;
    } else {
        *first = 1 << (d - 1);
        *count = 1 << (d - 1);
    }
}

static int check_ws(const wgb_ws *ws) {
    WGB_CHECK_ARG(ws != nullptr, "workspace is NULL");
    WGB_CHECK_ARG(ws->B >= 2 && ws->B <= 127, "num_bins must be in [2, 127], got %d", ws->B);
    WGB_CHECK_ARG(ws->D >= 1 && ws->D <= 24, "max_depth must be in [1, 24], got %d", ws->D);
    WGB_CHECK_ARG(ws->k >= 1 && ws->k <= ws->F, "k must be in [1, F]");
    WGB_CHECK_ARG(ws->E >= 1, "num_eras must be >= 1");
    WGB_CHECK_ARG(ws->N >= 0 && ws->N < (1ll << 31), "rows per rank must be < 2^31");
    WGB_CHECK_ARG(ws->S >= ws->F && ws->S % 4 == 0, "bins row stride must be >= F and a multiple of 4");
    WGB_CHECK_ARG(ws->hist_ew >= 1, "hist_ew must be >= 1");
    return WGB_OK;
}

int wgb_tree_reset(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    k_reset<<<1, 1, 0, as_stream(stream)>>>(ws->maxabs, LL(ws->rootsum));
    WGB_LAUNCHED("k_reset");
    return WGB_OK;
}

int wgb_tree_residual(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    if (ws->N == 0) return WGB_OK;
    k_residual<<<grid_for(ws->N, 256), 256, 0, as_stream(stream)>>>(ws->y, ws->pred, ws->K, ws->cls,
                                                                     ws->g, ws->N, ws->maxabs);
    WGB_LAUNCHED("k_residual");
    return WGB_OK;
}

int wgb_tree_quantize(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    k_quantize<<<grid_for(ws->N, 256), 256, 0, as_stream(stream)>>>(ws->g, ws->qg, ws->N, ws->maxabs,
                                                                     ws->shift, LL(ws->rootsum));
    WGB_LAUNCHED("k_quantize");
    return WGB_OK;
}

int wgb_tree_root(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    k_root<<<1, 1, 0, as_stream(stream)>>>(ws->nodes, ws->nn, ws->nact, ws->D, ws->N, ws->N_global,
                                           LL(ws->rootsum), ws->shift);
    WGB_LAUNCHED("k_root");
    return WGB_OK;
}

int wgb_level_hist(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    cudaStream_t st = as_stream(stream);
    int first, count;
    wgb_built_slots(d, &first, &count);
    const long long se = slot_elems(ws);
    WGB_CUDA(cudaMemsetAsync(ws->hg + (long long)first * se, 0, sizeof(int64_t) * se * count, st));
    WGB_CUDA(cudaMemsetAsync(ws->hc + (long long)first * se, 0, sizeof(int32_t) * se * count, st));
    wgb_node *lvl = level_nodes(ws, d);
    k_chunk_plan<<<1, 1024, 0, st>>>(lvl, ws->nn + d, reinterpret_cast<int4 *>(ws->chunks),
                                     ws->nchunks, ws->chunk_cap);
    WGB_LAUNCHED("k_chunk_plan");
    if (ws->N == 0) return WGB_OK;
    long long max_chunks = (ws->N + HIST_R - 1) / HIST_R + count;
    if (max_chunks > ws->chunk_cap) max_chunks = ws->chunk_cap;
    dim3 grid((unsigned)max_chunks, (unsigned)((ws->F + HIST_FT - 1) / HIST_FT));
    int EW = ws->E == 1 ? 1 : ws->hist_ew;
    size_t smem = hist_smem_bytes(ws->B, EW);
    const int *ord = level_order(ws, d);
    if (ws->E == 1) {
        WGB_CUDA(cudaFuncSetAttribute(k_hist<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_hist<false><<<grid, HIST_THREADS, smem, st>>>(
            ws->bins, ws->S, ws->F, ord, ws->qg, nullptr, nullptr, nullptr, ws->kpos, ws->k, ws->E, ws->B,
            1, reinterpret_cast<const int4 *>(ws->chunks), ws->nchunks, lvl, LL(ws->hg), ws->hc, se, ws->N);
    } else {
        WGB_CUDA(cudaFuncSetAttribute(k_hist<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_hist<true><<<grid, HIST_THREADS, smem, st>>>(
            ws->bins, ws->S, ws->F, ord, ws->qg, nullptr, nullptr, ws->era, ws->kpos, ws->k, ws->E, ws->B,
            EW, reinterpret_cast<const int4 *>(ws->chunks), ws->nchunks, lvl, LL(ws->hg), ws->hc, se, ws->N);
    }
    WGB_LAUNCHED("k_hist");
    return WGB_OK;
}

int wgb_level_split(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    cudaStream_t st = as_stream(stream);
    const long long se = slot_elems(ws);
    wgb_node *lvl = level_nodes(ws, d);
    const int cap = 1 << d;
    if (d > 0) {
        int bx = (int)((se + 255) / 256);
        if (bx > 64) bx = 64;
        dim3 g(bx, cap / 2);
        k_subtract<<<g, 256, 0, st>>>(lvl, ws->nn + d, LL(ws->hg), ws->hc, se);
        WGB_LAUNCHED("k_subtract");
    }
    const int nblk = (ws->k + SPLIT_THREADS - 1) / SPLIT_THREADS;
    WGB_CHECK_ARG(nblk <= ws->ncand_blk, "candidate buffer too small");
    dim3 g(nblk, cap);
    const int nb = ws->B - 1;
    int4 *cand = reinterpret_cast<int4 *>(ws->cand);
#define WGB_SPLIT_ARGS                                                                       \
    lvl, ws->nn + d, LL(ws->hg), ws->hc, se, ws->k, ws->E, ws->B, ws->shift, ws->mcw, ws->eps, \
        ws->msg, ws->mean_factor, cand, nblk
    if (ws->E == 1) {
        k_split<1, false><<<g, SPLIT_THREADS, 0, st>>>(WGB_SPLIT_ARGS);
    } else if (nb <= 8) {
        k_split<8, true><<<g, SPLIT_THREADS, 0, st>>>(WGB_SPLIT_ARGS);
    } else if (nb <= 32) {
        k_split<32, true><<<g, SPLIT_THREADS, 0, st>>>(WGB_SPLIT_ARGS);
    } else {
        k_split<128, true><<<g, SPLIT_THREADS, 0, st>>>(WGB_SPLIT_ARGS);
    }
#undef WGB_SPLIT_ARGS
    WGB_LAUNCHED("k_split");
    float *eg = ws->era_gain + (long long)((1 << d) - 1) * ws->E;
    k_split_final<<<cap, 256, 0, st>>>(lvl, ws->nn + d, LL(ws->hg), ws->hc, se, ws->k, ws->E, ws->B,
                                       ws->shift, ws->mcw, ws->eps, cand, nblk, eg);
    WGB_LAUNCHED("k_split_final");
    k_plan_next<<<1, 1024, 0, st>>>(lvl, level_nodes(ws, d + 1), ws->nn, d, ws->shift);
    WGB_LAUNCHED("k_plan_next");
    return WGB_OK;
}

int wgb_level_partition(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    if (ws->N == 0) return WGB_OK;
    cudaStream_t st = as_stream(stream);
    wgb_node *lvl = level_nodes(ws, d);
    const int ntiles = (int)((ws->N + PART_TILE - 1) / PART_TILE);
    WGB_CHECK_ARG(ntiles <= ws->ntiles, "tile buffer too small");
    const int *ord = level_order(ws, d);
    const int *pn = level_posnode(ws, d);
    k_flags<<<ntiles, PART_THREADS, 0, st>>>(lvl, ws->nact + d, ord, pn, ws->bins, ws->S, ws->feats,
                                              ws->flags, ws->tile_cnt);
    WGB_LAUNCHED("k_flags");
    k_scan_tiles<<<1, 1024, 0, st>>>(ws->tile_cnt, ws->tile_off, ntiles);
    WGB_LAUNCHED("k_scan_tiles");
    int4 *part = reinterpret_cast<int4 *>(ws->part);
    k_node_offsets<<<1, 1024, 0, st>>>(lvl, level_nodes(ws, d + 1), ws->nn, ws->nact, d, ws->flags,
                                       ws->tile_off, part);
    WGB_LAUNCHED("k_node_offsets");
    k_scatter<<<ntiles, PART_THREADS, 0, st>>>(lvl, ws->nact + d, ord, pn, ws->flags, ws->tile_off, part,
                                                ws->order[d & 1], ws->posnode[d & 1], ws->pred, ws->K,
                                                ws->cls, ws->lr, ws->N);
    WGB_LAUNCHED("k_scatter");
    return WGB_OK;
}

int wgb_tree_finish(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    if (ws->N == 0) return WGB_OK;
    const int D = ws->D;
    k_finish<<<grid_for(ws->N, 256), 256, 0, as_stream(stream)>>>(
        level_nodes(ws, D), ws->nact + D, level_order(ws, D), level_posnode(ws, D), ws->pred, ws->K,
        ws->cls, ws->lr);
    WGB_LAUNCHED("k_finish");
    return WGB_OK;
}

}  // extern "C"
