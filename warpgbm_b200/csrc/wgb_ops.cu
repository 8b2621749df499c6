// Binning, prediction and the reference-compatible entry points of
// warpgbm_b200 (sm_100a).  Compiled in the same translation unit as
// wgb_engine.cu (see wgb_lib.cu): it reuses k_hist and k_chunk_plan.

namespace wgb {

// ====================================================================== //
// binning                                                                //
// ====================================================================== //

// Row-major float [n][F] -> int8 [n][out_stride] in one pass.  CTA = 256
// rows x 128 features; lane l of a warp bins features l, l+32, l+64, l+96 of
// one row (four coalesced 128-byte loads, four 32-byte stores).  Per element
// the reference scan (binner.cu:20-23) counts leading edges with
// x >= edge, stopping at the first failure.  When a feature's edges are
// non-decreasing (always true for quantile edges; all-NaN edges included,
// where every comparison fails) that count is found by binary search; any
// other edge list keeps the linear scan.  Edges sit in shared memory
// edge-major ([b][128]), so the 32 lanes of a warp always read 32 distinct
// banks, whatever edge each one is looking at.
constexpr int BIN_FT = 128, BIN_ROWS = 256;

// NB > 0: num_bins - 1 == NB == 2^k - 1 at compile time (the search needs no
// bounds test and unrolls); NB == 0: any num_bins.
template <int NB>
__global__ void __launch_bounds__(256) k_bin_matrix(const float *__restrict__ X, long long n, int F,
                                                    long long xs, const float *__restrict__ edges,
                                                    int nb, int8_t *__restrict__ out, long long os) {
    extern __shared__ float s_e[];  // [nb][BIN_FT]
    __shared__ int s_mono[BIN_FT];
    const int f0 = blockIdx.y * BIN_FT;
    for (int t = threadIdx.x; t < BIN_FT * nb; t += blockDim.x) {
        const int fl = t / nb, b = t - fl * nb;
        const int f = f0 + fl;
        s_e[b * BIN_FT + fl] = f < F ? edges[(long long)f * nb + b] : 0.0f;
    }
    __syncthreads();
    for (int fl = threadIdx.x; fl < BIN_FT; fl += blockDim.x) {
        bool all_nan = true, mono = true;
        for (int b = 0; b < nb; ++b) all_nan &= isnan(s_e[b * BIN_FT + fl]);
        for (int b = 0; b + 1 < nb; ++b) mono &= s_e[b * BIN_FT + fl] <= s_e[(b + 1) * BIN_FT + fl];
        s_mono[fl] = all_nan || mono;
    }
    __syncthreads();
    const int tl = threadIdx.x & 31;
    bool mono[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) mono[j] = s_mono[tl + 32 * j];
    int top = 1;
    while (top * 2 <= nb) top *= 2;  // largest power of two <= nb
    const long long r0 = (long long)blockIdx.x * BIN_ROWS;
    for (int rr = threadIdx.x >> 5; rr < BIN_ROWS; rr += blockDim.x >> 5) {
        const long long r = r0 + rr;
        if (r >= n) break;
        const float *xr = X + r * xs;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int f = f0 + tl + 32 * j;
            v[j] = f < F ? __ldg(xr + f) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int f = f0 + tl + 32 * j;
            if (f >= os) continue;
            const float *e = s_e + tl + 32 * j;
            int b = 0;
            if (f < F) {
                if (NB > 0 && mono[j]) {
#pragma unroll
                    for (int step = (NB + 1) / 2; step >= 1; step >>= 1) {
                        const int c = b + step;  // <= NB for every path when NB = 2^k - 1
                        b = v[j] >= e[(c - 1) * BIN_FT] ? c : b;
                    }
                } else if (mono[j]) {
                    for (int step = top; step >= 1; step >>= 1)
                        if (b + step <= nb && v[j] >= e[(b + step - 1) * BIN_FT]) b += step;
                } else {
                    while (b < nb && v[j] >= e[b * BIN_FT]) ++b;
                }
            }
            out[r * os + f] = (int8_t)b;
        }
    }
}

// Pre-binned int8 input (core.py:499-517), one pass: copy X [n][F] into the
// padded bin matrix [n][S] (zeros past F), per-column maxima (the reference's
// pre-binned test is max(X, axis=0) < num_bins) and the global minimum and
// maximum (bins outside [0, B) need the checked histogram path).  CTA = 256
// rows x 128 columns, lane l of a warp owns columns 4l..4l+3 of one row.
__global__ void __launch_bounds__(256) k_prebinned(const int8_t *__restrict__ X, long long n, int F,
                                                   long long xs, int8_t *__restrict__ out, long long os,
                                                   int *__restrict__ colmax, int *__restrict__ minmax) {
    const int tl = threadIdx.x & 31;
    const int f = blockIdx.y * BIN_FT + 4 * tl;
    const bool in_row = f < os;  // lanes past the row stay for the warp reductions below
    const bool vec = (xs % 4 == 0) && (f + 4 <= F);
    int cmax[4] = {INT_MIN, INT_MIN, INT_MIN, INT_MIN};
    int gmin = INT_MAX, gmax = INT_MIN;
    const long long r0 = (long long)blockIdx.x * BIN_ROWS;
    constexpr int RU = 8;  // rows in flight per warp
    const int nw = blockDim.x >> 5;
    for (int rr = threadIdx.x >> 5; in_row && rr < BIN_ROWS; rr += nw * RU) {
        uint32_t w[RU];
#pragma unroll
        for (int u = 0; u < RU; ++u) {
            const long long r = r0 + rr + u * nw;
            w[u] = 0;
            if (rr + u * nw < BIN_ROWS && r < n) {
                const int8_t *xr = X + r * xs;
                if (vec) {
                    w[u] = __ldg(reinterpret_cast<const uint32_t *>(xr + f));
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (f + j < F) w[u] |= (uint32_t)(uint8_t)__ldg(xr + f + j) << (8 * j);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < RU; ++u) {
            const long long r = r0 + rr + u * nw;
            if (rr + u * nw >= BIN_ROWS || r >= n) break;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (f + j < F) {
                    const int v = (int)(int8_t)(w[u] >> (8 * j));
                    cmax[j] = max(cmax[j], v);
                    gmin = min(gmin, v);
                    gmax = max(gmax, v);
                }
            }
            *reinterpret_cast<uint32_t *>(out + r * os + f) = w[u];
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (f + j < F && cmax[j] != INT_MIN) atomicMax(colmax + f + j, cmax[j]);
    gmin = warp_min(gmin);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) gmax = max(gmax, __shfl_xor_sync(0xffffffffu, gmax, o));
    if (tl == 0 && gmax != INT_MIN) {
        atomicMin(minmax, gmin);
        atomicMax(minmax + 1, gmax);
    }
}

__global__ void k_bin_column(const float *__restrict__ X, long long n, const float *__restrict__ e,
                             int nb, int8_t *__restrict__ out) {
    long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = X[i];
    int b = 0;
    while (b < nb && v >= e[b]) ++b;
    out[i] = (int8_t)b;
}

// ====================================================================== //
// prediction                                                             //
// ====================================================================== //

// Packed forest: node = int2; internal {feature >= 0, bin | right << 8}
// (left child = node + 1, pre-order), leaf {-1, float bits of value}.
// One thread per row.  STAGED: the CTA stages its rows' bins in shared
// memory (row stride S + 4 bytes: the same feature of consecutive rows falls
// in consecutive banks); otherwise rows are read from global memory (rows
// too wide to stage).  Trees are walked PRED_G at a time (independent chains
// for latency hiding) and their leaves added strictly in tree order.  Any
// depth; the heap predictor below is the fast path for depth <= 12.
constexpr int PRED_ROWS = 128, PRED_G = 4;

template <bool STAGED>
__global__ void __launch_bounds__(PRED_ROWS) k_predict_packed(
    const int8_t *__restrict__ bins, long long n, long long S, const int2 *__restrict__ nodes,
    const int *__restrict__ tree_off, int T, int K, float lr, float *__restrict__ out) {
    extern __shared__ uint32_t s_rows[];
    const int SW = (int)(S / 4) + 1;  // words per staged row
    const int RP = blockDim.x;        // rows per CTA (<= PRED_ROWS, fewer for wide rows)
    const long long r0 = (long long)blockIdx.x * RP;
    const int nrows = (int)min((long long)RP, n - r0);
    if (STAGED) {
        for (int t = threadIdx.x; t < nrows * (SW - 1); t += RP) {
            int rr = t / (SW - 1), w = t - rr * (SW - 1);
            s_rows[rr * SW + w] = __ldg(reinterpret_cast<const uint32_t *>(bins + (r0 + rr) * S) + w);
        }
        __syncthreads();
    }
    if (threadIdx.x >= nrows) return;
    const long long row = r0 + threadIdx.x;
    const int8_t *myrow = STAGED ? reinterpret_cast<const int8_t *>(s_rows + threadIdx.x * SW) : bins + row * S;
    for (int c = 0; c < K; ++c) {
        float acc = out[row * K + c];
        for (int t0 = c; t0 < T; t0 += K * PRED_G) {
            float val[PRED_G];
            int node[PRED_G], base[PRED_G], lim[PRED_G];
            bool live[PRED_G];
#pragma unroll
            for (int u = 0; u < PRED_G; ++u) {
                int t = t0 + u * K;
                live[u] = t < T;
                base[u] = live[u] ? tree_off[t] : 0;
                lim[u] = live[u] ? tree_off[t + 1] - base[u] : 0;
                node[u] = 0;
                val[u] = 0.0f;
            }
            bool any = true;
            while (any) {
                any = false;
#pragma unroll
                for (int u = 0; u < PRED_G; ++u) {
                    if (!live[u]) continue;
                    int2 nd = __ldg(nodes + base[u] + node[u]);
                    if (nd.x < 0) {
                        val[u] = __int_as_float(nd.y);
                        live[u] = false;
                        continue;
                    }
                    if (nd.x >= S) {  // malformed feature index
                        val[u] = __int_as_float(0x7fc00000);
                        live[u] = false;
                        continue;
                    }
                    int b = (int)(STAGED ? myrow[nd.x] : __ldg(myrow + nd.x));
                    int nxt = (b <= (nd.y & 0xff)) ? node[u] + 1 : (nd.y >> 8);
                    // pre-order ids only grow; anything else is a malformed tree
                    if (nxt <= node[u] || nxt >= lim[u]) {
                        val[u] = __int_as_float(0x7fc00000);
                        live[u] = false;
                        continue;
                    }
                    node[u] = nxt;
                    any = true;
                }
            }
#pragma unroll
            for (int u = 0; u < PRED_G; ++u)
                if (t0 + u * K < T) acc = __fadd_rn(acc, __fmul_rn(lr, val[u]));
        }
        out[row * K + c] = acc;
    }
}

// Heap forest (depth D <= HEAP_DMAX): tree t is 2^(D+1) 32-bit words at
// heap + t * 2^(D+1): words [0, 2^D - 1) are the internal slots of a
// complete binary tree in heap order (children of slot i: 2i+1, 2i+2), each
// (feature & 0xFFFF) | (uint8 split bin << 16); word 2^D - 1 is unused;
// the leaf value of depth-D slot h (2^D - 1 <= h < 2^(D+1) - 1) is word
// h + 1, so words [2^D, 2^(D+1)) hold the leaves.  A leaf at depth
// d < D becomes a chain of pass-through slots {feature 0, bin 127} (every
// int8 bin is <= 127, so rows go left) ending at its leftmost depth-D
// descendant, which holds its value.  Every walk is then exactly D steps
// with no data-dependent trip count.
//
// One thread per row, two CTAs per SM.  A CTA stages its R rows' bins in
// shared memory with 16-byte cp.async copies (STAGED: row stride a multiple
// of 16 and at least 64 rows fit; else rows are read from global memory) and
// streams the forest through two shared-memory buffers of G trees each:
// group g + 1 is copied while every thread walks its row through the trees
// of group g, up to four trees at a time, adding leaves strictly in tree order
// (class of tree t = t % K).  While one CTA of an SM waits for its rows,
// the other walks trees.
constexpr int HEAP_DMAX = 12;
constexpr int HEAP_THREADS = 192;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <bool STAGED, int CH>  // CH: trees walked at once per thread (<= trees per buffer)
__global__ void __launch_bounds__(HEAP_THREADS, 2) k_predict_heap(
    const int8_t *__restrict__ bins, long long n, long long S, const uint32_t *__restrict__ heap, int T, int K,
    int D, int G, float lr, float *__restrict__ out) {
    extern __shared__ __align__(16) uint32_t s_heap[];
    const int TW = 2 << D;                 // words per tree
    uint32_t *tb = s_heap;                 // [2][G * TW]
    uint8_t *rows = reinterpret_cast<uint8_t *>(s_heap + 2 * G * TW);  // [R][RS]
    const int RS = (int)S + 16;            // staged row stride: 16-byte aligned, shifts banks by 4 per row
    const int Smax = (int)S - 1;
    const int R = blockDim.x;
    const long long r0 = (long long)blockIdx.x * R;
    const int nrows = (int)min((long long)R, n - r0);
    auto prefetch = [&](int g) {
        const int t0 = g * G, nt = min(G, T - t0);
        const uint4 *src = reinterpret_cast<const uint4 *>(heap + (long long)t0 * TW);
        uint4 *dst = reinterpret_cast<uint4 *>(tb + (g & 1) * G * TW);
        for (int i = threadIdx.x; i < nt * TW / 4; i += R) cp_async16(dst + i, src + i);
    };
    const int ngroups = (T + G - 1) / G;
    if (STAGED) {  // the CTA's rows, 16 bytes per copy, all in flight at once
        const int v16 = (int)(S / 16);
        for (int t = threadIdx.x; t < nrows * v16; t += R) {
            const int rr = t / v16, c = t - rr * v16;
            cp_async16(rows + (size_t)rr * RS + 16 * c, bins + (r0 + rr) * S + 16 * c);
        }
    }
    prefetch(0);
    cp_async_commit();  // group: rows + trees of group 0
    const bool live = threadIdx.x < nrows;
    const long long row = r0 + threadIdx.x;
    const int8_t *myrow = STAGED ? reinterpret_cast<const int8_t *>(rows + (size_t)threadIdx.x * RS)
                                 : bins + (live ? row : 0) * S;
    float acc = (live && K == 1) ? out[row] : 0.0f;
    for (int g = 0; g < ngroups; ++g) {
        if (g + 1 < ngroups) {
            prefetch(g + 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();  // group g (and, first time, the rows) visible to every thread
        if (live) {
            const uint32_t *grp = tb + (g & 1) * G * TW;
            const int t0 = g * G, nt = min(G, T - t0);
            for (int u0 = 0; u0 < nt; u0 += CH) {
                const uint32_t *tr[CH];
                int node[CH];
#pragma unroll
                for (int u = 0; u < CH; ++u) {
                    tr[u] = grp + min(u0 + u, nt - 1) * TW;
                    node[u] = 0;
                }
                for (int d = 0; d < D; ++d) {
#pragma unroll
                    for (int u = 0; u < CH; ++u) {
                        const uint32_t w = tr[u][node[u]];
                        const int f = min((int)(w & 0xFFFFu), Smax);  // a feature past the row reads its last byte
                        const int sb = (int)(int8_t)(w >> 16);
                        const int b = (int)(STAGED ? myrow[f] : __ldg(myrow + f));
                        node[u] = 2 * node[u] + 1 + (b > sb ? 1 : 0);
                    }
                }
#pragma unroll
                for (int u = 0; u < CH; ++u) {
                    if (u0 + u >= nt) break;
                    const float v = __uint_as_float(tr[u][node[u] + 1]);
                    const int t = t0 + u0 + u;
                    if (K == 1) {
                        acc = __fadd_rn(acc, __fmul_rn(lr, v));
                    } else {
                        float *o = out + row * K + (t % K);
                        *o = __fadd_rn(*o, __fmul_rn(lr, v));
                    }
                }
            }
        }
        __syncthreads();  // group g's buffer is read before group g + 2 overwrites it
    }
    if (live && K == 1) out[row] = acc;
}

// The reference's flattened format (core.py:1215-1252): [T][max_nodes][6].
__global__ void k_predict_flat(const int8_t *__restrict__ bins, long long n, long long F,
                               const float *__restrict__ forest, int T, int max_nodes, float lr,
                               float *__restrict__ out) {
    long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int8_t *r = bins + i * F;
    float acc = out[i];
    for (int t = 0; t < T; ++t) {
        const float *tree = forest + (long long)t * max_nodes * 6;
        int node = 0;
        float v = __int_as_float(0x7fc00000);
        for (int step = 0; step < max_nodes; ++step) {
            const float *nd = tree + node * 6;
            if (nd[4] > 0.5f) {
                v = nd[5];
                break;
            }
            int f = (int)nd[0], sb = (int)nd[1];
            if (f < 0 || f >= F) break;
            int nxt = (r[f] <= sb) ? (int)nd[2] : (int)nd[3];
            if (nxt <= node || nxt >= max_nodes) break;
            node = nxt;
        }
        acc = __fadd_rn(acc, __fmul_rn(lr, v));
    }
    out[i] = acc;
}

// ====================================================================== //
// reference-compatible split / histogram                                 //
// ====================================================================== //

__global__ void k_ref_split(const float *__restrict__ G, const float *__restrict__ H, int E, int k, int B,
                            float mcs, float eps, float *__restrict__ gain, float *__restrict__ dir) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    int e = blockIdx.y;
    if (j >= k || e >= E) return;
    const long long base = ((long long)e * k + j) * B;
    const long long bg = ((long long)e * k + j) * (B - 1);
    float GT = 0.0f, HT = 0.0f;
    for (int b = 0; b < B; ++b) {
        GT = __fadd_rn(GT, G[base + b]);
        HT = __fadd_rn(HT, H[base + b]);
    }
    float GL = 0.0f, HL = 0.0f;
    for (int b = 0; b < B - 1; ++b) {
        GL = __fadd_rn(GL, G[base + b]);
        HL = __fadd_rn(HL, H[base + b]);
        SplitEval r = eval_split(GL, HL, GT, HT, mcs, eps);
        gain[bg + b] = r.gain;
        dir[bg + b] = r.dir;
    }
}

__global__ void k_max_abs_rows(const float *__restrict__ g, const int *__restrict__ rows, long long n,
                               long long nrows, float *maxabs) {
    float m = 0.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        int r = rows[i];
        if (r >= 0 && r < nrows) m = fmaxf(m, fabsf(g[r]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<int *>(maxabs), __float_as_int(m));
}

__global__ void k_single_node(const float *maxabs, int *shift, wgb_node *nd, int n, int *nn) {
    *shift = quant_shift(*maxabs);
    wgb_node r{};
    r.lstart = 0;
    r.lcnt = n;
    r.slot = 0;
    r.built = 1;
    r.fpos = -1;
    r.child = -1;
    *nd = r;
    *nn = 1;
}

__global__ void k_kpos(const int *__restrict__ feats, int k, int F, int *__restrict__ kpos) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= k) return;
    int f = feats[j];
    if (f >= 0 && f < F) kpos[f] = j;
}

__global__ void k_hist_to_float(const long long *__restrict__ hg, const long long *__restrict__ hc, long long m,
                                int B, const int *shift, float *__restrict__ G, float *__restrict__ H) {
    const float inv = pow2f(-*shift);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < m * B;
         i += (long long)gridDim.x * blockDim.x) {
        long long c = i / B;
        int b = (int)(i - c * B);
        long long src = c * (B + 1) + b;
        G[i] = __fadd_rn(G[i], __fmul_rn(__ll2float_rn(hg[src]), inv));
        H[i] = __fadd_rn(H[i], __ll2float_rn(hc[src]));
    }
}

static int grid_cap(long long n, int threads) {
    long long b = (n + threads - 1) / threads;
    if (b < 1) b = 1;
    if (b > 148 * 16) b = 148 * 16;
    return (int)b;
}

}  // namespace wgb

using namespace wgb;

extern "C" {

int wgb_bin_matrix(const float *X, int64_t n, int32_t F, int64_t x_stride, const float *edges,
                   int32_t num_bins, int8_t *out, int64_t out_stride, void *stream) {
    WGB_CHECK_ARG(n >= 0 && F >= 1, "bad shape n=%lld F=%d", (long long)n, F);
    WGB_CHECK_ARG(num_bins >= 2 && num_bins <= 127, "num_bins must be in [2, 127]");
    WGB_CHECK_ARG(x_stride >= F, "x_stride < F");
    WGB_CHECK_ARG(out_stride >= F && out_stride % 4 == 0, "out_stride must be >= F and a multiple of 4");
    if (n == 0) return WGB_OK;
    WGB_CHECK_ARG(X && edges && out, "NULL pointer");
    const int nb = num_bins - 1;
    size_t smem = (size_t)nb * BIN_FT * sizeof(float);
    dim3 grid((unsigned)((n + BIN_ROWS - 1) / BIN_ROWS), (unsigned)((out_stride + BIN_FT - 1) / BIN_FT));
#define WGB_BIN_CASE(NB_)                                                                                  \
    if (NB_ == 0 || nb == NB_) {                                                                          \
        WGB_CUDA(cudaFuncSetAttribute(k_bin_matrix<NB_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
        k_bin_matrix<NB_><<<grid, 256, smem, as_stream(stream)>>>(X, n, F, x_stride, edges, nb, out, out_stride); \
        WGB_LAUNCHED("k_bin_matrix");                                                                     \
        return WGB_OK;                                                                                    \
    }
    WGB_BIN_CASE(31)
    WGB_BIN_CASE(15)
    WGB_BIN_CASE(63)
    WGB_BIN_CASE(7)
    WGB_BIN_CASE(3)
    WGB_BIN_CASE(1)
    WGB_BIN_CASE(0)
#undef WGB_BIN_CASE
    return WGB_OK;
}

int wgb_prebinned_ingest(const int8_t *X, int64_t n, int32_t F, int64_t x_stride, int8_t *out,
                         int64_t out_stride, int32_t *colmax, int32_t *minmax, void *stream) {
    WGB_CHECK_ARG(n >= 0 && F >= 1 && x_stride >= F, "bad shape n=%lld F=%d", (long long)n, F);
    WGB_CHECK_ARG(out_stride >= F && out_stride % 4 == 0, "out_stride must be >= F and a multiple of 4");
    WGB_CHECK_ARG(colmax && minmax && (out || n == 0) && (X || n == 0), "NULL pointer");
    cudaStream_t st = as_stream(stream);
    // sentinels: 0x80808080 is below every int8, 0x7f7f7f7f above
    WGB_CUDA(cudaMemsetAsync(colmax, 0x80, sizeof(int32_t) * F, st));
    WGB_CUDA(cudaMemsetAsync(minmax, 0x7f, sizeof(int32_t), st));
    WGB_CUDA(cudaMemsetAsync(minmax + 1, 0x80, sizeof(int32_t), st));
    if (n == 0) return WGB_OK;
    dim3 grid((unsigned)((n + BIN_ROWS - 1) / BIN_ROWS), (unsigned)((out_stride + BIN_FT - 1) / BIN_FT));
    k_prebinned<<<grid, 256, 0, st>>>(X, n, F, x_stride, out, out_stride, colmax, minmax);
    WGB_LAUNCHED("k_prebinned");
    return WGB_OK;
}

int wgb_custom_cuda_binner(const float *X, int64_t n, const float *bin_edges, int32_t num_edges,
                           int8_t *bin_indices, void *stream) {
    WGB_CHECK_ARG(n >= 0 && num_edges >= 0, "bad sizes");
    if (n == 0) return WGB_OK;
    WGB_CHECK_ARG(X && bin_indices && (bin_edges || num_edges == 0), "NULL pointer");
    k_bin_column<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(X, n, bin_edges, num_edges,
                                                                              bin_indices);
    WGB_LAUNCHED("k_bin_column");
    return WGB_OK;
}

// rows per CTA of the staged predictors: the largest multiple of 32 (at
// most `cap`) whose rows fit `budget` bytes; 0 = rows too wide to stage
static int staged_rows(long long S, int cap, size_t budget) {
    int r = cap;
    while (r >= 64 && (size_t)r * (size_t)(S + 4) > budget) r -= 32;
    return (size_t)r * (size_t)(S + 4) <= budget && r >= 64 ? r : 0;
}

int wgb_predict_packed(const int8_t *bins, int64_t n, int64_t S, const int32_t *nodes,
                       const int32_t *tree_off, int32_t T, int32_t K, float lr, float *out,
                       void *stream) {
    WGB_CHECK_ARG(n >= 0 && S >= 4 && S % 4 == 0, "bad bins shape (stride must be a multiple of 4)");
    WGB_CHECK_ARG(T >= 0 && K >= 1, "bad forest shape");
    if (n == 0 || T == 0) return WGB_OK;
    const int rp = staged_rows(S, PRED_ROWS, 160 * 1024);
    if (rp) {
        const size_t smem = (size_t)rp * (S + 4);
        WGB_CUDA(cudaFuncSetAttribute(k_predict_packed<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        k_predict_packed<true><<<(unsigned)((n + rp - 1) / rp), rp, smem, as_stream(stream)>>>(
            bins, n, S, reinterpret_cast<const int2 *>(nodes), tree_off, T, K, lr, out);
    } else {
        k_predict_packed<false><<<(unsigned)((n + PRED_ROWS - 1) / PRED_ROWS), PRED_ROWS, 0, as_stream(stream)>>>(
            bins, n, S, reinterpret_cast<const int2 *>(nodes), tree_off, T, K, lr, out);
    }
    WGB_LAUNCHED("k_predict_packed");
    return WGB_OK;
}

int wgb_predict_heap(const int8_t *bins, int64_t n, int64_t S, const uint32_t *heap, int32_t T, int32_t K,
                     int32_t D, float lr, float *out, void *stream) {
    WGB_CHECK_ARG(n >= 0 && S >= 4 && S % 4 == 0, "bad bins shape (stride must be a multiple of 4)");
    WGB_CHECK_ARG(T >= 0 && K >= 1, "bad forest shape");
    WGB_CHECK_ARG(D >= 1 && D <= HEAP_DMAX, "heap forests hold depth 1..%d, got %d", HEAP_DMAX, D);
    WGB_CHECK_ARG((reinterpret_cast<uintptr_t>(heap) & 15) == 0, "heap must be 16-byte aligned");
    if (n == 0 || T == 0) return WGB_OK;
    const size_t tree_bytes = (size_t)8 << D;  // 2^(D+1) words
    // two CTAs per SM (one stages its rows while the other walks trees):
    // each gets up to 110 KB -- trees per buffer up to 8 within 32 KB for
    // both buffers together, the rest for its rows
    int G = (int)std::min<size_t>(8, std::max<size_t>(1, (32 * 1024) / (2 * tree_bytes)));
    if (G > T) G = T;
    const size_t tsm = 2 * (size_t)G * tree_bytes;
    const size_t budget = tsm < 110 * 1024 ? 110 * 1024 - tsm : 0;
    int R = 0;
    if (S % 16 == 0) {
        R = HEAP_THREADS;
        while (R >= 64 && (size_t)R * (size_t)(S + 16) > budget) R -= 32;
        if (R < 64 || (size_t)R * (size_t)(S + 16) > budget) R = 0;
    }
    cudaStream_t st = as_stream(stream);
#define WGB_HEAP_LAUNCH(CH_)                                                                                 \
    if (R) {                                                                                                 \
        const size_t smem = tsm + (size_t)R * (S + 16);                                                      \
        WGB_CUDA(cudaFuncSetAttribute(k_predict_heap<true, CH_>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                      (int)smem));                                                          \
        k_predict_heap<true, CH_><<<(unsigned)((n + R - 1) / R), R, smem, st>>>(bins, n, S, heap, T, K, D, G, lr, \
                                                                               out);                          \
    } else {                                                                                                 \
        WGB_CUDA(cudaFuncSetAttribute(k_predict_heap<false, CH_>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                      (int)tsm));                                                           \
        k_predict_heap<false, CH_><<<(unsigned)((n + HEAP_THREADS - 1) / HEAP_THREADS), HEAP_THREADS, tsm, st>>>( \
            bins, n, S, heap, T, K, D, G, lr, out);                                                          \
    }
    if (G >= 4) {
        WGB_HEAP_LAUNCH(4)
    } else if (G >= 2) {
        WGB_HEAP_LAUNCH(2)
    } else {
        WGB_HEAP_LAUNCH(1)
    }
#undef WGB_HEAP_LAUNCH
    WGB_LAUNCHED("k_predict_heap");
    return WGB_OK;
}

int wgb_predict_forest(const int8_t *bin_indices, int64_t n, int64_t F, const float *tree_tensor,
                       int32_t T, int32_t max_nodes, float learning_rate, float *out, void *stream) {
    WGB_CHECK_ARG(n >= 0 && F >= 1 && T >= 0 && max_nodes >= 1, "bad shapes");
    if (n == 0 || T == 0) return WGB_OK;
    k_predict_flat<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(
        bin_indices, n, F, tree_tensor, T, max_nodes, learning_rate, out);
    WGB_LAUNCHED("k_predict_flat");
    return WGB_OK;
}

int wgb_compute_split(const float *G, const float *H, int32_t num_eras, int32_t k, int32_t num_bins,
                      float min_split_gain, float min_child_samples, float eps, float *per_era_gain,
                      float *per_era_direction, int32_t threads, void *stream) {
    (void)min_split_gain;  // unused by the reference kernel as well
    WGB_CHECK_ARG(num_eras >= 1 && k >= 0 && num_bins >= 2, "bad histogram shape");
    WGB_CHECK_ARG(threads >= 1 && threads <= 1024, "threads must be in [1, 1024]");
    if (k == 0) return WGB_OK;
    dim3 grid((unsigned)((k + threads - 1) / threads), (unsigned)num_eras);
    k_ref_split<<<grid, threads, 0, as_stream(stream)>>>(G, H, num_eras, k, num_bins, min_child_samples, eps,
                                                         per_era_gain, per_era_direction);
    WGB_LAUNCHED("k_ref_split");
    return WGB_OK;
}

int wgb_compute_histogram3(const int8_t *bin_indices, int64_t num_rows, int64_t F_master,
                           const float *residuals, const int32_t *sample_indices, int64_t n,
                           const int32_t *feature_indices, int32_t k, const int32_t *era_indices,
                           float *grad_hist, float *hess_hist, int32_t num_eras, int32_t num_bins,
                           int32_t threads_per_block, int32_t rows_per_thread, void *stream) {
    WGB_CHECK_ARG(threads_per_block > 0 && threads_per_block % 32 == 0,
                  "threads_per_block should be a positive multiple of 32");
    WGB_CHECK_ARG(rows_per_thread >= 1 && rows_per_thread <= 16, "rows_per_thread must be in [1, 16]");
    WGB_CHECK_ARG(num_bins >= 2 && num_bins <= 127, "num_bins must be in [2, 127]");
    WGB_CHECK_ARG(num_eras >= 1 && k >= 0 && n >= 0 && num_rows >= 0 && F_master >= 1, "bad sizes");
    WGB_CHECK_ARG(n < (1ll << 31), "too many samples");
    if (n == 0 || k == 0) return WGB_OK;
    cudaStream_t st = as_stream(stream);
    const long long se = (long long)num_eras * k * (num_bins + 1);
    const int nchunk = (int)((n + HIST_R - 1) / HIST_R);
    // scratch from the stream-ordered pool
    long long *hg = nullptr, *hc = nullptr;
    int *kpos = nullptr, *small = nullptr;
    int4 *chunks = nullptr;
    wgb_node *nd = nullptr;
    WGB_CUDA(cudaMallocAsync((void **)&hg, sizeof(long long) * se, st));
    WGB_CUDA(cudaMallocAsync((void **)&hc, sizeof(long long) * se, st));
    WGB_CUDA(cudaMallocAsync((void **)&kpos, sizeof(int) * F_master, st));
    WGB_CUDA(cudaMallocAsync((void **)&chunks, sizeof(int4) * nchunk, st));
    WGB_CUDA(cudaMallocAsync((void **)&small, sizeof(int) * 8, st));
    WGB_CUDA(cudaMallocAsync((void **)&nd, sizeof(wgb_node), st));
    int *nchunks = small, *shift = small + 1, *nn = small + 2;
    float *maxabs = reinterpret_cast<float *>(small + 3);
    int rc = WGB_OK;
    do {
        if (cudaMemsetAsync(hg, 0, sizeof(long long) * se, st) != cudaSuccess ||
            cudaMemsetAsync(hc, 0, sizeof(long long) * se, st) != cudaSuccess ||
            cudaMemsetAsync(kpos, 0xff, sizeof(int) * F_master, st) != cudaSuccess ||
            cudaMemsetAsync(small, 0, sizeof(int) * 8, st) != cudaSuccess) {
            set_error("cudaMemsetAsync failed");
            rc = WGB_ERR_CUDA;
            break;
        }
        k_kpos<<<(k + 255) / 256, 256, 0, st>>>(feature_indices, k, (int)F_master, kpos);
        k_max_abs_rows<<<grid_cap(n, 256), 256, 0, st>>>(residuals, sample_indices, n, num_rows, maxabs);
        k_single_node<<<1, 1, 0, st>>>(maxabs, shift, nd, (int)n, nn);
        k_chunk_plan<<<1, 1024, 0, st>>>(nd, nn, chunks, nchunks, nchunk, 0);
        cudaError_t le = launch_hist(nchunk, bin_indices, F_master, (int)F_master, sample_indices, nullptr,
                                     residuals, shift, num_eras > 1 ? era_indices : nullptr, kpos, k,
                                     num_eras, num_bins, 0, false, chunks, nchunks, nd,
                                     HistOut{hg, hc, se, 0, k, 0}, num_rows, st);
        if (le != cudaSuccess) {
            set_error("k_hist launch failed: %s", cudaGetErrorString(le));
            rc = WGB_ERR_CUDA;
            break;
        }
        k_hist_to_float<<<grid_cap((long long)num_eras * k * num_bins, 256), 256, 0, st>>>(
            hg, hc, (long long)num_eras * k, num_bins, shift, grad_hist, hess_hist);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            set_error("wgb_compute_histogram3 launch failed: %s", cudaGetErrorString(e));
            rc = WGB_ERR_CUDA;
        }
    } while (0);
    cudaFreeAsync(hg, st);
    cudaFreeAsync(hc, st);
    cudaFreeAsync(kpos, st);
    cudaFreeAsync(chunks, st);
    cudaFreeAsync(small, st);
    cudaFreeAsync(nd, st);
    return rc;
}

}  // extern "C"
