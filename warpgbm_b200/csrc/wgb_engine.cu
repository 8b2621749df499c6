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
#include <algorithm>
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

__global__ void k_reset(float *maxabs, long long *rootsum, int ntree) {
    pdl_wait();  // the previous kernel on the stream has completed
    for (int t = threadIdx.x; t < ntree; t += blockDim.x) {
        maxabs[t] = 0.0f;
        rootsum[t] = 0;
    }
}

// Tree t = blockIdx.y of the batch: g[t][i] = y - pred[:, cls + t]
// (regression, core.py:719; y == NULL: g is given, e.g. the softmax
// residuals of a multiclass round, core.py:782) and max |g| of the tree.
__global__ void k_residual(const float *__restrict__ y, const float *__restrict__ pred, int K,
                           int cls, float *__restrict__ g, long long n, float *maxabs) {
    pdl_wait();  // the previous kernel on the stream has completed
    const int t = blockIdx.y;
    g += (long long)t * n;
    float m = 0.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v;
        if (y) {
            v = __fsub_rn(y[i], pred[i * K + cls + t]);
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
        atomicMax(reinterpret_cast<int *>(maxabs + t), __float_as_int(m));
    }
}

// Tree t = blockIdx.y: q = rint(g * 2^s) with the tree's own shift, sum of q.
__global__ void k_quantize(const float *__restrict__ g, int *__restrict__ qg, long long n,
                           const float *maxabs, int *shift_out, long long *rootsum) {
    pdl_wait();  // the previous kernel on the stream has completed
    const int t = blockIdx.y;
    g += (long long)t * n;
    qg += (long long)t * n;
    const int s = quant_shift(maxabs[t]);
    if (blockIdx.x == 0 && threadIdx.x == 0) shift_out[t] = s;
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
        atomicAdd(reinterpret_cast<unsigned long long *>(rootsum + t), (unsigned long long)acc);
    }
}

// Root records of the batch's trees (root t = node t of level 0, slot t,
// local positions [t*N, (t+1)*N)); their sums of q and leaves are filled by
// k_root_total once the level-0 histograms (which carry the root sums) are
// complete on every rank.
__global__ void k_root(wgb_node *nodes, int *nn, int *nact, int D, long long n_local,
                       long long n_global, int ntree) {
    pdl_wait();  // the previous kernel on the stream has completed
    for (int t = threadIdx.x; t < ntree; t += blockDim.x) {
        wgb_node r;
        r.sumq = 0;
        r.count = n_global;
        r.lsumq = 0;
        r.lcount = 0;
        r.lstart = (int)(t * n_local);
        r.lcnt = (int)n_local;
        r.slot = t;
        r.built = node_flags(true, t);
        r.fpos = -1;
        r.bin = 0;
        r.child = -1;
        r.leaf = 0.0f;
        nodes[t] = r;
    }
    if (threadIdx.x == 0) {
        for (int d = 0; d <= D; ++d) {
            nn[d] = d == 0 ? ntree : 0;
            nact[d] = d == 0 ? (int)(ntree * n_local) : 0;
        }
    }
}

// Copies each tree's local root sum into its root slot's first spare cell
// (of every slice region of a sliced fit's staging buffer), so that the
// level-0 reduction carries it.
// out[0, n) = 0: a level's histogram slots before its build (a kernel, so
// the level's launches stay one chain of dependent launches).
__global__ void __launch_bounds__(256) k_zero(long long *out, long long n) {
    pdl_wait();  // the previous kernel on the stream has completed
    for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long long)gridDim.x * 256) out[i] = 0;
}
static inline unsigned zero_grid(long long n) {
    const long long g = (n + 255) / 256;
    return (unsigned)(g < 1 ? 1 : (g > 148 * 8 ? 148 * 8 : g));
}

__global__ void k_root_cells(long long *hg, const long long *rootsum, long long slot_elems, long long nc,
                             int ntree, int nregion, long long region_stride) {
    pdl_wait();  // the previous kernel on the stream has completed
    for (int i = threadIdx.x; i < ntree * nregion; i += blockDim.x) {
        const int t = i % ntree, r = i / ntree;
        hg[r * region_stride + t * slot_elems + 2 * nc] = rootsum[t];
    }
}

__global__ void k_root_total(wgb_node *nodes, const long long *hg, long long slot_elems, long long nc,
                             const int *shift, int ntree) {
    pdl_wait();  // the previous kernel on the stream has completed
    for (int t = threadIdx.x; t < ntree; t += blockDim.x) {
        wgb_node &r = nodes[t];
        r.sumq = hg[t * slot_elems + 2 * nc];
        r.leaf = canon_leaf(r.sumq, r.count, pow2f(-shift[t]));
    }
}

// ====================================================================== //
// histogram build                                                        //
// ====================================================================== //

// Chunk list of a level, by one block (any size up to 1024 threads): every
// built node's local rows cut into m = ceil(rows / R) pieces of equal size
// (at most R <= HIST_R rows each).  With wave = 0, R = HIST_R.  With wave > 0
// (the chunks that one wave of the histogram kernel's resident CTAs builds at
// once, all feature tiles included), R is chosen so that the chunk count fills the
// waves that HIST_R-row chunks would start: one full wave plus a few chunks
// would otherwise take two wave times.  R never goes below HIST_R / 2 nor
// below what keeps the list within `cap` entries.  The level's records come
// from earlier launches or from this block (visible after its barrier).
__device__ __forceinline__ void plan_chunks(const wgb_node *__restrict__ lvl, int nnd, int4 *chunks, int *nchunks,
                                            int cap, int wave) {
    __shared__ int s_cnt[1024];
    __shared__ int s_off[1025];
    __shared__ int s_scan[33];
    const int nt = blockDim.x;
    int R = HIST_R;
    if (wave > 0) {
        int T = 0, nb = 0, u0 = 0;  // rows, nodes and HIST_R-row chunks of the built nodes
        for (int b0 = 0; b0 < nnd; b0 += nt) {
            const int i = b0 + threadIdx.x;
            const int n = i < nnd && node_built(lvl[i].built) ? lvl[i].lcnt : 0;
            int t;
            block_scan_excl(n, s_scan, t);
            T += t;
            block_scan_excl(n > 0 ? 1 : 0, s_scan, t);
            nb += t;
            block_scan_excl((n + HIST_R - 1) / HIST_R, s_scan, t);
            u0 += t;
        }
        if (nb > 0) {
            const long long K = (long long)((u0 + wave - 1) / wave) * wave;  // chunks of those whole waves
            long long r = K > nb ? ((long long)T + K - nb - 1) / (K - nb) : HIST_R;
            if (cap > nb) r = max(r, ((long long)T + cap - nb - 1) / (cap - nb));
            else r = HIST_R;
            if (r < HIST_R / 2) r = HIST_R / 2;
            R = r < HIST_R ? (int)r : HIST_R;
        }
    }
    int base = 0;
    for (int b0 = 0; b0 < nnd; b0 += nt) {
        int i = b0 + threadIdx.x;
        int c = 0;
        if (i < nnd && node_built(lvl[i].built)) c = (lvl[i].lcnt + R - 1) / R;
        s_cnt[threadIdx.x] = c;
        int tot;
        const int ex = block_scan_excl(c, s_scan, tot);
        s_off[threadIdx.x] = base + ex;
        if (threadIdx.x == 0) s_off[nt] = base + tot;
        __syncthreads();
        int lo = s_off[0], hi = s_off[nt];
        for (int c2 = lo + threadIdx.x; c2 < hi; c2 += nt) {
            // node of chunk c2: last t with s_off[t] <= c2 and s_cnt[t] > 0
            int a = 0, z = nt - 1;
            while (a < z) {
                int m = (a + z + 1) >> 1;
                if (s_off[m] <= c2) a = m; else z = m - 1;
            }
            while (s_cnt[a] == 0) --a;
            const int node = b0 + a;
            const long long piece = c2 - s_off[a], m = s_cnt[a], n = lvl[node].lcnt;
            const int p0 = lvl[node].lstart + (int)(piece * n / m);
            const int p1 = lvl[node].lstart + (int)((piece + 1) * n / m);
            if (c2 < cap) chunks[c2] = make_int4(node, p0, p1, 0);
        }
        __syncthreads();
        base = hi;
    }
    if (threadIdx.x == 0) *nchunks = min(base, cap);
}

// Chunk list of level 0 (later levels are planned by k_node_offsets).
__global__ void __launch_bounds__(1024) k_chunk_plan(const wgb_node *__restrict__ lvl, const int *nn_d,
                                                     int4 *chunks, int *nchunks, int cap, int wave) {
    pdl_wait();  // the previous kernel on the stream has completed
    plan_chunks(lvl, *nn_d, chunks, nchunks, cap, wave);
}

// One CTA = one chunk (<= HIST_R rows of one node) x one tile of 32*FPL
// features.  Lane l of every warp owns features FPL*l .. FPL*l+FPL-1 of the
// tile (one FPL-byte load per row).  Every histogram cell is two 32-bit
// shared words updated with native 32-bit reductions (64-bit shared atomics
// are several times slower on sm_100):
//     A  += (1 << 20) + (q & 0x1FF)       count (<= 2048) | low 9 bits of q
//     Bw += q >> 9                        high bits of q (arithmetic shift)
// so sum(q) = Bw * 512 + (A & 0xFFFFF) and count = A >> 20 exactly for up
// to HIST_R = 2048 rows per chunk (HIST_CNT_SHIFT / HIST_LO_BITS).
// Shared layout of each word array: [era slot][j/2][bin slot 0..NSC-1][j%2][lane]
// -- a bin slot is 256 bytes, so one byte-permute turns a bin into its byte
// offset, the feature term is an immediate, and a warp's 32 reductions hit
// 32 consecutive words (no bank conflicts).  Slots: 0..B-1 bins, B negative
// bins (they always go left, core.py:629), B+1 trash for bins >= B (skipped
// by the reference, histogram_kernel.cu:41); REGULAR instantiations know
// every bin lies in [0, B).  Every feature of a lane is accumulated
// unconditionally -- cells of unselected or padding features are never
// flushed -- so an update is four instructions: permute, add, two reductions.
// When q == nullptr the residual g is quantised on the fly with 2^shift (the
// drop-in wgb_compute_histogram3).
template <int IMM>
__device__ __forceinline__ void red_shared(uint32_t addr, uint32_t v) {
    asm volatile("red.shared.add.u32 [%0+%2], %1;" ::"r"(addr), "r"(v), "n"(IMM) : "memory");
}

template <int FPL, int NSC, int J>
__device__ __forceinline__ void hist_update(uint32_t ra, uint32_t b8, uint32_t pa, uint32_t pb) {
    constexpr int OFF = (J >> 1) * NSC * 256 + (J & 1) * 128;
    constexpr int BOFF = (FPL / 2) * NSC * 256;  // word array B follows A within an era slot
    const uint32_t a = ra + b8;
    red_shared<OFF>(a, pa);
    red_shared<BOFF + OFF>(a, pb);
}

template <int FPL, int NSC, bool REGULAR, int J = 0>
__device__ __forceinline__ void hist_row(const uint32_t (&w)[FPL / 4], uint32_t ra, uint32_t pa, uint32_t pb,
                                         int B) {
    if constexpr (J < FPL) {
        uint32_t b8;
        if constexpr (REGULAR) {
            b8 = __byte_perm(w[J >> 2], 0u, 0x4404u | ((J & 3) << 4));  // bin << 8
        } else {
            const int sb = (int)(int8_t)__byte_perm(w[J >> 2], 0u, 0x4440u | (J & 3));
            b8 = (uint32_t)(sb < 0 ? B : (sb >= B ? B + 1 : sb)) << 8;
        }
        hist_update<FPL, NSC, J>(ra, b8, pa, pb);
        hist_row<FPL, NSC, REGULAR, J + 1>(w, ra, pa, pb, B);
    }
}

// Fast-path row update (one era, every bin in [0, B)): one byte-permute
// puts the bin into byte 1 of the lane's word offset (4*lane < 256), so the
// cell address is a single instruction and an update is three: permute and
// the two reductions.
template <int FPL, int NSC, int J = 0>
__device__ __forceinline__ void hist_row_fast(const uint32_t (&w)[FPL / 4], uint32_t sh0, uint32_t lane4,
                                              uint32_t pa, uint32_t pb) {
    if constexpr (J < FPL) {
        constexpr int OFF = (J >> 1) * NSC * 256 + (J & 1) * 128;
        constexpr int BOFF = (FPL / 2) * NSC * 256;
        const uint32_t a = sh0 + __byte_perm(w[J >> 2], lane4, 0x7604u | ((J & 3) << 4));
        red_shared<OFF>(a, pa);
        red_shared<BOFF + OFF>(a, pb);
        hist_row_fast<FPL, NSC, J + 1>(w, sh0, lane4, pa, pb);
    }
}

// FPL bytes of one row at src (FPL-aligned)
template <int FPL>
__device__ __forceinline__ void load_row(const int8_t *src, uint32_t (&w)[FPL / 4]) {
    if constexpr (FPL == 16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src));
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (FPL == 8) {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(src));
        w[0] = v.x; w[1] = v.y;
    } else {
        w[0] = __ldg(reinterpret_cast<const uint32_t *>(src));
    }
}

template <int FPL, int NT, int MINB, int NSC, int EWC, bool HAS_ERA, bool REGULAR>
__device__ __forceinline__ void hist_item(
    int c, int ft, int ntile, const int8_t *__restrict__ bins, long long S, int F, const int *__restrict__ order,
    const int *__restrict__ q, const float *__restrict__ g, const int *shift,
    const int *__restrict__ era, const int *__restrict__ kpos, int k, int E, int B, int EW,
    const int4 *__restrict__ chunks, const wgb_node *__restrict__ lvl,
    const HistOut &out, long long nrows, uint2 *__restrict__ part) {
    constexpr int FT = 32 * FPL;             // features per tile
    constexpr int U = (FPL >= 16 || MINB > 1) ? 4 : 8;  // rows per pipeline step per warp
    constexpr int NW = NT / 32;
    constexpr int WPR = FPL / 4;             // 32-bit words per lane per row
    constexpr int ESLOT = 2 * NSC * FT;      // words per era slot (A and B arrays)
    constexpr int UF = 8;                    // rows per fast-path step per warp
    constexpr int PADR = NW * UF;            // padding rows read past the chunk's end
    extern __shared__ uint32_t sh32[];       // [EWC][A|B][j/2][NSC][j%2][32]
    __shared__ int s_kp[FT];                 // lane-major: [j][lane]
    // per chunk row: the row (0 when skipped or padding) and its two word
    // increments; pa == 0 marks a skipped or padding row (pa >= 2^20 otherwise)
    __shared__ __align__(16) int s_row[HIST_R + PADR];
    __shared__ __align__(16) uint2 s_pq[HIST_R + PADR];
    __shared__ int s_era[HIST_ERA_R(HAS_ERA)];
    __shared__ int s_red[33];

    const int f0 = ft * FT;
    int any = 0;
    for (int t = threadIdx.x; t < FT; t += NT) {
        int f = f0 + t;
        int kp = f < F ? kpos[f] : -1;
        s_kp[(t % FPL) * 32 + t / FPL] = kp;
        any |= kp >= 0;
    }
    if (!__syncthreads_or(any)) return;

    const int4 ch = chunks[c];
    const int cnt = ch.z - ch.y;
    const long long slot = lvl[ch.x].slot;
    if (q) q += (long long)node_tree(lvl[ch.x].built) * nrows;  // the node's tree's residuals
    float sc = 0.0f;
    if (!q) sc = pow2f(*shift);
    // rows outside [0, nrows) or eras outside [0, E) are skipped (only the
    // drop-in entry point can receive them; the engine never produces them)
    for (int i = threadIdx.x; i < cnt + PADR; i += NT) {
        int r = -1, e = 0;
        bool ok = false;
        if (i < cnt) {
            r = order[ch.y + i];
            ok = r >= 0 && r < nrows;
            if (HAS_ERA && ok) {
                e = era[r];
                ok = e >= 0 && e < E;
            }
        }
        const int qv = ok ? (q ? q[r] : __float2int_rn(__fmul_rn(g[r], sc))) : 0;
        s_row[i] = ok ? r : 0;
        s_pq[i] = ok ? make_uint2((1u << HIST_CNT_SHIFT) | ((uint32_t)qv & HIST_LO_MASK), (uint32_t)(qv >> HIST_LO_BITS))
                     : make_uint2(0u, 0u);
        if (HAS_ERA && i < cnt) s_era[i] = ok ? e : INT_MAX;
    }
    __syncthreads();
    const bool aligned = (S % FPL) == 0;
    const int ew_n = HAS_ERA ? min(EW, EWC) : 1;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    bool lane_live = false;
#pragma unroll
    for (int j = 0; j < FPL; ++j) lane_live |= s_kp[j * 32 + lane] >= 0;
    const int B1 = B + 1;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(sh32) + 4u * lane;
    const int8_t *tile = bins + f0 + FPL * lane;

    int e_lo = 0;
    bool era_sorted = false;
    if (HAS_ERA) {
        int m = INT_MAX;
        for (int i = threadIdx.x; i < cnt; i += NT) m = min(m, s_era[i]);
        e_lo = block_min(m, s_red);
        if (e_lo == INT_MAX) return;  // no valid row (uniform)
        // the engine's node rows are era-sorted: each window is then one
        // contiguous run of the chunk (the drop-in entry may pass any order)
        int uns = 0;
        for (int i = threadIdx.x; i + 1 < cnt; i += NT) uns |= s_era[i] > s_era[i + 1];
        era_sorted = !__syncthreads_or(uns);
    }
    for (;;) {
        // rows [i_lo, i_hi) of the chunk and era slots [0, nsl) of this window
        int i_lo = 0, i_hi = cnt, nsl = ew_n;
        if (HAS_ERA && era_sorted) {
            i_lo = lower_bound_int(s_era, cnt, e_lo);           // e_lo is some row's era
            i_hi = lower_bound_int(s_era, cnt, e_lo + ew_n);    // > i_lo
            nsl = s_era[i_hi - 1] - e_lo + 1;                  // in [1, ew_n]
        }
        {
            uint4 *z = reinterpret_cast<uint4 *>(sh32);
            const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
            for (int t = threadIdx.x; t < (nsl * ESLOT) / 4; t += NT) z[t] = zero;
        }
        __syncthreads();
        bool fast = false;
        if constexpr (!HAS_ERA && REGULAR) fast = aligned;
        if constexpr (!HAS_ERA && REGULAR) {
            if (lane_live && fast) {
                // rows of step k+1 load into one register set while step k's
                // cells are updated from the other (no copies between steps);
                // a warp takes UF consecutive rows of a step, so their row
                // ids and increments arrive in 16-byte shared loads; rows past
                // the chunk's end are row 0 with zero increments
                uint32_t wa[UF][WPR], wb[UF][WPR];
                const uint32_t sh0 = (uint32_t)__cvta_generic_to_shared(sh32), lane4 = 4u * lane;
                const unsigned S32 = (unsigned)S;
                auto load = [&](int i0, uint32_t (&ww)[UF][WPR]) {
#pragma unroll
                    for (int u = 0; u < UF; u += 4) {
                        const int4 r4 = *reinterpret_cast<const int4 *>(&s_row[i0 + u]);
                        load_row<FPL>(tile + (unsigned long long)(unsigned)r4.x * S32, ww[u]);
                        load_row<FPL>(tile + (unsigned long long)(unsigned)r4.y * S32, ww[u + 1]);
                        load_row<FPL>(tile + (unsigned long long)(unsigned)r4.z * S32, ww[u + 2]);
                        load_row<FPL>(tile + (unsigned long long)(unsigned)r4.w * S32, ww[u + 3]);
                    }
                };
                auto update = [&](int i0, const uint32_t (&ww)[UF][WPR]) {
#pragma unroll
                    for (int u = 0; u < UF; u += 2) {
                        const uint4 pq = *reinterpret_cast<const uint4 *>(&s_pq[i0 + u]);
                        hist_row_fast<FPL, NSC>(ww[u], sh0, lane4, pq.x, pq.y);
                        hist_row_fast<FPL, NSC>(ww[u + 1], sh0, lane4, pq.z, pq.w);
                    }
                };
                int i0 = warp * UF;
                if (i0 < cnt) load(i0, wa);
                while (i0 < cnt) {
                    const int i1 = i0 + NW * UF;
                    if (i1 < cnt) load(i1, wb);
                    update(i0, wa);
                    if (i1 >= cnt) break;
                    i0 = i1 + NW * UF;
                    if (i0 < cnt) load(i0, wa);
                    update(i1, wb);
                }
            }
        }
        if constexpr (HAS_ERA && REGULAR) {
            // era windows of an era-sorted chunk: rows [i_lo, i_hi), each
            // added into its era's slot (the slot's base joins the cell
            // address); the same branchless ping-pong steps as above, rows
            // past the window with zero increments
            fast = aligned && era_sorted;
            if (lane_live && fast) {
                constexpr int UE = 4;  // rows per step per warp
                uint32_t wa[UE][WPR], wb[UE][WPR];
                const uint32_t sh0 = (uint32_t)__cvta_generic_to_shared(sh32), lane4 = 4u * lane;
                const unsigned S32 = (unsigned)S;
                auto load = [&](int i0, uint32_t (&ww)[UE][WPR]) {
#pragma unroll
                    for (int u = 0; u < UE; ++u)
                        load_row<FPL>(tile + (unsigned long long)(unsigned)s_row[i0 + u] * S32, ww[u]);
                };
                auto update = [&](int i0, const uint32_t (&ww)[UE][WPR]) {
#pragma unroll
                    for (int u = 0; u < UE; ++u) {
                        const int i = i0 + u;
                        const bool in = i < i_hi;
                        const uint2 pq = in ? s_pq[i] : make_uint2(0u, 0u);
                        const uint32_t rb = sh0 + (in ? (uint32_t)(s_era[i] - e_lo) * (uint32_t)(ESLOT * 4) : 0u);
                        hist_row_fast<FPL, NSC>(ww[u], rb, lane4, pq.x, pq.y);
                    }
                };
                int i0 = i_lo + warp * UE;
                if (i0 < i_hi) load(i0, wa);
                while (i0 < i_hi) {
                    const int i1 = i0 + NW * UE;
                    if (i1 < i_hi) load(i1, wb);
                    update(i0, wa);
                    if (i1 >= i_hi) break;
                    i0 = i1 + NW * UE;
                    if (i0 < i_hi) load(i0, wa);
                    update(i1, wb);
                }
            }
        }
        if (lane_live && !fast) {
            // software pipeline: rows of step k+1 are loaded while step k's
            // cells are updated
            uint32_t w[U][WPR], wn[U][WPR];
            int2 rec[U], recn[U];                // {row or -1, era slot}
            auto fetch = [&](int i0, int2 (&rr)[U], uint32_t (&ww)[U][WPR]) {
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int i = i0 + NW * u;
                    int2 r4 = make_int2(i < i_hi && s_pq[i].x ? s_row[i] : -1, 0);
                    if (HAS_ERA && r4.x >= 0) {
                        const int e = s_era[i] - e_lo;
                        if (e < 0 || e >= ew_n) r4.x = -1;
                        r4.y = e;
                    }
                    rr[u] = r4;
#pragma unroll
                    for (int x = 0; x < WPR; ++x) ww[u][x] = 0u;
                    if (r4.x >= 0) {
                        const int8_t *src = tile + (long long)r4.x * S;
                        if (aligned) {
                            if constexpr (FPL == 16) {
                                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(src));
                                ww[u][0] = v.x; ww[u][1] = v.y; ww[u][2] = v.z; ww[u][3] = v.w;
                            } else if constexpr (FPL == 8) {
                                const uint2 v = __ldg(reinterpret_cast<const uint2 *>(src));
                                ww[u][0] = v.x; ww[u][1] = v.y;
                            } else {
                                ww[u][0] = __ldg(reinterpret_cast<const uint32_t *>(src));
                            }
                        } else {
                            const int nv = min(FPL, F - (f0 + FPL * lane));  // bytes inside the row
#pragma unroll
                            for (int j = 0; j < FPL; ++j)
                                if (j < nv) ww[u][j >> 2] |= (uint32_t)(uint8_t)__ldg(src + j) << (8 * (j & 3));
                        }
                    }
                }
            };
            fetch(i_lo + warp, rec, w);
            for (int i0 = i_lo + warp; i0 < i_hi; i0 += NW * U) {
                const int i1 = i0 + NW * U;
                if (i1 < i_hi) fetch(i1, recn, wn);
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    if (rec[u].x < 0) continue;
                    const uint32_t ra = sbase + (HAS_ERA ? (uint32_t)rec[u].y * (ESLOT * 4) : 0u);
                    const uint2 pq = s_pq[i0 + NW * u];
                    hist_row<FPL, NSC, REGULAR>(w[u], ra, pq.x, pq.y, B);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    rec[u] = recn[u];
#pragma unroll
                    for (int x = 0; x < WPR; ++x) w[u][x] = wn[u][x];
                }
            }
        }
        __syncthreads();
        // one era and a partial buffer: store the chunk's raw words (coalesced,
        // no atomics); k_hist_reduce sums the chunks of each node afterwards
        if (!HAS_ERA && part) {
            uint2 *dst = part + ((long long)c * ntile + ft) * (NSC * FT);
            for (int wi = threadIdx.x; wi < NSC * FT; wi += NT) dst[wi] = make_uint2(sh32[wi], sh32[NSC * FT + wi]);
            break;
        }
        // flush bins 0..B of every feature (the trash slot is dropped),
        // walking the words in layout order (conflict-free reads); a word's
        // cell index is decoded once for all era slots of the window
        {
            const long long estride = (long long)out.ks * B1;
            const long long wbase = (slot - out.slot0) * out.slot_elems + (long long)e_lo * estride;
            for (int wi = threadIdx.x; wi < NSC * FT; wi += NT) {
                const int jb = wi / (NSC * 64), rem = wi % (NSC * 64);
                const int sl = rem >> 6, r2 = rem & 63;
                if (sl > B) continue;
                const int jj = 2 * jb + (r2 >> 5), lj = r2 & 31;
                const int kp = s_kp[jj * 32 + lj];
                if (kp < 0) continue;
                const long long cidx = wbase + (long long)(kp / out.ks) * out.slice_stride +
                                       (long long)(kp % out.ks) * B1 + sl;
                for (int ew = 0; ew < nsl; ++ew) {
                    const uint32_t a = sh32[ew * ESLOT + wi];
                    if (a == 0u) continue;
                    const uint32_t bw = sh32[ew * ESLOT + NSC * FT + wi];
                    const int cntv = (int)(a >> HIST_CNT_SHIFT);
                    const long long gs = (long long)(int)bw * (1ll << HIST_LO_BITS) + (long long)(a & HIST_A_SUM_MASK);
                    const long long idx = cidx + (long long)ew * estride;
                    atomicAdd(reinterpret_cast<unsigned long long *>(out.g + idx), (unsigned long long)gs);
                    atomicAdd(reinterpret_cast<unsigned long long *>(out.c + idx), (unsigned long long)cntv);
                }
            }
        }
        if (!HAS_ERA) break;
        int m = INT_MAX;
        for (int i = threadIdx.x; i < cnt; i += NT)
            if (s_era[i] >= e_lo + ew_n) m = min(m, s_era[i]);
        m = block_min(m, s_red);  // also orders the flush before the next zeroing
        if (m == INT_MAX) break;
        e_lo = m;
    }
}

// The histogram kernel: CTA x builds item x -- chunk x / ntile of the
// level's list, feature tile x % ntile -- when the chunk exists (the grid is
// sized for the most chunks the level can have; the tiles of a chunk are
// neighbours, so they share its row records through L2, and CTAs past the
// list come last).
template <int FPL, int NT, int MINB, int NSC, int EWC, bool HAS_ERA, bool REGULAR>
__global__ void __launch_bounds__(NT, MINB) k_hist(
    const int8_t *__restrict__ bins, long long S, int F, const int *__restrict__ order,
    const int *__restrict__ q, const float *__restrict__ g, const int *shift,
    const int *__restrict__ era, const int *__restrict__ kpos, int k, int E, int B, int EW,
    const int4 *__restrict__ chunks, const int *nchunks, const wgb_node *__restrict__ lvl,
    const HistOut out, long long nrows, uint2 *__restrict__ part, int ntile) {
    pdl_wait();  // the previous kernel on the stream has completed
    const int c = blockIdx.x / ntile;
    if (c >= *nchunks) return;
    hist_item<FPL, NT, MINB, NSC, EWC, HAS_ERA, REGULAR>(c, blockIdx.x - c * ntile, ntile, bins, S, F, order, q, g,
                                                         shift, era, kpos, k, E, B, EW, chunks, lvl, out, nrows, part);
}

// Sums the per-chunk words k_hist stored for each node (one era): thread =
// two neighbouring cells of one feature tile (one 16-byte load per chunk)
// over a segment of `seg` consecutive chunks; chunks of one node are
// consecutive, so a thread adds its running totals to the node's int64
// cells whenever the node changes -- one atomic per cell, node and segment
// instead of one per chunk.  Both cells of a pair share their bin slot and
// feature pair index (cell indices 2i, 2i+1 differ in the lane only).
template <int FPL, int NSC>
__global__ void __launch_bounds__(256) k_hist_reduce(const uint2 *__restrict__ part, const int4 *__restrict__ chunks,
                                                     const int *nchunks, const wgb_node *__restrict__ lvl,
                                                     const int *__restrict__ kpos, int F, int B, int seg,
                                                     const HistOut out) {
    pdl_wait();  // the previous kernel on the stream has completed
    constexpr int FT = 32 * FPL, CELLS = NSC * FT;
    const int nch = *nchunks;
    const int wi = 2 * (blockIdx.x * 256 + threadIdx.x);
    if ((int)blockIdx.z * seg >= nch || wi >= CELLS) return;
    const int jb = wi / (NSC * 64), rem = wi % (NSC * 64);
    const int sl = rem >> 6, r2 = rem & 63;
    if (sl > B) return;  // trash slot
    const int jj = 2 * jb + (r2 >> 5), lj = r2 & 31;
    const int f = blockIdx.y * FT + lj * FPL + jj;
    const int kp0 = f < F ? kpos[f] : -1, kp1 = f + FPL < F ? kpos[f + FPL] : -1;
    if (kp0 < 0 && kp1 < 0) return;
    const int B1 = B + 1;
    const int ntile = gridDim.y;
    auto kofs = [&](int kp) {
        return (long long)(kp / out.ks) * out.slice_stride + (long long)(kp % out.ks) * B1 + sl;
    };
    const long long k0 = kp0 >= 0 ? kofs(kp0) : 0, k1 = kp1 >= 0 ? kofs(kp1) : 0;
    constexpr int UR = 8;  // chunk word pairs in flight per thread
    const uint4 *src = reinterpret_cast<const uint4 *>(part + (long long)blockIdx.y * CELLS + wi);
    const long long cstride = (long long)ntile * CELLS / 2;  // in uint4
    // segments z, z + gridDim.z, ... (the grid may hold fewer segments than the list)
    for (int c0 = blockIdx.z * seg; c0 < nch; c0 += gridDim.z * seg) {
        const int c1 = min(nch, c0 + seg);
        long long gs0 = 0, cn0 = 0, gs1 = 0, cn1 = 0;
        int node = chunks[c0].x;
        auto add = [&]() {
            const long long base = (long long)(lvl[node].slot - out.slot0) * out.slot_elems;
            if (kp0 >= 0 && cn0 != 0) {
                atomicAdd(reinterpret_cast<unsigned long long *>(out.g + base + k0), (unsigned long long)gs0);
                atomicAdd(reinterpret_cast<unsigned long long *>(out.c + base + k0), (unsigned long long)cn0);
            }
            if (kp1 >= 0 && cn1 != 0) {
                atomicAdd(reinterpret_cast<unsigned long long *>(out.g + base + k1), (unsigned long long)gs1);
                atomicAdd(reinterpret_cast<unsigned long long *>(out.c + base + k1), (unsigned long long)cn1);
            }
        };
        for (int cb = c0; cb < c1; cb += UR) {
            uint4 v[UR];
            int nd[UR];
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                const int c = cb + u;
                v[u] = c < c1 ? __ldcs(src + c * cstride) : make_uint4(0u, 0u, 0u, 0u);
                nd[u] = c < c1 ? chunks[c].x : node;
            }
#pragma unroll
            for (int u = 0; u < UR; ++u) {
                if (nd[u] != node) {
                    add();
                    node = nd[u];
                    gs0 = cn0 = gs1 = cn1 = 0;
                }
                cn0 += v[u].x >> HIST_CNT_SHIFT;
                gs0 += (long long)(int)v[u].y * (1ll << HIST_LO_BITS) + (long long)(v[u].x & HIST_A_SUM_MASK);
                cn1 += v[u].z >> HIST_CNT_SHIFT;
                gs1 += (long long)(int)v[u].w * (1ll << HIST_LO_BITS) + (long long)(v[u].z & HIST_A_SUM_MASK);
            }
        }
        add();
    }
}

// Feature width per lane and bin-slot capacity of the histogram kernel
// for a matrix (row stride S, F features, B bins); the same choice
// launch_hist makes.
static inline void hist_shape(long long S, int F, int B, int &fpl, int &nsc) {
    fpl = (S % 8 == 0 && F > 128 && B <= 32) ? 8 : 4;
    nsc = (B + 2 <= 8) ? 8 : (B + 2 <= 34 ? 34 : 130);
}

// Multiprocessors of the current device (cached per device).
static int num_sms() {
    static int cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

// Launch of the histogram kernel for one level: picks the feature width per
// lane, the bin-slot capacity and the era window from the row alignment,
// feature count, num_bins and era count.  Returns a cudaError_t.
static cudaError_t launch_hist(int grid_x, const int8_t *bins, long long S, int F, const int *order,
                               const int *q, const float *g, const int *shift, const int *era,
                               const int *kpos, int k, int E, int B, int EW, bool regular,
                               const int4 *chunks, const int *nchunks, const wgb_node *lvl,
                               const HistOut &out, long long nrows, cudaStream_t st, uint2 *part = nullptr) {
    const bool has_era = E > 1;
    int fpl, nsc;
    hist_shape(S, F, B, fpl, nsc);
#define WGB_HIST_CASE(FPL_, NT_, MINB_, NSC_, EWC_, ERA_, REG_)                                       \
    if (fpl == FPL_ && nsc == NSC_ && has_era == ERA_ && regular == REG_) {                            \
        auto fn = k_hist<FPL_, NT_, MINB_, NSC_, EWC_, ERA_, REG_>;                                    \
        const int ew = ERA_ ? (EW > 0 ? min(EW, EWC_) : EWC_) : 1;                                     \
        size_t smem = (size_t)EWC_ * 2 * NSC_ * 32 * FPL_ * 4;                                         \
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
        if (e != cudaSuccess) return e;                                                                \
        const int ntile = (F + 32 * FPL_ - 1) / (32 * FPL_);                                          \
        e = launch_pdl(fn, dim3((unsigned)grid_x * ntile), dim3(NT_), smem, st, bins, S, F, order, q, g, \
                       shift, era, kpos, k, E, B, ew, chunks, nchunks, lvl, out, nrows, part, ntile);     \
        if (e != cudaSuccess || !part || ERA_) return e;                                              \
        const int seg = 16;                                                                            \
        dim3 rg((unsigned)((NSC_ * 16 * FPL_ + 255) / 256), (unsigned)ntile, (unsigned)((grid_x + seg - 1) / seg)); \
        return launch_pdl(k_hist_reduce<FPL_, NSC_>, rg, dim3(256), 0, st, part, chunks, nchunks, lvl, kpos, \
                          F, B, seg, out);                                                             \
    }
#define WGB_HIST_REG(FPL_, NT_, MINB_, NSC_, EWC_, ERA_) \
    WGB_HIST_CASE(FPL_, NT_, MINB_, NSC_, EWC_, ERA_, true) WGB_HIST_CASE(FPL_, NT_, MINB_, NSC_, EWC_, ERA_, false)
    // one era: 2 CTAs x 16 warps per SM
    WGB_HIST_REG(8, 512, 2, 34, 1, false)
    WGB_HIST_REG(8, 512, 2, 8, 1, false)
    WGB_HIST_REG(4, 256, 1, 34, 1, false)
    WGB_HIST_REG(4, 256, 1, 8, 1, false)
    WGB_HIST_REG(4, 256, 1, 130, 1, false)
    // eras: several era slots per window; up to 8 bins, 4 slots keep two
    // CTAs per SM (one CTA's window barriers overlap the other's updates)
    WGB_HIST_REG(8, 512, 2, 8, 4, true)
    WGB_HIST_REG(8, 512, 1, 34, 2, true)
    WGB_HIST_REG(4, 256, 1, 8, 8, true)
    WGB_HIST_REG(4, 256, 1, 34, 4, true)
    WGB_HIST_REG(4, 256, 1, 130, 1, true)
#undef WGB_HIST_REG
#undef WGB_HIST_CASE
    return cudaErrorInvalidValue;
}

// ====================================================================== //
// split search                                                           //
// ====================================================================== //

// Single-era split search (criterion = gain, core.py:577-579): one warp =
// (node, feature position j), SPLIT_WARPS features per block.  The warp
// stages the feature's B bins in shared memory (G = float(sum q) * 2^-s,
// H = float(count)); every lane then forms the reference's sequential fp32
// sums (totals over all B bins, prefix over b < B-1, best_split_kernel.cu:
// 25-53) from the staged values -- the additions stay in bin order, so the
// sums are the reference's bit for bit -- and evaluates the split points
// b = lane, lane + 32, ...  (one gain per lane instead of B-1 per thread:
// a level with one node still fills the GPU).  A node whose histogram was
// not built (the larger child, core.py:636-643) first becomes parent -
// built sibling, written back in place of the parent unless this is the
// tree's last split level (its children are leaves; nothing reads it).
// Block arg-max -> cand[node][blk].
template <int NBW>  // split points per lane: ceil((B-1) / 32)
__global__ void __launch_bounds__(SPLIT_WARPS * 32) k_split(
    const wgb_node *__restrict__ lvl, const int *nn_d, long long *hg, long long *hc, long long slot_elems,
    int k, int jofs, int B, const int *shift,
    float mcw, float eps, float msg, int4 *cand, int nblk, float *crit_out, bool writeback) {
    pdl_wait();  // the previous kernel on the stream has completed
    __shared__ float sG[SPLIT_WARPS][32 * NBW + 1], sH[SPLIT_WARPS][32 * NBW + 1];
    __shared__ Key s_k[SPLIT_WARPS];
    const int n = blockIdx.x / nblk, jb = blockIdx.x - n * nblk;  // node, feature block
    if (n >= *nn_d) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int j = jb * SPLIT_WARPS + warp;
    const int nb = B - 1;
    Key best = key_none();
    if (j < k) {
        const wgb_node &nd = lvl[n];
        const float inv = pow2f(-shift[node_tree(nd.built)]);
        const long long off = nd.slot * slot_elems + (long long)j * (B + 1);
        if (node_built(nd.built)) {
            for (int b = lane; b < B; b += 32) {
                sG[warp][b] = __fmul_rn(__ll2float_rn(hg[off + b]), inv);
                sH[warp][b] = __ll2float_rn(hc[off + b]);
            }
        } else {
            // sibling = parent - built sibling, in place of the parent (whose
            // slot it inherits), for all B+1 cells; exact in integers
            const long long boff = lvl[n ^ 1].slot * slot_elems + (long long)j * (B + 1);
            for (int b = lane; b <= B; b += 32) {
                const long long gv = hg[off + b] - hg[boff + b];
                const long long cv = hc[off + b] - hc[boff + b];
                if (writeback) {
                    hg[off + b] = gv;
                    hc[off + b] = cv;
                }
                if (b < B) {
                    sG[warp][b] = __fmul_rn(__ll2float_rn(gv), inv);
                    sH[warp][b] = __ll2float_rn(cv);
                }
            }
        }
        __syncwarp();
        const float *g = sG[warp], *h = sH[warp];
        float GT = 0.0f, HT = 0.0f;
        for (int b = 0; b < B; ++b) {
            GT = __fadd_rn(GT, g[b]);
            HT = __fadd_rn(HT, h[b]);
        }
        float GL = 0.0f, HL = 0.0f;
        int b = 0;
#pragma unroll
        for (int i = 0; i < NBW; ++i) {
            const int bi = lane + 32 * i;  // this lane's i-th split point
            if (bi >= nb) break;
            for (; b <= bi; ++b) {
                GL = __fadd_rn(GL, g[b]);
                HL = __fadd_rn(HL, h[b]);
            }
            const SplitEval r = eval_split(GL, HL, GT, HT, mcw, eps);
            if (crit_out && n == 0) crit_out[(jofs + j) * nb + bi] = r.gain;
            const Key kk{0, r.gain > msg ? r.gain : -INFINITY, (jofs + j) * nb + bi};
            if (key_better(kk, best)) best = kk;
        }
    }
    best = warp_key_max(best);
    if (lane == 0) s_k[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < SPLIT_WARPS; ++w)
            if (key_better(s_k[w], best)) best = s_k[w];
        cand[(long long)n * nblk + jb] = make_int4(best.A, __float_as_int(best.c), best.idx, 0);
    }
}

// ---------------------------------------------------------------------- //
// Era criterion in the order of torch's CUDA mean                         //
// ---------------------------------------------------------------------- //
//
// The reference's DES criterion is per_era_gain.mean(dim=0) on CUDA
// (core.py:581-582).  torch's reduce kernel (ATen/native/cuda/Reduce.cuh)
// does not add the eras one after another: depending on E and on the output
// count M = k*(B-1) it spreads them over the rows of a block and over
// several blocks, gives each thread four accumulators, and combines the
// partial sums by fixed trees.  fp32 addition is not associative, so the
// criterion is reproduced bit for bit only by adding in that order.  The
// host turns the launch shape into a plan: a schedule of the eras in the
// order they are first needed and a program for a small accumulator stack
// per output cell:
//     ERA_PUSH0  push the running accumulator, start a new one at 0
//     ERA_ADD2   accumulator = popped value + accumulator
//     ERA_ADD    accumulator += gain of the next scheduled era
// which k_split_eras runs for every (feature, bin) cell of its block.
enum : uint8_t { ERA_PUSH0 = 0, ERA_ADD2 = 1, ERA_ADD = 2 };

// Launch shape of torch's reduce kernel for mean(dim=0) of a contiguous fp32
// [E, M] tensor (setReduceConfig / set_block_dimension, torch 2.11): the eras
// go to `rows` block rows and `ctas` blocks.
static void era_mean_layout(int E, long long M, int num_sms, int max_threads_per_sm, int &rows, int &ctas) {
    int vec = 4;
    while (M % vec) vec >>= 1;
    const long long dim0 = M / vec;
    const int mnt = 512 / vec;
    auto p2 = [mnt](long long n) {
        if (n >= mnt) return mnt;
        int p = 1;
        while ((long long)p * 2 <= n) p *= 2;
        return p;
    };
    int bw = std::min(p2(dim0), 32);
    const int bh = std::min(p2(E), mnt / bw);
    bw = std::min(p2(dim0), mnt / bh);
    rows = 1;
    ctas = 1;
    if (!(E >= std::min(bh * 16, 256))) return;  // each thread sums whole outputs
    rows = bh;
    const long long vpt = (E + bh - 1) / bh;
    const long long grid = (dim0 + bw - 1) / bw;
    const long long target = (long long)num_sms * (max_threads_per_sm / (bw * bh));
    if (vpt >= 256 && grid <= target) {
        const long long c1 = (target + grid - 1) / grid, c2 = (vpt + 15) / 16, c3 = (vpt + 255) / 256;
        const long long c = std::max(std::min(c1, c2), c3);
        if (c > 1) ctas = (int)c;
    }
}

struct EraPlanWriter {
    int32_t *sched;
    uint8_t *ops;
    long long cap, n = 0, ns = 0;
    int sp = 0, depth = 0;
    void op(uint8_t o) {
        if (ops && n < cap) ops[n] = o;
        ++n;
        if (o == ERA_PUSH0) depth = std::max(depth, ++sp);
        if (o == ERA_ADD2) --sp;
    }
    void era(int e) {
        if (sched) sched[ns] = e;
        ++ns;
        op(ERA_ADD);
    }
};

// thread_reduce_impl of one thread: its t-th era (e = lane + L*t) goes to
// accumulator t % 4; the result is ((a0 + a1) + a2) + a3.
static void era_plan_lane(EraPlanWriter &w, int E, int lane, int L) {
    for (int a = 0; a < 4; ++a) {
        w.op(ERA_PUSH0);
        for (long long e = lane + (long long)L * a; e < E; e += 4ll * L) w.era((int)e);
        if (a) w.op(ERA_ADD2);
    }
}

// block_y_reduce's halving tree (r[y] += r[y + off], off = count/2 .. 1)
// over the values leaf(first + stride*i), i < count (a power of two): the
// result is tree(even positions) + tree(odd positions) of that list, so
// leaf y meets leaf y + count/2 first.
template <class Leaf>
static void era_plan_tree(EraPlanWriter &w, int first, int stride, int count, Leaf &&leaf) {
    if (count == 1) {
        leaf(first);
        return;
    }
    era_plan_tree(w, first, stride * 2, count / 2, leaf);
    era_plan_tree(w, first + stride, stride * 2, count / 2, leaf);
    w.op(ERA_ADD2);
}

// The whole plan: per block c the tree over its rows' lanes y + rows*c;
// with several blocks, row y of the last one adds the block results
// c = y, y + rows, ... in order from 0 (global_reduce), then the tree again.
static void era_plan(EraPlanWriter &w, int E, int rows, int ctas) {
    const int L = rows * ctas;
    auto block = [&](int c) {
        era_plan_tree(w, 0, 1, rows, [&](int y) { era_plan_lane(w, E, y + rows * c, L); });
    };
    if (ctas == 1) {
        block(0);
        return;
    }
    era_plan_tree(w, 0, 1, rows, [&](int y) {
        w.op(ERA_PUSH0);
        for (int c = y; c < ctas; c += rows) {
            block(c);
            w.op(ERA_ADD2);
        }
    });
}

// Era split search (E > 1) with the eras spread over warps: block = one
// node x FB features, eras in batches of EB taken in the plan's schedule
// order, one warp per era.  Phase 1: a warp stages its era's FB feature
// rows in shared memory with coalesced loads (G = float(sum q) * 2^-s,
// H = float(count); odd row stride, conflict-free), then lane f scans
// feature f's bins with the reference arithmetic and leaves the era's B-1
// gains and directions in shared memory.  Phase 2: thread = (bin, feature)
// cells run the plan's program over the batch -- the criterion is then
// torch's CUDA mean bit for bit -- and add the directions to an integer
// agreement (exact in any order).  Block arg-max -> cand[node][blk]
// (ceil(k/FB) blocks).
constexpr int SPLIT_ERA_EB = 8;   // eras per batch (= warps)

template <int NB>
struct EraSplitShape {
    static constexpr int FB = NB <= 32 ? 32 : 8;      // features per block
    static constexpr int IPT = (FB * NB + 255) / 256;  // cells per thread
};

static inline int split_era_fb(int B) { return B - 1 <= 32 ? 32 : 8; }

static inline size_t split_eras_smem(int B, int NB, int FB, int depth) {
    const int B1p = (B + 1) | 1;
    const int ipt = (FB * NB + 255) / 256;
    return (size_t)SPLIT_ERA_EB * 2 * FB * B1p * sizeof(float) +      // staged rows
           (size_t)SPLIT_ERA_EB * NB * FB * sizeof(float) +           // gains
           (size_t)depth * ipt * 256 * sizeof(float) +                // accumulator stacks
           (size_t)SPLIT_ERA_EB * NB * FB;                            // directions
}

template <int NB>
__global__ void __launch_bounds__(256) k_split_eras(
    const wgb_node *__restrict__ lvl, const int *nn_d, long long *hg, long long *hc, long long slot_elems,
    int k, int kl, int jofs, int E, int B, const int *shift,
    float mcw, float eps, float msg, float factor, const int *__restrict__ sched,
    const uint8_t *__restrict__ ops, int nops, int depth, int4 *cand, int nblk, float *crit_out,
    bool writeback) {
    pdl_wait();  // the previous kernel on the stream has completed
    constexpr int FB = EraSplitShape<NB>::FB, IPT = EraSplitShape<NB>::IPT, EB = SPLIT_ERA_EB;
    extern __shared__ float s_era_split[];
    const int n = blockIdx.x / nblk, jb = blockIdx.x - n * nblk;  // node, feature block
    if (n >= *nn_d) return;
    const int j0 = jb * FB;
    const int nf = min(FB, k - j0);
    const int B1 = B + 1, nb = B - 1, B1p = B1 | 1;
    const float inv = pow2f(-shift[node_tree(lvl[n].built)]);
    const long long slot = lvl[n].slot;
    const bool built = node_built(lvl[n].built);
    const long long bslot = built ? slot : lvl[n ^ 1].slot;  // built sibling of an unbuilt node
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float *stg = s_era_split + warp * 2 * FB * B1p;
    float *sg = s_era_split + EB * 2 * FB * B1p;
    float *stk = sg + EB * NB * FB;
    signed char *sd = reinterpret_cast<signed char *>(stk + depth * IPT * 256);
    float acc[IPT];
    int ds[IPT];
#pragma unroll
    for (int t = 0; t < IPT; ++t) {
        acc[t] = 0.0f;
        ds[t] = 0;
    }
    int pc = 0, sp = 0;  // program counter and stack depth (uniform over the block)
    auto step = [&](uint8_t op) {
        if (op == ERA_PUSH0) {
#pragma unroll
            for (int t = 0; t < IPT; ++t) {
                stk[(sp * IPT + t) * 256 + threadIdx.x] = acc[t];
                acc[t] = 0.0f;
            }
            ++sp;
        } else {  // ERA_ADD2
            --sp;
#pragma unroll
            for (int t = 0; t < IPT; ++t) acc[t] = __fadd_rn(stk[(sp * IPT + t) * 256 + threadIdx.x], acc[t]);
        }
    };
    for (int e0 = 0; e0 < E; e0 += EB) {
        const int ne = min(EB, E - e0);
        if (warp < ne) {
            const int e = sched[e0 + warp];
            const long long base = slot * slot_elems + ((long long)e * kl + j0) * B1;
            const long long bbase = bslot * slot_elems + ((long long)e * kl + j0) * B1;
            // groups of LU cells per lane: every load of a group is issued
            // before its write-back stores (which may alias later loads as
            // far as the compiler knows), so a group costs one round trip
            constexpr int LU = 4;
            const int ncell = nf * B1;
            // t / B1 without an integer division: t < 2^12, so the fp32
            // product (t + 0.5) / B1 stays more than 0.5/B1 away from an
            // integer and truncates to the exact quotient
            const float rB1 = 1.0f / (float)B1;
            for (int t0 = lane; t0 < ncell; t0 += 32 * LU) {
                long long gv[LU], cv[LU], gb[LU], cb[LU];
#pragma unroll
                for (int u = 0; u < LU; ++u) {
                    const int t = t0 + 32 * u;
                    gv[u] = cv[u] = gb[u] = cb[u] = 0;
                    if (t < ncell) {
                        gv[u] = hg[base + t];
                        cv[u] = hc[base + t];
                        if (!built) {
                            gb[u] = hg[bbase + t];
                            cb[u] = hc[bbase + t];
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < LU; ++u) {
                    const int t = t0 + 32 * u;
                    if (t >= ncell) break;
                    const int f = (int)(((float)t + 0.5f) * rB1), b = t - f * B1;
                    long long g = gv[u], c = cv[u];
                    if (!built) {  // sibling = parent - built sibling, written back in place
                        g -= gb[u];
                        c -= cb[u];
                        if (writeback) {  // (not at the last split level: its children are leaves)
                            hg[base + t] = g;
                            hc[base + t] = c;
                        }
                    }
                    stg[f * B1p + b] = __fmul_rn(__ll2float_rn(g), inv);
                    stg[(FB + f) * B1p + b] = __int2float_rn((int)c);  // counts < 2^31: the same float
                }
            }
            __syncwarp();
            if (lane < nf) {
                const float *g = stg + lane * B1p, *h = stg + (FB + lane) * B1p;
                float GT = 0.0f, HT = 0.0f;
                for (int b = 0; b < B; ++b) {
                    GT = __fadd_rn(GT, g[b]);
                    HT = __fadd_rn(HT, h[b]);
                }
                const float t3 = parent_term(GT, HT, eps);
                float GL = 0.0f, HL = 0.0f;
                for (int b = 0; b < nb; ++b) {
                    GL = __fadd_rn(GL, g[b]);
                    HL = __fadd_rn(HL, h[b]);
                    const SplitEval r = eval_split_pt(GL, HL, GT, HT, t3, mcw, eps);
                    sg[(warp * NB + b) * FB + lane] = r.gain;
                    sd[(warp * NB + b) * FB + lane] = (signed char)r.dir;
                }
            }
        }
        __syncthreads();
        for (int w = 0; w < ne; ++w) {
            uint8_t op;
            while (pc < nops && (op = __ldg(ops + pc++)) != ERA_ADD) step(op);
#pragma unroll
            for (int t = 0; t < IPT; ++t) {
                const int it = threadIdx.x + 256 * t;  // it / FB < NB by construction
                acc[t] = __fadd_rn(acc[t], sg[(w * NB) * FB + it]);
                ds[t] += sd[(w * NB) * FB + it];
            }
        }
        __syncthreads();  // the batch's gains are consumed before the next batch writes them
    }
    while (pc < nops) step(__ldg(ops + pc++));
    Key best = key_none();
#pragma unroll
    for (int t = 0; t < IPT; ++t) {
        const int it = threadIdx.x + 256 * t;
        const int b = it / FB, f = it - b * FB;
        if (b < nb && f < nf) {
            const float cr = __fmul_rn(acc[t], factor);
            if (crit_out && n == 0) crit_out[(jofs + j0 + f) * nb + b] = cr;
            const Key kk{abs(ds[t]), cr > msg ? cr : -INFINITY, (jofs + j0 + f) * nb + b};
            if (key_better(kk, best)) best = kk;
        }
    }
    best = warp_key_max(best);
    __shared__ Key s_k[8];
    if (lane == 0) s_k[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w)
            if (key_better(s_k[w], best)) best = s_k[w];
        cand[(long long)n * nblk + jb] = make_int4(best.A, __float_as_int(best.c), best.idx, 0);
    }
}

// Next level's node records, by one block: children of splitting nodes in
// node order, smaller child built (left on ties, core.py:636), the built
// child in a fresh slot 2^d + r, the sibling in the parent's slot.  The
// level's records were written by other blocks of the same launch: they are
// read through L2 (ld.global.cg).
__device__ void plan_next_level(wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt, int *nn, int d,
                                const int *shift, int ntree, int *s_scan) {
    const int nnd = __ldcg(nn + d);
    int base = 0;
    for (int b0 = 0; b0 < nnd; b0 += blockDim.x) {
        const int i = b0 + threadIdx.x;
        const int fp = i < nnd ? __ldcg(&lvl[i].fpos) : -1;
        const int f = fp >= 0 ? 1 : 0;
        int tot;
        const int r = base + block_scan_excl(f, s_scan, tot);
        if (f) {
            wgb_node &p = lvl[i];
            p.child = 2 * r;
            const long long cl = __ldcg(&p.lcount), cnt = __ldcg(&p.count);
            const long long sl = __ldcg(&p.lsumq), sm = __ldcg(&p.sumq);
            const long long cr = cnt - cl, sr = sm - sl;
            const int pslot = __ldcg(&p.slot);
            const int tree = node_tree(__ldcg(&p.built));
            const float inv = pow2f(-shift[tree]);
            const int builtL = cl <= cr;
            const int fresh = (ntree << d) + r;  // level d+1's built slots: [ntree 2^d, ntree 2^(d+1))
            wgb_node L, R;
            L.sumq = sl; L.count = cl; R.sumq = sr; R.count = cr;
            L.lsumq = R.lsumq = 0; L.lcount = R.lcount = 0;
            L.lstart = R.lstart = 0; L.lcnt = R.lcnt = 0;
            L.built = node_flags(builtL, tree); R.built = node_flags(!builtL, tree);
            L.slot = builtL ? fresh : pslot;
            R.slot = builtL ? pslot : fresh;
            L.fpos = R.fpos = -1; L.bin = R.bin = 0; L.child = R.child = -1;
            L.leaf = canon_leaf(sl, cl, inv);
            R.leaf = canon_leaf(sr, cr, inv);
            nxt[2 * r] = L;
            nxt[2 * r + 1] = R;
        } else if (i < nnd) {
            lvl[i].child = -1;
        }
        base += tot;
    }
    if (threadIdx.x == 0) nn[d + 1] = 2 * base;
}

// Row layout of the next level for the one-launch partition.  Per
// splitting node n (node order): part[n] = {left cursor 0, start ns of n's
// children in the next order, left count, right cursor 0}; the partition
// puts n's left rows at ns, ns+1, ... and its right rows at ns+lcnt-1,
// ns+lcnt-2, ...  Single-rank fits (local_known): a node's exact left count
// (lcount, from its histogram) is also its local one, so the children's
// segments [ns, ns+L) and [ns+L, ns+lcnt), the next level's active rows and
// (chunks != NULL) its histogram chunk list are planned here.  Multi-rank
// fits know only global counts: the partition's last CTA finishes the
// layout from its left cursors (finish_children).  Runs after
// plan_next_level in the same block.
__device__ void plan_children(const wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt, const int *nn,
                              int *nact, int d, int4 *part, int4 *chunks, int *nchunks, int chunk_cap, int wave,
                              bool local_known, int *s_scan) {
    __syncthreads();  // nxt records and nn[d + 1] of plan_next_level
    const int nnd = __ldcg(nn + d);
    int base = 0;
    for (int b0 = 0; b0 < nnd; b0 += blockDim.x) {
        const int i = b0 + threadIdx.x;
        const bool spl = i < nnd && __ldcg(&lvl[i].fpos) >= 0;
        const int v = spl ? __ldcg(&lvl[i].lcnt) : 0;
        int tot;
        const int ns = base + block_scan_excl(v, s_scan, tot);
        if (spl) {
            const int L = local_known ? (int)__ldcg(&lvl[i].lcount) : 0;
            part[i] = make_int4(0, ns, L, 0);
            if (local_known) {
                const int c = __ldcg(&lvl[i].child);
                nxt[c].lstart = ns;
                nxt[c].lcnt = L;
                nxt[c + 1].lstart = ns + L;
                nxt[c + 1].lcnt = v - L;
            }
        }
        base += tot;
    }
    if (!local_known) return;
    if (threadIdx.x == 0) nact[d + 1] = base;
    if (chunks) {
        __syncthreads();
        plan_chunks(nxt, nn[d + 1], chunks, nchunks, chunk_cap, wave);
    }
}

// Multi-rank fits, by the partition's last CTA: each splitting node's local
// left count is its final left cursor part[n].x; the children's segments,
// the next level's active rows and (chunks != NULL) its chunk list follow.
__device__ void finish_children(const wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt, const int *nn,
                                int *nact, int d, const int4 *part, int4 *chunks, int *nchunks, int chunk_cap,
                                int wave, int *s_scan) {
    const int nnd = __ldcg(nn + d);
    int base = 0;
    for (int b0 = 0; b0 < nnd; b0 += blockDim.x) {
        const int i = b0 + threadIdx.x;
        const bool spl = i < nnd && __ldcg(&lvl[i].fpos) >= 0;
        const int v = spl ? __ldcg(&lvl[i].lcnt) : 0;
        int tot;
        block_scan_excl(v, s_scan, tot);
        if (spl) {
            const int L = __ldcg(&part[i].x), ns = __ldcg(&part[i].y);
            const int c = __ldcg(&lvl[i].child);
            nxt[c].lstart = ns;
            nxt[c].lcnt = L;
            nxt[c + 1].lstart = ns + L;
            nxt[c + 1].lcnt = v - L;
        }
        base += tot;
    }
    if (threadIdx.x == 0) nact[d + 1] = base;
    if (chunks) {
        __syncthreads();
        plan_chunks(nxt, __ldcg(nn + d + 1), chunks, nchunks, chunk_cap, wave);
    }
}

// Per node: final arg-max, per-era gain of the chosen split (importance,
// core.py:624-627) and the exact left-child totals (bins <= bin plus the
// negative-bin slot, which always goes left).  The last block of the launch
// to finish then plans the next level (plan_next_level); `done` is a
// zero-initialised counter that this block returns to zero.
// Feature-sliced fits (win != NULL): the arg-max, totals and gains are this
// rank's best among its own positions [jofs, jofs + k) (pool layout width
// kl), written as the node's record in this rank's region of win --
// {key A, key c, key idx, -, lcount (int64), lsumq (int64), gain[E]} -- for
// k_split_pick to choose from after the all-gather; nothing is planned.
__global__ void __launch_bounds__(256) k_split_final(
    wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt, int *nn, int d, int ntree,
    const long long *__restrict__ hg, const long long *__restrict__ hc, long long slot_elems, int kl, int jofs,
    int E, int B, const int *shift, float mcw, float eps, const int4 *__restrict__ cand, int nblk, float *era_gain,
    int *done, bool writeback, int4 *part, int *nact, int4 *chunks, int *nchunks, int chunk_cap, int *win,
    int win_words, int wslice, int wave, bool local_known) {
    pdl_wait();  // the previous kernel on the stream has completed
    const int n = blockIdx.x;
    __shared__ Key s_best, s_kw[8];
    __shared__ long long s_c[8], s_g[8];
    __shared__ int s_scan[33];
    __shared__ bool s_last;
    int *rec = win ? win + ((long long)wslice * (ntree << d) + n) * win_words : nullptr;
    if (n < nn[d]) {
        const float inv = pow2f(-shift[node_tree(lvl[n].built)]);
        {   // arg-max over the node's candidate blocks, all threads
            Key best = key_none();
            for (int b = threadIdx.x; b < nblk; b += blockDim.x) {
                const int4 v = cand[(long long)n * nblk + b];
                const Key kk{v.x, __int_as_float(v.y), v.z};
                if (key_better(kk, best)) best = kk;
            }
            best = warp_key_max(best);
            if ((threadIdx.x & 31) == 0) s_kw[threadIdx.x >> 5] = best;
            __syncthreads();
            if (threadIdx.x == 0) {
                for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
                    if (key_better(s_kw[w], best)) best = s_kw[w];
                s_best = best;
            }
            __syncthreads();
        }
        const Key best = s_best;
        wgb_node &nd = lvl[n];
        if (!(best.c > -INFINITY)) {
            if (threadIdx.x == 0) {
                if (rec) {
                    rec[0] = best.A;
                    rec[1] = __float_as_int(best.c);
                    rec[2] = best.idx;
                    rec[3] = 0;
                    *reinterpret_cast<long long *>(rec + 4) = 0;
                    *reinterpret_cast<long long *>(rec + 6) = 0;
                } else {
                    nd.fpos = -1;
                    nd.lsumq = 0;
                    nd.lcount = 0;
                }
            }
        } else {
            const int nb = B - 1, B1 = B + 1;
            const int fpos = best.idx / nb, bin = best.idx - fpos * nb;
            const int fl = fpos - jofs;  // position in the pool's layout
            const long long slot = nd.slot;
            // an unbuilt node's histogram is parent - built sibling; the split
            // search wrote it back except at the last split level
            const bool sub = !node_built(nd.built) && !writeback;
            const long long bslot = sub ? lvl[n ^ 1].slot : 0;
            float *gain_out = rec ? reinterpret_cast<float *>(rec + 8) : era_gain + (long long)n * E;
            // one era: the block loads the feature's cells in parallel first
            // (the sums below stay sequential in bin order)
            __shared__ long long s_cg[128], s_cc[128];
            const bool staged = E == 1;
            if (staged) {
                const long long off = slot * slot_elems + (long long)fl * B1;
                const long long boff = bslot * slot_elems + (long long)fl * B1;
                for (int b = threadIdx.x; b < B1; b += blockDim.x) {
                    s_cg[b] = hg[off + b] - (sub ? hg[boff + b] : 0ll);
                    s_cc[b] = hc[off + b] - (sub ? hc[boff + b] : 0ll);
                }
                __syncthreads();
            }
            long long lc = 0, ls = 0;
            for (int e = threadIdx.x; e < E; e += blockDim.x) {
                const long long off = slot * slot_elems + ((long long)e * kl + fl) * B1;
                const long long boff = bslot * slot_elems + ((long long)e * kl + fl) * B1;
                auto gq = [&](int b) { return staged ? s_cg[b] : hg[off + b] - (sub ? hg[boff + b] : 0ll); };
                auto cq = [&](int b) { return staged ? s_cc[b] : hc[off + b] - (sub ? hc[boff + b] : 0ll); };
                float GT = 0.0f, HT = 0.0f, GL = 0.0f, HL = 0.0f;
                for (int b = 0; b < B; ++b) {
                    const long long gb = gq(b), cb = cq(b);
                    float gv = __fmul_rn(__ll2float_rn(gb), inv);
                    float hv = __ll2float_rn(cb);
                    GT = __fadd_rn(GT, gv);
                    HT = __fadd_rn(HT, hv);
                    if (b <= bin) {
                        GL = __fadd_rn(GL, gv);
                        HL = __fadd_rn(HL, hv);
                        lc += cb;
                        ls += gb;
                    }
                }
                lc += cq(B);
                ls += gq(B);
                gain_out[e] = eval_split(GL, HL, GT, HT, mcw, eps).gain;
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
                if (rec) {
                    rec[0] = best.A;
                    rec[1] = __float_as_int(best.c);
                    rec[2] = best.idx;
                    rec[3] = 0;
                    *reinterpret_cast<long long *>(rec + 4) = lc;
                    *reinterpret_cast<long long *>(rec + 6) = ls;
                } else {
                    nd.fpos = fpos;
                    nd.bin = bin;
                    nd.lcount = lc;
                    nd.lsumq = ls;
                }
            }
        }
    }
    if (rec) return;  // k_split_pick decides and plans
    // the last block to get here plans the next level
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    plan_next_level(lvl, nxt, nn, d, shift, ntree, s_scan);
    if (part) plan_children(lvl, nxt, nn, nact, d, part, chunks, nchunks, chunk_cap, wave, local_known, s_scan);
    if (threadIdx.x == 0) *done = 0;
}

// Feature-sliced fits, after the all-gather of win: per node the best of the
// ranks' records by the same key order (so the choice is the one a single
// rank searching every position makes), its totals and per-era gains into
// the node; the last block plans the next level and (part != NULL: the
// one-launch partition) each splitting node's children range.
__global__ void __launch_bounds__(256) k_split_pick(wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt, int *nn,
                                                    int d, int ntree, int B, int E, const int *shift,
                                                    const int *__restrict__ win, int win_words, int nslice,
                                                    float *era_gain, int *done, int4 *part) {
    pdl_wait();  // the previous kernel on the stream has completed
    const int n = blockIdx.x;
    __shared__ int s_w;
    __shared__ int s_scan[33];
    __shared__ bool s_last;
    const long long region = (long long)(ntree << d) * win_words;
    if (n < nn[d]) {
        if (threadIdx.x == 0) {
            Key best = key_none();
            int w = -1;
            for (int r = 0; r < nslice; ++r) {
                const int *rc = win + r * region + (long long)n * win_words;
                const Key kk{rc[0], __int_as_float(rc[1]), rc[2]};
                if (key_better(kk, best)) {
                    best = kk;
                    w = r;
                }
            }
            wgb_node &nd = lvl[n];
            if (w < 0 || !(best.c > -INFINITY)) {
                nd.fpos = -1;
                nd.lsumq = 0;
                nd.lcount = 0;
                w = -1;
            } else {
                const int *rc = win + w * region + (long long)n * win_words;
                const int nb = B - 1;
                nd.fpos = best.idx / nb;
                nd.bin = best.idx % nb;
                nd.lcount = *reinterpret_cast<const long long *>(rc + 4);
                nd.lsumq = *reinterpret_cast<const long long *>(rc + 6);
            }
            s_w = w;
        }
        __syncthreads();
        if (s_w >= 0) {
            const float *g = reinterpret_cast<const float *>(win + s_w * region + (long long)n * win_words + 8);
            for (int e = threadIdx.x; e < E; e += blockDim.x) era_gain[(long long)n * E + e] = g[e];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        s_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    plan_next_level(lvl, nxt, nn, d, shift, ntree, s_scan);
    if (part) plan_children(lvl, nxt, nn, nullptr, d, part, nullptr, nullptr, 0, 0, false, s_scan);
    if (threadIdx.x == 0) *done = 0;
}

// ====================================================================== //
// partition                                                              //
// ====================================================================== //

// bins [N][S] -> out [F][NT] (NT = N rounded up to 16).  Tile = 128 rows x
// 128 features through shared memory; 16-byte loads and stores.
__global__ void __launch_bounds__(256) k_bins_fm(const int8_t *__restrict__ bins, long long N, long long S, int F,
                                                 long long NT, int8_t *__restrict__ out) {
    __shared__ __align__(16) uint8_t t[128][144];
    const long long r0 = (long long)blockIdx.x * 128;
    const int f0 = blockIdx.y * 128;
    for (int i = threadIdx.x; i < 128 * 8; i += 256) {
        const int rr = i >> 3, c16 = (i & 7) * 16;
        const long long r = r0 + rr;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < N && f0 + c16 < S) v = __ldg(reinterpret_cast<const uint4 *>(bins + r * S + f0 + c16));
        *reinterpret_cast<uint4 *>(&t[rr][c16]) = v;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 128 * 8; i += 256) {
        const int fl = i >> 3, r16 = (i & 7) * 16;
        const int f = f0 + fl;
        if (f >= F || r0 + r16 >= NT) continue;
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
            w[q] = (uint32_t)t[r16 + 4 * q][fl] | ((uint32_t)t[r16 + 4 * q + 1][fl] << 8) |
                   ((uint32_t)t[r16 + 4 * q + 2][fl] << 16) | ((uint32_t)t[r16 + 4 * q + 3][fl] << 24);
        *reinterpret_cast<uint4 *>(out + (long long)f * NT + r0 + r16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// flag per position: 1 left, 0 right, 2 node is a leaf; left count per tile.
// The split feature's bin comes from the feature-major copy when there is
// one (rows of a node are ascending, so neighbouring positions read
// neighbouring bytes), else from the row-major matrix.
__global__ void __launch_bounds__(PART_THREADS) k_flags(
    const wgb_node *__restrict__ lvl, const int *nn_d, const int *nact_d, const int *__restrict__ order,
    const int *__restrict__ posnode, const int8_t *__restrict__ bins, long long S,
    const int8_t *__restrict__ bins_fm, long long NT,
    const int *__restrict__ feats, uint8_t *flags, int *tile_cnt, long long nloc) {
    pdl_wait();  // the previous kernel on the stream has completed
    // (split feature or -1, split bin) of the level's nodes, cached once per CTA
    constexpr int CACHE = 1024, IPT = PART_TILE / PART_THREADS;
    __shared__ int2 s_nd[CACHE];
    const int nnd = *nn_d;
    for (int i = threadIdx.x; i < min(nnd, CACHE); i += PART_THREADS) {
        const int fp = lvl[i].fpos;
        s_nd[i] = make_int2(fp >= 0 ? feats[fp] : -1, lvl[i].bin);
    }
    __syncthreads();
    const int nact = *nact_d;
    const long long t0 = (long long)blockIdx.x * PART_TILE;
    // positions t0 + tid + 256u: the loads of all IPT positions are issued
    // before any of them is used
    int nd[IPT], row[IPT];
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        const long long p = t0 + threadIdx.x + (long long)u * PART_THREADS;
        const bool ok = p < nact;
        nd[u] = ok ? (posnode ? posnode[p] : (int)(p / nloc)) : -1;  // level 0: tree t's root owns [tN, (t+1)N)
        row[u] = ok ? order[p] : 0;
    }
    int8_t bv[IPT];
    int2 sp[IPT];
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        sp[u] = make_int2(-1, 0);
        if (nd[u] >= 0) {
            if (nd[u] < CACHE) {
                sp[u] = s_nd[nd[u]];
            } else {
                const int fp = lvl[nd[u]].fpos;
                sp[u] = make_int2(fp >= 0 ? feats[fp] : -1, lvl[nd[u]].bin);
            }
        }
        bv[u] = 0;
        if (sp[u].x >= 0)
            bv[u] = bins_fm ? bins_fm[(long long)sp[u].x * NT + row[u]] : bins[(long long)row[u] * S + sp[u].x];
    }
    int cnt = 0;
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        if (nd[u] < 0) continue;
        const long long p = t0 + threadIdx.x + (long long)u * PART_THREADS;
        uint8_t fl = 2;
        if (sp[u].x >= 0) {
            fl = bv[u] <= sp[u].y ? 1 : 0;
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

// lefts before position p (p may equal nact)
// (flags are read as 32-bit words from the tile start, which is 2048-byte
// aligned; the flag buffer is padded by 16 bytes past the last position)
__device__ __forceinline__ int lefts_before(long long p, const uint8_t *flags, const int *tile_off,
                                            int lane) {
    const long long t = p / PART_TILE, a = t * PART_TILE;
    const int len = (int)(p - a);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(flags + a);
    int c = 0;
    for (int i = lane; 4 * i < len; i += 32) {
        uint32_t x = w[i];
        const int rem = len - 4 * i;
        if (rem < 4) x &= (1u << (8 * rem)) - 1u;     // bytes at or past p
        c += __popc(__vcmpeq4(x, 0x01010101u)) >> 3;  // bytes equal to 1 (left)
    }
    c = warp_sum(c);
    return tile_off[t] + c;
}

// Per splitting node: local left count and the start of its children in the
// next order; children's local segments; next level's active rows; then the
// next level's histogram chunk list.
__global__ void __launch_bounds__(1024) k_node_offsets(wgb_node *__restrict__ lvl, wgb_node *__restrict__ nxt,
                                                       const int *nn, int *nact, int d,
                                                       const uint8_t *flags, const int *tile_cnt,
                                                       int *tile_off, int ntiles, int4 *part, int4 *chunks,
                                                       int *nchunks, int chunk_cap, int wave) {
    pdl_wait();  // the previous kernel on the stream has completed
    __shared__ int s_scan[33];
    {   // exclusive scan of the tiles' left counts (tile_off[ntiles] = total)
        int base = 0;
        for (int b0 = 0; b0 < ntiles; b0 += 1024) {
            const int i = b0 + threadIdx.x;
            const int v = i < ntiles ? tile_cnt[i] : 0;
            int tot;
            const int ex = block_scan_excl(v, s_scan, tot);
            if (i < ntiles) tile_off[i] = base + ex;
            base += tot;
        }
        if (threadIdx.x == 0) tile_off[ntiles] = base;
        __syncthreads();
    }
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
    int base = 0;
    for (int b0 = 0; b0 < nnd; b0 += 1024) {
        int i = b0 + threadIdx.x;
        int v = (i < nnd && lvl[i].fpos >= 0) ? lvl[i].lcnt : 0;
        int tot;
        const int ex = block_scan_excl(v, s_scan, tot);
        if (v > 0 || (i < nnd && lvl[i].fpos >= 0)) {
            int ns = base + ex;
            int4 pr = part[i];
            pr.y = ns;
            part[i] = pr;
            int c = lvl[i].child;
            nxt[c].lstart = ns;
            nxt[c].lcnt = pr.z;
            nxt[c + 1].lstart = ns + pr.z;
            nxt[c + 1].lcnt = v - pr.z;
        }
        base += tot;
    }
    if (threadIdx.x == 0) nact[d + 1] = base;
    // the next level's histogram chunk list (chunks == NULL at the last level)
    if (chunks) {
        __syncthreads();
        plan_chunks(nxt, nn[d + 1], chunks, nchunks, chunk_cap, wave);
    }
}

// Scatter rows into the next level's order; finished rows get their leaf
// update pred += lr * leaf (core.py:598-621).  At the tree's last split
// level (`last` = the next level's records, all leaves) every row gets its
// leaf update instead of a place in the next order.
struct ScatterNode {
    float leaf;
    int lstart, child, px, py, pz;  // part[n]: lefts before the node, start of its children, left count
    int tree;                       // the node's tree in the batch (its output column is cls + tree)
};

__global__ void __launch_bounds__(PART_THREADS) k_scatter(
    const wgb_node *__restrict__ lvl, const int *nn_d, const int *nact_d, const int *__restrict__ order,
    const int *__restrict__ posnode, const uint8_t *__restrict__ flags,
    const int *__restrict__ tile_off, const int4 *__restrict__ part, int *__restrict__ order_next,
    int *__restrict__ posnode_next, float *__restrict__ pred, int K, int cls, float lr, long long npos,
    long long nloc, const wgb_node *__restrict__ last) {
    pdl_wait();  // the previous kernel on the stream has completed
    constexpr int IPT = PART_TILE / PART_THREADS;  // 8 consecutive positions per thread
    constexpr int CACHE = 512;                     // nodes whose records are cached per CTA
    __shared__ ScatterNode s_nc[CACHE];
    const int nnd = *nn_d;
    for (int i = threadIdx.x; i < min(nnd, CACHE); i += PART_THREADS) {
        const wgb_node &nd = lvl[i];
        const int4 pr = nd.fpos >= 0 ? part[i] : make_int4(0, 0, 0, 0);
        s_nc[i] = ScatterNode{nd.leaf, nd.lstart, nd.child, pr.x, pr.y, pr.z, node_tree(nd.built)};
    }
    const int nact = *nact_d;
    const long long p0 = (long long)blockIdx.x * PART_TILE + threadIdx.x * IPT;
    const bool full = p0 + IPT <= nact;
    uint8_t f[IPT];
    int nid[IPT], row[IPT];
    if (full) {  // p0 is a multiple of 8: 8-byte flag and 32-byte index loads
        const uint2 fw = *reinterpret_cast<const uint2 *>(flags + p0);
#pragma unroll
        for (int u = 0; u < IPT; ++u) f[u] = (uint8_t)(((u < 4 ? fw.x : fw.y) >> (8 * (u & 3))) & 0xFF);
        const int4 *o4 = reinterpret_cast<const int4 *>(order + p0);
        const int4 a = o4[0], b = o4[1];
        row[0] = a.x; row[1] = a.y; row[2] = a.z; row[3] = a.w;
        row[4] = b.x; row[5] = b.y; row[6] = b.z; row[7] = b.w;
        if (posnode) {
            const int4 *n4 = reinterpret_cast<const int4 *>(posnode + p0);
            const int4 c = n4[0], d = n4[1];
            nid[0] = c.x; nid[1] = c.y; nid[2] = c.z; nid[3] = c.w;
            nid[4] = d.x; nid[5] = d.y; nid[6] = d.z; nid[7] = d.w;
        } else {
#pragma unroll
            for (int u = 0; u < IPT; ++u) nid[u] = (int)((p0 + u) / nloc);
        }
    } else {
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
            const bool ok = p0 + u < nact;
            f[u] = ok ? flags[p0 + u] : 3;
            row[u] = ok ? order[p0 + u] : 0;
            nid[u] = !ok ? 0 : (posnode ? posnode[p0 + u] : (int)((p0 + u) / nloc));
        }
    }
    int c = 0;
#pragma unroll
    for (int u = 0; u < IPT; ++u) c += f[u] == 1;
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
    __syncthreads();  // also publishes the node cache
    int wbase = 0;
    for (int w = 0; w < warp; ++w) wbase += sw[w];
    int lp = tile_off[blockIdx.x] + wbase + incl - c;
    if (last) {
        // every row's leaf update (the children are the tree's last level);
        // the rows are distinct, so all prediction loads go before any store
        float lv[IPT], pv[IPT];
        long long at[IPT];
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
            at[u] = -1;
            lv[u] = 0.0f;
            if (f[u] == 3) continue;
            const int n = nid[u];
            ScatterNode nd;
            if (n < CACHE) {
                nd = s_nc[n];
            } else {
                const wgb_node &g = lvl[n];
                nd = ScatterNode{g.leaf, g.lstart, g.child, 0, 0, 0, node_tree(g.built)};
            }
            lv[u] = f[u] == 2 ? nd.leaf : last[nd.child + (f[u] == 1 ? 0 : 1)].leaf;
            at[u] = (long long)row[u] * K + cls + nd.tree;
        }
#pragma unroll
        for (int u = 0; u < IPT; ++u) pv[u] = at[u] >= 0 ? pred[at[u]] : 0.0f;
#pragma unroll
        for (int u = 0; u < IPT; ++u)
            if (at[u] >= 0) pred[at[u]] = __fadd_rn(pv[u], __fmul_rn(lr, lv[u]));
        return;
    }
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        if (f[u] == 3) break;
        const long long p = p0 + u;
        const int n = nid[u];
        ScatterNode nd;
        if (n < CACHE) {
            nd = s_nc[n];
        } else {
            const wgb_node &g = lvl[n];
            const int4 pr = g.fpos >= 0 ? part[n] : make_int4(0, 0, 0, 0);
            nd = ScatterNode{g.leaf, g.lstart, g.child, pr.x, pr.y, pr.z, node_tree(g.built)};
        }
        if (f[u] == 2) {
            float *pp = pred + (long long)row[u] * K + cls + nd.tree;
            *pp = __fadd_rn(*pp, __fmul_rn(lr, nd.leaf));
        } else {
            const int lb = lp - nd.px;  // lefts before p inside the node
            int np, child;
            if (f[u] == 1) {
                np = nd.py + lb;
                child = nd.child;
            } else {
                np = nd.py + nd.pz + (int)(p - nd.lstart) - lb;
                child = nd.child + 1;
            }
            if (np >= 0 && np < npos) {  // always true for consistent offsets; guards memory
                order_next[np] = row[u];
                posnode_next[np] = child;
            }
            if (f[u] == 1) ++lp;
        }
    }
}

// One-era level partition in one launch.  plan_children has given each
// splitting node n its children's range [ns, ns + lcnt) of the next order
// (part[n] = {left cursor 0, ns, -, right cursor 0}).  Each CTA takes
// PART_TILE consecutive positions, computes their flags (k_flags' rule),
// ranks its rows per (node, side) with shared atomics, reserves each (node,
// side) range with one global atomic on the node's cursor, and writes left
// rows upward from ns and right rows downward from ns + lcnt - 1, so the
// left count need not be known in advance.  Within a child the rows are not
// in their previous relative order: nothing depends on it with one era (the
// histograms are exact integer sums; era windows, which need era-sorted
// rows, take the stable three-kernel partition).  Multi-rank fits (finish):
// the last CTA to finish, counted in `done` (zero-initialised, returned to
// zero), lays out the next level from the final left cursors
// (finish_children).  At the tree's last level (`last`) every row only gets
// its leaf update.
__global__ void __launch_bounds__(PART_THREADS) k_partition(
    const wgb_node *__restrict__ lvl, const int *nn_d, const int *nact_d, const int *__restrict__ order,
    const int *__restrict__ posnode, const int8_t *__restrict__ bins, long long S,
    const int8_t *__restrict__ bins_fm, long long NT, const int *__restrict__ feats, int4 *part,
    int *__restrict__ order_next, int *__restrict__ posnode_next, float *__restrict__ pred, int K, int cls,
    float lr, long long npos, long long nloc, const wgb_node *__restrict__ last, bool finish, wgb_node *nxt,
    int *nn, int *nact_all, int d, int *done, int4 *chunks, int *nchunks, int chunk_cap, int wave) {
    pdl_wait();  // the previous kernel on the stream has completed
    constexpr int IPT = PART_TILE / PART_THREADS;  // 8 consecutive positions per thread
    constexpr int CACHE = 512;                     // nodes whose records are cached per CTA
    struct PNode {
        float leaf;
        int child, ns, cnt;   // children's range [ns, ns + cnt) of the next order
        int tree, feat, bin;  // feat: split feature, -1 leaf
    };
    __shared__ PNode s_nc[CACHE];
    __shared__ int s_key[2 * PART_TILE];  // per (node - first node, side): local count, then range start
    __shared__ int s_first, s_lastn;
    const int nnd = *nn_d;
    auto node_rec = [&](int i) {
        const wgb_node &nd = lvl[i];
        const int fp = nd.fpos;
        const int4 pr = fp >= 0 ? part[i] : make_int4(0, 0, 0, 0);
        return PNode{nd.leaf, nd.child, pr.y, nd.lcnt, node_tree(nd.built), fp >= 0 ? feats[fp] : -1, nd.bin};
    };
    auto rec = [&](int n) { return n < CACHE ? s_nc[n] : node_rec(n); };
    for (int i = threadIdx.x; i < min(nnd, CACHE); i += PART_THREADS) s_nc[i] = node_rec(i);
    if (!last)
        for (int i = threadIdx.x; i < 2 * PART_TILE; i += PART_THREADS) s_key[i] = 0;
    if (threadIdx.x == 0) {
        s_first = INT_MAX;
        s_lastn = -1;
    }
    const int nact = *nact_d;
    const long long p0 = (long long)blockIdx.x * PART_TILE + threadIdx.x * IPT;
    int nid[IPT], row[IPT];
    if (p0 + IPT <= nact) {  // p0 is a multiple of 8: 32-byte index loads
        const int4 *o4 = reinterpret_cast<const int4 *>(order + p0);
        const int4 a = o4[0], b = o4[1];
        row[0] = a.x; row[1] = a.y; row[2] = a.z; row[3] = a.w;
        row[4] = b.x; row[5] = b.y; row[6] = b.z; row[7] = b.w;
        if (posnode) {
            const int4 *n4 = reinterpret_cast<const int4 *>(posnode + p0);
            const int4 c4 = n4[0], d4 = n4[1];
            nid[0] = c4.x; nid[1] = c4.y; nid[2] = c4.z; nid[3] = c4.w;
            nid[4] = d4.x; nid[5] = d4.y; nid[6] = d4.z; nid[7] = d4.w;
        } else {
#pragma unroll
            for (int u = 0; u < IPT; ++u) nid[u] = (int)((p0 + u) / nloc);  // level 0: tree t owns [tN, (t+1)N)
        }
    } else {
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
            const bool ok = p0 + u < nact;
            row[u] = ok ? order[p0 + u] : 0;
            nid[u] = !ok ? -1 : (posnode ? posnode[p0 + u] : (int)((p0 + u) / nloc));
        }
    }
    __syncthreads();  // node cache, zeroed counters
    // flags: 1 left, 0 right, 2 the node is a leaf, 3 no position
    uint32_t fb = 0;  // 2 bits per position
    int nmin = INT_MAX, nmax = -1;
#pragma unroll
    for (int u = 0; u < IPT; ++u) {
        if ((unsigned)nid[u] >= (unsigned)nnd || (unsigned long long)(unsigned)row[u] >= (unsigned long long)nloc)
            nid[u] = -1;  // out of range: treated as no position (guards memory)
        uint32_t fu = 3u;
        if (nid[u] >= 0) {
            int feat, bin;
            if (nid[u] < CACHE) {
                feat = s_nc[nid[u]].feat;
                bin = s_nc[nid[u]].bin;
            } else {
                const PNode r = node_rec(nid[u]);
                feat = r.feat;
                bin = r.bin;
            }
            fu = 2u;
            if (feat >= 0) {
                const int8_t bv = bins_fm ? bins_fm[(long long)feat * NT + row[u]] : bins[(long long)row[u] * S + feat];
                fu = bv <= bin ? 1u : 0u;
                nmin = min(nmin, nid[u]);
                nmax = max(nmax, nid[u]);
            }
        }
        fb |= fu << (2 * u);
    }
    if (!last) {
        // the splitting nodes of the tile (positions are in node order)
        if (nmax >= 0) {
            atomicMin(&s_first, nmin);
            atomicMax(&s_lastn, nmax);
        }
        __syncthreads();
        const int first = s_first;
        const bool local = s_lastn - first < PART_TILE;  // else per-row global atomics (sparse node ids)
        int rank[IPT];
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
            const uint32_t fu = (fb >> (2 * u)) & 3u;
            rank[u] = 0;
            if (local && fu <= 1u) rank[u] = atomicAdd(&s_key[2 * (nid[u] - first) + (fu == 1u ? 0 : 1)], 1);
        }
        __syncthreads();
        if (local) {
            const int nk = s_lastn >= first ? 2 * (s_lastn - first + 1) : 0;
            for (int key = threadIdx.x; key < nk; key += PART_THREADS) {
                const int cnt = s_key[key];
                if (cnt > 0) {
                    int4 *pr = part + first + (key >> 1);
                    s_key[key] = atomicAdd((key & 1) ? &pr->w : &pr->x, cnt);
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
            const uint32_t fu = (fb >> (2 * u)) & 3u;
            if (fu == 3u) continue;
            const PNode nd = rec(nid[u]);
            if (fu == 2u) {
                float *pp = pred + (long long)row[u] * K + cls + nd.tree;
                *pp = __fadd_rn(*pp, __fmul_rn(lr, nd.leaf));
                continue;
            }
            const int side = fu == 1u ? 0 : 1;
            int r;
            if (local) {
                r = s_key[2 * (nid[u] - first) + side] + rank[u];
            } else {
                int4 *pr = part + nid[u];
                r = atomicAdd(side ? &pr->w : &pr->x, 1);
            }
            const long long np = side ? (long long)nd.ns + nd.cnt - 1 - r : (long long)nd.ns + r;
            if (np >= 0 && np < npos) {  // always true for consistent counts; guards memory
                order_next[np] = row[u];
                posnode_next[np] = nd.child + side;
            }
        }
        if (finish) {
            __shared__ int s_scan[33];
            __shared__ bool s_last;
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence();  // this CTA's cursor reservations precede its count
                s_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
            }
            __syncthreads();
            if (!s_last) return;
            __threadfence();
            finish_children(lvl, nxt, nn, nact_all, d, part, chunks, nchunks, chunk_cap, wave, s_scan);
            if (threadIdx.x == 0) *done = 0;
        }
    } else {
        // every row's leaf update; the rows are distinct, so all eight
        // prediction loads are issued before any store
        float lv[IPT], pv[IPT];
        long long at[IPT];
#pragma unroll
        for (int u = 0; u < IPT; ++u) {
            const uint32_t fu = (fb >> (2 * u)) & 3u;
            at[u] = -1;
            lv[u] = 0.0f;
            if (fu != 3u) {
                const PNode nd = rec(nid[u]);
                lv[u] = fu == 2u ? nd.leaf : last[nd.child + (fu == 1u ? 0 : 1)].leaf;
                at[u] = (long long)row[u] * K + cls + nd.tree;
            }
        }
#pragma unroll
        for (int u = 0; u < IPT; ++u) pv[u] = at[u] >= 0 ? pred[at[u]] : 0.0f;
#pragma unroll
        for (int u = 0; u < IPT; ++u)
            if (at[u] >= 0) pred[at[u]] = __fadd_rn(pv[u], __fmul_rn(lr, lv[u]));
    }
}

// The tree's feature subset as its own bin matrix: out[r][j] = bins[r][feats[j]]
// (j < k; padding bytes 0) and kpos_out[j] = j (-1 past k).  A block takes 16
// rows; the row bytes it gathers sit in L1, the writes are whole rows.
__global__ void __launch_bounds__(256) k_bins_subset(const int8_t *__restrict__ bins, long long N, long long S,
                                                     const int *__restrict__ feats, int k, int8_t *__restrict__ out,
                                                     long long So, int *__restrict__ kpos_out) {
    pdl_wait();  // the previous kernel on the stream has completed
    extern __shared__ int s_feat[];
    for (int j = threadIdx.x; j < So; j += blockDim.x) {
        s_feat[j] = j < k ? feats[j] : -1;
        if (blockIdx.x == 0) kpos_out[j] = j < k ? j : -1;
    }
    __syncthreads();
    const long long r0 = (long long)blockIdx.x * 16;
    const int words = (int)(So / 4);
    for (int t = threadIdx.x; t < 16 * words; t += blockDim.x) {
        const long long r = r0 + t / words;
        if (r >= N) break;
        const int j0 = (t % words) * 4;
        const int8_t *src = bins + r * S;
        uint32_t w = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int f = s_feat[j0 + u];
            if (f >= 0) w |= (uint32_t)(uint8_t)__ldg(src + f) << (8 * u);
        }
        *reinterpret_cast<uint32_t *>(out + r * So + j0) = w;
    }
}

// ====================================================================== //
// host side                                                              //
// ====================================================================== //

static inline long long *LL(int64_t *p) { return reinterpret_cast<long long *>(p); }
// trees grown together (a multiclass round: one per class); levels hold
// ntree << d node records
static inline int ws_ntree(const wgb_ws *ws) { return ws->ntree > 1 ? ws->ntree : 1; }
// One-era fits partition each level in one launch (k_partition).  On a
// single rank (the local rows are all rows) the split's exact left counts
// are the local ones, so the split plans the next level's row layout; on
// several ranks the partition's last CTA finishes it from the rows it moved.
static inline bool fused_partition(const wgb_ws *ws) { return ws->E == 1 && ws->sync != nullptr; }
static inline bool single_rank(const wgb_ws *ws) { return ws->N_global == ws->N && ws->nslice <= 1; }
static inline wgb_node *level_nodes(const wgb_ws *ws, int d) {
    return ws->nodes + (long long)ws_ntree(ws) * ((1 << d) - 1);
}
static inline const int *level_order(const wgb_ws *ws, int d) {
    return d == 0 ? ws->root_order : ws->order[(d - 1) & 1];
}
static inline const int *level_posnode(const wgb_ws *ws, int d) {
    return d == 0 ? nullptr : ws->posnode[(d - 1) & 1];
}
// Feature-sliced multi-rank fit: rank `slice` keeps and searches positions
// [slice*ks, slice*ks + ks) of the tree's k (the last slices may be short
// or empty).
static inline bool sliced(const wgb_ws *ws) { return ws->nslice > 1; }
// The histogram's matrix: the tree's own feature matrix when there is one
// (k columns in position order), else the full bin matrix.
static inline long long hist_S(const wgb_ws *ws) { return ws->bins_sub ? ws->S_sub : ws->S; }
static inline int hist_F(const wgb_ws *ws) { return ws->bins_sub ? ws->k : ws->F; }
// One-era levels: the chunks that one wave of the histogram kernel's
// resident CTAs builds at once over all feature tiles -- the chunk planner
// sizes the level's chunks to fill whole waves -- or 0 (era levels: chunks
// of HIST_R rows).
static int hist_wave(const wgb_ws *ws) {
    if (ws->E != 1) return 0;
    int fpl, nsc;
    hist_shape(hist_S(ws), hist_F(ws), ws->B, fpl, nsc);
    const int minb = (fpl == 8 && nsc <= 34) ? 2 : 1;  // CTAs per SM of the one-era instantiations
    const int ntile = (hist_F(ws) + 32 * fpl - 1) / (32 * fpl);
    const int w = minb * num_sms() / (ntile > 0 ? ntile : 1);
    return w > 0 ? w : 1;
}
static inline int hist_k(const wgb_ws *ws) { return sliced(ws) ? ws->ks : ws->k; }  // the pool's k
static inline int slice_j0(const wgb_ws *ws) { return sliced(ws) ? ws->slice * ws->ks : 0; }
static inline int slice_kr(const wgb_ws *ws) {
    if (!sliced(ws)) return ws->k;
    const int r = ws->k - slice_j0(ws);
    return r < 0 ? 0 : (r < ws->ks ? r : ws->ks);
}
// Histogram pool: one int64 region per slot, [sums E*k*(B+1)][counts E*k*(B+1)][2 spare]
// (ks in place of k when sliced); root slot t's first spare cell carries
// tree t's root sum of q through the level-0 reduction, so one collective
// per level covers sums, counts and roots.
static inline long long hist_cells(const wgb_ws *ws) { return (long long)ws->E * hist_k(ws) * (ws->B + 1); }
static inline long long slot_elems(const wgb_ws *ws) { return 2 * hist_cells(ws) + 2; }

static int grid_for(long long n, int threads, int cap = 148 * 16) {
    long long b = (n + threads - 1) / threads;
    if (b < 1) b = 1;
    return (int)(b < cap ? b : cap);
}



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

void wgb_level_slots(const wgb_ws *ws, int32_t d, int32_t *first, int32_t *count) {
    wgb_built_slots(d, first, count);
    const int nt = ws ? ws_ntree(ws) : 1;
    *first *= nt;
    *count *= nt;
}

int64_t wgb_era_mean_plan(int32_t E, int64_t M, int32_t num_sms, int32_t max_threads_per_sm,
                          int32_t *sched, uint8_t *ops, int64_t ops_cap, int32_t *depth) {
    if (E < 1 || M < 1) {
        set_error("E and M must be >= 1");
        return -WGB_ERR_ARG;
    }
    if (num_sms <= 0 || max_threads_per_sm <= 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&max_threads_per_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev) != cudaSuccess) {
            set_error("no device to take the SM count from; pass num_sms and max_threads_per_sm");
            return -WGB_ERR_CUDA;
        }
    }
    EraPlanWriter w{sched, ops, ops ? ops_cap : 0};
    if (M == 1) {
        // a single output is reduced along another path of torch (contiguous
        // eras, vectorised loads, warp shuffles) that is not restated here:
        // sequential sum (only the test crit > min_split_gain reads it)
        w.op(ERA_PUSH0);
        for (int e = 0; e < E; ++e) w.era(e);
    } else {
        int rows, ctas;
        era_mean_layout(E, M, num_sms, max_threads_per_sm, rows, ctas);
        era_plan(w, E, rows, ctas);
    }
    if (depth) *depth = w.depth;
    return w.n;
}

static int check_ws(const wgb_ws *ws) {
    WGB_CHECK_ARG(ws != nullptr, "workspace is NULL");
    WGB_CHECK_ARG(ws->B >= 2 && ws->B <= 127, "num_bins must be in [2, 127], got %d", ws->B);
    WGB_CHECK_ARG(ws->D >= 1 && ws->D <= 24, "max_depth must be in [1, 24], got %d", ws->D);
    WGB_CHECK_ARG(ws->k >= 1 && ws->k <= ws->F, "k must be in [1, F]");
    WGB_CHECK_ARG(ws->E >= 1, "num_eras must be >= 1");
    WGB_CHECK_ARG(ws->N >= 0 && ws->N < (1ll << 31), "rows per rank must be < 2^31");
    WGB_CHECK_ARG(ws->S >= ws->F && ws->S % 4 == 0, "bins row stride must be >= F and a multiple of 4");
    WGB_CHECK_ARG(ws->hist_ew >= 0, "hist_ew must be >= 0");
    WGB_CHECK_ARG(ws->ntree >= 0 && ws->cls >= 0 && ws->cls + ws_ntree(ws) <= ws->K,
                  "trees cls .. cls + ntree - 1 must be output columns (< K)");
    WGB_CHECK_ARG((long long)ws_ntree(ws) * ws->N < (1ll << 31), "ntree * rows per rank must be < 2^31");
    if (sliced(ws)) {
        WGB_CHECK_ARG(ws->slice >= 0 && ws->slice < ws->nslice, "slice %d of %d", ws->slice, ws->nslice);
        WGB_CHECK_ARG(ws->ks >= 1 && (long long)ws->ks * ws->nslice >= ws->k, "ks * nslice must cover k");
        WGB_CHECK_ARG(ws->hstage != nullptr && ws->win != nullptr && ws->win_words >= 8 + ws->E &&
                          ws->win_words % 2 == 0 && (reinterpret_cast<uintptr_t>(ws->win) & 7) == 0,
                      "a sliced fit needs hstage and an 8-byte aligned win of even win_words >= 8 + E");
    }
    return WGB_OK;
}

int wgb_tree_reset(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_PDL("k_reset", k_reset, dim3(1), dim3(32), 0, as_stream(stream), ws->maxabs, LL(ws->rootsum),
            ws_ntree(ws));
    return WGB_OK;
}

int wgb_tree_residual(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    if (ws->N == 0) return WGB_OK;
    const dim3 grid((unsigned)grid_for(ws->N, 256, 148 * 16 / ws_ntree(ws) + 1), (unsigned)ws_ntree(ws));
    WGB_PDL("k_residual", k_residual, grid, dim3(256), 0, as_stream(stream), ws->y, ws->pred, ws->K, ws->cls, ws->g,
            ws->N, ws->maxabs);
    return WGB_OK;
}

int wgb_tree_quantize(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    const dim3 grid((unsigned)grid_for(ws->N, 256, 148 * 16 / ws_ntree(ws) + 1), (unsigned)ws_ntree(ws));
    WGB_PDL("k_quantize", k_quantize, grid, dim3(256), 0, as_stream(stream), ws->g, ws->qg, ws->N, ws->maxabs,
            ws->shift, LL(ws->rootsum));
    return WGB_OK;
}

int wgb_tree_subset(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    if (!ws->bins_sub) return WGB_OK;
    WGB_CHECK_ARG(ws->kpos_sub && ws->S_sub >= ws->k && ws->S_sub % 32 == 0, "bins_sub needs kpos_sub and a stride "
                  "S_sub >= k, a multiple of 32");
    if (ws->N == 0) return WGB_OK;
    const size_t sm = (size_t)ws->S_sub * sizeof(int);
    WGB_CUDA(cudaFuncSetAttribute(k_bins_subset, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    WGB_PDL("k_bins_subset", k_bins_subset, dim3((unsigned)((ws->N + 15) / 16)), dim3(256), sm, as_stream(stream),
            ws->bins, ws->N, ws->S, ws->feats, ws->k, ws->bins_sub, ws->S_sub, ws->kpos_sub);
    return WGB_OK;
}

int wgb_tree_root(const wgb_ws *ws, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_PDL("k_root", k_root, dim3(1), dim3(32), 0, as_stream(stream), ws->nodes, ws->nn, ws->nact, ws->D, ws->N,
            ws->N_global, ws_ntree(ws));
    return WGB_OK;
}

int64_t wgb_hist_part_elems(int64_t S, int32_t F, int32_t B, int64_t chunks) {
    int fpl, nsc;
    hist_shape(S, F, B, fpl, nsc);
    const long long ft = 32ll * fpl;
    return chunks * ((F + ft - 1) / ft) * nsc * ft;
}

int wgb_level_hist(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    cudaStream_t st = as_stream(stream);
    int first, count;
    wgb_level_slots(ws, d, &first, &count);
    const long long se = slot_elems(ws), nc = hist_cells(ws);
    // where the build adds its cells: the built slots of the pool, or (a
    // sliced fit) the staging buffer, one region of `count` slots per slice,
    // which the reduce-scatter over the ranks turns into those slots of each
    // rank's pool
    HistOut out;
    if (sliced(ws)) {
        const long long region = (long long)count * se;
        WGB_CHECK_ARG(region * ws->nslice <= ws->hstage_elems, "hstage holds %lld elements, level %d needs %lld",
                      (long long)ws->hstage_elems, d, region * ws->nslice);
        WGB_PDL("k_zero", k_zero, dim3(zero_grid(region * ws->nslice)), dim3(256), 0, st, LL(ws->hstage),
                region * ws->nslice);
        if (d == 0) {  // this rank's root sums ride along with the level-0 reduction
            WGB_PDL("k_root_cells", k_root_cells, dim3(1), dim3(32), 0, st, LL(ws->hstage), LL(ws->rootsum), se, nc,
                    ws_ntree(ws), ws->nslice, region);
        }
        out = HistOut{LL(ws->hstage), LL(ws->hstage) + nc, se, region, ws->ks, first};
    } else {
        WGB_PDL("k_zero", k_zero, dim3(zero_grid(se * count)), dim3(256), 0, st, LL(ws->hg) + (long long)first * se,
                se * count);
        if (d == 0) {
            WGB_PDL("k_root_cells", k_root_cells, dim3(1), dim3(32), 0, st, LL(ws->hg), LL(ws->rootsum), se, nc,
                    ws_ntree(ws), 1, 0ll);
        }
        out = HistOut{LL(ws->hg), LL(ws->hg) + nc, se, 0, ws->k, 0};
    }
    wgb_node *lvl = level_nodes(ws, d);
    if (d == 0) {  // later levels' chunk lists are planned by the previous level's partition
        WGB_PDL("k_chunk_plan", k_chunk_plan, dim3(1), dim3(1024), 0, st, lvl, ws->nn + d,
                reinterpret_cast<int4 *>(ws->chunks), ws->nchunks, ws->chunk_cap, hist_wave(ws));
    }
    if (ws->N == 0) return WGB_OK;
    // most chunks the level can have: pieces of at least HIST_R rows, or of
    // HIST_R / 2 where the planner balances the chunk size
    const int rmin = hist_wave(ws) > 0 ? HIST_R / 2 : HIST_R;
    long long max_chunks = ((long long)ws_ntree(ws) * ws->N + rmin - 1) / rmin + count;
    if (max_chunks > ws->chunk_cap) max_chunks = ws->chunk_cap;
    const int *ord = level_order(ws, d);
    const bool sub = ws->bins_sub != nullptr;
    const int8_t *hb = sub ? ws->bins_sub : ws->bins;
    const long long hS = hist_S(ws);
    const int hF = hist_F(ws);
    const int *hkpos = sub ? ws->kpos_sub : ws->kpos;
    cudaError_t e = launch_hist((int)max_chunks, hb, hS, hF, ord, ws->qg, nullptr, nullptr,
                                ws->E > 1 ? ws->era : nullptr, hkpos, ws->k, ws->E, ws->B, ws->hist_ew,
                                ws->regular != 0, reinterpret_cast<const int4 *>(ws->chunks), ws->nchunks,
                                lvl, out, ws->N, st,
                                ws->E == 1 && ws->part_hist &&
                                        ws->part_hist_elems >= wgb_hist_part_elems(hS, hF, ws->B, max_chunks)
                                    ? reinterpret_cast<uint2 *>(ws->part_hist)
                                    : nullptr);
    if (e != cudaSuccess) {
        set_error("k_hist launch failed: %s", cudaGetErrorString(e));
        return WGB_ERR_CUDA;
    }

    return WGB_OK;
}

int wgb_level_split(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    cudaStream_t st = as_stream(stream);
    const long long se = slot_elems(ws), nc = hist_cells(ws);
    long long *hg = LL(ws->hg), *hc = hg + nc;
    wgb_node *lvl = level_nodes(ws, d);
    const int cap = ws_ntree(ws) << d;
    if (d == 0) {
        WGB_PDL("k_root_total", k_root_total, dim3(1), dim3(32), 0, st, ws->nodes, hg, se, nc, ws->shift,
                ws_ntree(ws));
    }
    // (from level 1 on, the split kernels first turn each unbuilt node's
    // parent histogram into parent - built sibling)
    const int nb = ws->B - 1;
    // this rank's positions (all k unless the fit is feature-sliced)
    const int j0 = slice_j0(ws), kr = slice_kr(ws), kl = hist_k(ws);
    int4 *cand = reinterpret_cast<int4 *>(ws->cand);
    int nblk;
    if (ws->E == 1) {
        nblk = (kr + SPLIT_WARPS - 1) / SPLIT_WARPS;
        WGB_CHECK_ARG(nblk <= ws->ncand_blk, "candidate buffer too small: %d blocks per node needed", nblk);
        const unsigned g = (unsigned)nblk * (unsigned)cap;  // node-major blocks
#define WGB_SPLIT_W(NBW_)                                                                                  \
    WGB_PDL("k_split", k_split<NBW_>, dim3(g), dim3(SPLIT_WARPS * 32), 0, st, lvl, ws->nn + d, hg, hc, se, kr, \
            j0, ws->B, ws->shift, ws->mcw, ws->eps, ws->msg, cand, nblk, ws->crit_out, d < ws->D - 1)
        if (g > 0) {
            if (nb <= 32) WGB_SPLIT_W(1); else if (nb <= 64) WGB_SPLIT_W(2); else WGB_SPLIT_W(4);
        }
#undef WGB_SPLIT_W
    } else {
        WGB_CHECK_ARG(ws->era_sched && ws->era_ops && ws->era_nops >= ws->E && ws->era_depth >= 1,
                      "levels with eras need the criterion plan of wgb_era_mean_plan in the workspace");
        const int fb = split_era_fb(ws->B);
        nblk = (kr + fb - 1) / fb;
        WGB_CHECK_ARG(nblk <= ws->ncand_blk, "candidate buffer too small: %d blocks per node needed", nblk);
        const unsigned g = (unsigned)nblk * (unsigned)cap;
        int dev = 0, smem_max = 0;
        WGB_CUDA(cudaGetDevice(&dev));
        WGB_CUDA(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
#define WGB_SPLIT_ERAS(NB_)                                                                                    \
    {                                                                                                          \
        const size_t sm = split_eras_smem(ws->B, NB_, EraSplitShape<NB_>::FB, ws->era_depth);                  \
        WGB_CHECK_ARG(sm <= (size_t)smem_max, "era criterion plan too deep (%d) for shared memory", ws->era_depth); \
        WGB_CUDA(cudaFuncSetAttribute(k_split_eras<NB_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm)); \
        WGB_PDL("k_split_eras", k_split_eras<NB_>, dim3(g), dim3(256), sm, st, lvl, ws->nn + d, hg, hc, se, kr, \
                kl, j0, ws->E, ws->B, ws->shift, ws->mcw, ws->eps, ws->msg, ws->mean_factor, ws->era_sched,    \
                ws->era_ops, ws->era_nops, ws->era_depth, cand, nblk, ws->crit_out, d < ws->D - 1);            \
    }
        if (g > 0) {
            if (nb <= 8) WGB_SPLIT_ERAS(8) else if (nb <= 32) WGB_SPLIT_ERAS(32) else WGB_SPLIT_ERAS(128)
        }
#undef WGB_SPLIT_ERAS
    }
    float *eg = ws->era_gain + (long long)ws_ntree(ws) * ((1 << d) - 1) * ws->E;
    WGB_CHECK_ARG(ws->sync != nullptr, "workspace needs its sync counters");
    const bool fp = fused_partition(ws), one = single_rank(ws);
    WGB_PDL("k_split_final", k_split_final, dim3(cap), dim3(256), 0, st, lvl, level_nodes(ws, d + 1), ws->nn, d,
            ws_ntree(ws), hg, hc, se, kl, j0, ws->E, ws->B, ws->shift, ws->mcw, ws->eps, cand, nblk, eg, ws->sync,
            d < ws->D - 1, fp ? reinterpret_cast<int4 *>(ws->part) : nullptr, ws->nact,
            fp && one && d < ws->D - 1 ? reinterpret_cast<int4 *>(ws->chunks) : nullptr, ws->nchunks, ws->chunk_cap,
            sliced(ws) ? ws->win : nullptr, ws->win_words, ws->slice, hist_wave(ws), one);
    return WGB_OK;
}

int wgb_level_pick(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    if (!sliced(ws)) return WGB_OK;  // wgb_level_split already decided
    const int cap = ws_ntree(ws) << d;
    float *eg = ws->era_gain + (long long)ws_ntree(ws) * ((1 << d) - 1) * ws->E;
    WGB_PDL("k_split_pick", k_split_pick, dim3(cap), dim3(256), 0, as_stream(stream), level_nodes(ws, d),
            level_nodes(ws, d + 1), ws->nn, d, ws_ntree(ws), ws->B, ws->E, ws->shift, ws->win, ws->win_words,
            ws->nslice, eg, ws->sync, fused_partition(ws) ? reinterpret_cast<int4 *>(ws->part) : nullptr);
    return WGB_OK;
}

int wgb_bins_feature_major(const wgb_ws *ws, int8_t *out, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(out != nullptr && (reinterpret_cast<uintptr_t>(out) & 15) == 0,
                  "out must be a 16-byte aligned buffer of F * NT bytes");
    WGB_CHECK_ARG(ws->S % 16 == 0, "bins row stride must be a multiple of 16");
    if (ws->N == 0) return WGB_OK;
    const long long NT = (ws->N + 15) & ~15ll;
    dim3 g((unsigned)((NT + 127) / 128), (unsigned)((ws->F + 127) / 128));
    k_bins_fm<<<g, 256, 0, as_stream(stream)>>>(ws->bins, ws->N, ws->S, ws->F, NT, out);
    WGB_LAUNCHED("k_bins_fm");
    return WGB_OK;
}

int wgb_level_partition(const wgb_ws *ws, int32_t d, void *stream) {
    int rc = check_ws(ws);
    if (rc) return rc;
    WGB_CHECK_ARG(d >= 0 && d < ws->D, "level %d out of range", d);
    if (ws->N == 0) return WGB_OK;
    cudaStream_t st = as_stream(stream);
    wgb_node *lvl = level_nodes(ws, d);
    const long long npos = (long long)ws_ntree(ws) * ws->N;  // positions: tree t's rows at level 0 are [tN, (t+1)N)
    const int ntiles = (int)((npos + PART_TILE - 1) / PART_TILE);
    WGB_CHECK_ARG(ntiles <= ws->ntiles, "tile buffer too small");
    const int *ord = level_order(ws, d);
    const int *pn = level_posnode(ws, d);
    const bool last = d == ws->D - 1;
    int4 *part = reinterpret_cast<int4 *>(ws->part);
    if (fused_partition(ws)) {
        // several ranks: the last CTA lays out the next level (sync[1] counts the CTAs)
        const bool finish = !single_rank(ws) && !last;
        WGB_PDL("k_partition", k_partition, dim3(ntiles), dim3(PART_THREADS), 0, st, lvl, ws->nn + d,
                ws->nact + d, ord, pn, ws->bins, ws->S, ws->bins_fm, (ws->N + 15) & ~15ll, ws->feats, part,
                ws->order[d & 1], ws->posnode[d & 1], ws->pred, ws->K, ws->cls, ws->lr, npos, ws->N,
                last ? level_nodes(ws, d + 1) : nullptr, finish, level_nodes(ws, d + 1), ws->nn, ws->nact, d,
                ws->sync + 1, reinterpret_cast<int4 *>(ws->chunks), ws->nchunks, ws->chunk_cap, hist_wave(ws));
        return WGB_OK;
    }
    WGB_PDL("k_flags", k_flags, dim3(ntiles), dim3(PART_THREADS), 0, st, lvl, ws->nn + d, ws->nact + d, ord, pn,
            ws->bins, ws->S, ws->bins_fm, (ws->N + 15) & ~15ll, ws->feats, ws->flags, ws->tile_cnt, ws->N);
    WGB_PDL("k_node_offsets", k_node_offsets, dim3(1), dim3(1024), 0, st, lvl, level_nodes(ws, d + 1), ws->nn,
            ws->nact, d, ws->flags, ws->tile_cnt, ws->tile_off, ntiles, part,
            last ? nullptr : reinterpret_cast<int4 *>(ws->chunks), ws->nchunks, ws->chunk_cap, hist_wave(ws));
    WGB_PDL("k_scatter", k_scatter, dim3(ntiles), dim3(PART_THREADS), 0, st, lvl, ws->nn + d, ws->nact + d, ord, pn,
            ws->flags, ws->tile_off, part, ws->order[d & 1], ws->posnode[d & 1], ws->pred, ws->K, ws->cls, ws->lr,
            npos, ws->N, last ? level_nodes(ws, d + 1) : nullptr);
    return WGB_OK;
}

int wgb_tree_finish(const wgb_ws *ws, void *stream) {
    // the last level's leaf updates happen in wgb_level_partition(D - 1)
    (void)stream;
    return check_ws(ws);
}

}  // extern "C"
