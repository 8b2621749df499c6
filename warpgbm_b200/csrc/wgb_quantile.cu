// Exact quantile edges of every feature column (sm_100a), replacing the
// per-column torch.quantile(X[:, f], linspace(0, 1, B+1)[1:-1]) of the
// reference's preprocess_gpu_data (warpgbm/core.py:527-538).
//
// torch.quantile (linear) sorts the column, takes rank = q * (n - 1) in fp32,
// below = trunc(rank), above = ceil(rank), w = rank - below and returns
// lerp(sorted[below], sorted[above], w); any NaN in the column sets every
// rank to n - 1 (the NaN), so all edges are NaN.  Only the 2 (B - 1) order
// statistics are needed, so instead of a sort each column does a radix
// select: four passes over the column, one digit of the
// order-preserving key per pass, histogramming only elements whose higher
// digits match a still-active target prefix.  Keys order exactly like the
// radix sort torch uses (-0.0 before +0.0), so the selected elements -- and
// the edges, computed with torch's lerp formula and one fused multiply-add
// per branch -- are bit-identical.  Digits are 12, 8, 8 and 4 bits wide.
namespace wgb {

// Digits of the 32-bit order-preserving key, high to low: 12, 8, 8, 4 bits.
// The first digit (sign, exponent, 3 mantissa bits) spreads typical float
// columns over many buckets, so plain shared atomics see little contention.
constexpr int QS_NT = 512;      // threads per column CTA
constexpr int QS_V = 4;         // 16-byte loads in flight per thread per sweep step
constexpr int QS_MAXQ = 32;     // quantiles per sweep (64 target ranks)
constexpr int QS_MAXT = 2 * QS_MAXQ;
constexpr int QS_H0 = 4096;     // buckets of the first digit
constexpr size_t QS_SMEM = QS_MAXT * 256 * 4 + QS_H0 + 2 * QS_MAXT * 256;  // hist | tbl12 | tbl8a | tbl8b
constexpr uint8_t QS_NONE = 0xFF;

__device__ __forceinline__ uint32_t f2key(uint32_t b) { return b ^ ((b >> 31) ? 0xFFFFFFFFu : 0x80000000u); }
__device__ __forceinline__ uint32_t key2f(uint32_t k) { return k ^ ((k >> 31) ? 0x80000000u : 0xFFFFFFFFu); }

// XT[f * ld + r] = X[r][f], ld = n rounded up to a multiple of 4 (every
// column starts 16-byte aligned): 64 x 64 tiles through shared memory, a
// thread moving four consecutive floats per access -- a row's four columns
// in one 16-byte load when X allows it (vec: 16-byte aligned, row stride a
// multiple of 4), a column's four rows in one 16-byte store.  Rows in
// [n, ld) of XT get zeros (nothing reads them).
__global__ void __launch_bounds__(256) k_transpose(const float *__restrict__ X, long long n, int F, long long xs,
                                                   long long ld, float *__restrict__ XT, bool vec) {
    __shared__ float t[64][65];
    const long long r0 = (long long)blockIdx.x * 64;
    const int f0 = blockIdx.y * 64;
    const int lo = threadIdx.x & 15, hi = threadIdx.x >> 4;  // 16 groups of four x 16 lines
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rr = hi + 16 * i;
        const long long r = r0 + rr;
        const int f = f0 + 4 * lo;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r < n) {
            const float *src = X + r * xs + f;
            if (vec && f + 3 < F) {
                v = __ldg(reinterpret_cast<const float4 *>(src));
            } else {
                if (f < F) v.x = __ldg(src);
                if (f + 1 < F) v.y = __ldg(src + 1);
                if (f + 2 < F) v.z = __ldg(src + 2);
                if (f + 3 < F) v.w = __ldg(src + 3);
            }
        }
        t[rr][4 * lo] = v.x;
        t[rr][4 * lo + 1] = v.y;
        t[rr][4 * lo + 2] = v.z;
        t[rr][4 * lo + 3] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int fl = hi + 16 * i;
        const int f = f0 + fl;
        const long long r = r0 + 4 * lo;
        if (f < F && r < n)  // r + 3 < ld: r is a multiple of 4 below n
            *reinterpret_cast<float4 *>(XT + (long long)f * ld + r) =
                make_float4(t[4 * lo][fl], t[4 * lo + 1][fl], t[4 * lo + 2][fl], t[4 * lo + 3][fl]);
    }
}

// Launch of k_transpose for X [n][F] (row stride xs) into XT (ld = n rounded
// up to 4).
static cudaError_t launch_transpose(const float *X, long long n, int F, long long xs, long long ld, float *XT,
                                   cudaStream_t st) {
    const bool vec = (reinterpret_cast<uintptr_t>(X) & 15) == 0 && xs % 4 == 0;
    dim3 tg((unsigned)((n + 63) / 64), (unsigned)((F + 63) / 64));
    k_transpose<<<tg, 256, 0, st>>>(X, n, F, xs, ld, XT, vec);
    return cudaGetLastError();
}

// Cumulative search of one L-bucket row by one warp: bucket holding the
// resid-th element (0-based) and the count before it.
template <int L>
__device__ __forceinline__ void qs_find(const uint32_t *row, uint32_t resid, int &digit, uint32_t &before) {
    constexpr int PER = L / 32;
    const int lane = threadIdx.x & 31;
    uint32_t s = 0;
    for (int i = 0; i < PER; ++i) s += row[lane * PER + i];
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    const uint32_t excl = incl - s;
    const bool mine = resid >= excl && resid < incl;
    const unsigned who = __ballot_sync(0xffffffffu, mine);
    const int src = who ? __ffs(who) - 1 : 31;
    int d = 0;
    uint32_t b = 0;
    if (lane == src) {
        uint32_t acc = excl;
        d = lane * PER + PER - 1;
        for (int i = 0; i < PER; ++i) {
            const uint32_t c = row[lane * PER + i];
            if (resid < acc + c) {
                d = lane * PER + i;
                break;
            }
            acc += c;
        }
        b = acc;
    }
    digit = __shfl_sync(0xffffffffu, d, src);
    before = __shfl_sync(0xffffffffu, b, src);
}

// Digits of QS_V vectors (4 elements each) loaded by one sweep step, for
// digit pass P (0..3): elements whose higher digits match a target prefix
// (slot tables of the previous passes) are counted; pass 0 counts runs of
// one bucket with one atomic per run and reports NaNs.
template <int P>
__device__ __forceinline__ int qs_count(const uint4 (&x)[QS_V], long long v0, long long n, uint32_t *hist,
                                        const uint8_t *tbl12, const uint8_t *tbl8a, const uint8_t *tbl8b) {
    int nan_seen = 0;
    uint32_t last = 0xFFFFFFFFu, run = 0;  // pass 0: runs of one bucket, one atomic per run
#pragma unroll
    for (int u = 0; u < QS_V; ++u) {
        const long long e0 = (v0 + (long long)u * QS_NT) * 4;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if (e0 + c >= n) continue;
            const uint32_t b = c == 0 ? x[u].x : c == 1 ? x[u].y : c == 2 ? x[u].z : x[u].w;
            const uint32_t k = f2key(b);
            if (P == 0) {
                nan_seen |= (b & 0x7FFFFFFFu) > 0x7F800000u;
                const uint32_t d = k >> 20;
                if (d != last) {
                    if (run) atomicAdd(hist + last, run);
                    last = d;
                    run = 0;
                }
                ++run;
                continue;
            }
            uint32_t sl = tbl12[k >> 20];
            if (sl == QS_NONE) continue;
            if (P >= 2) {
                sl = tbl8a[sl * 256 + ((k >> 12) & 0xFF)];
                if (sl == QS_NONE) continue;
            }
            if (P >= 3) {
                sl = tbl8b[sl * 256 + ((k >> 4) & 0xFF)];
                if (sl == QS_NONE) continue;
            }
            const uint32_t d = P == 1 ? (k >> 12) & 0xFF : P == 2 ? (k >> 4) & 0xFF : k & 0xF;
            atomicAdd(hist + sl * 256 + d, 1u);
        }
    }
    if (P == 0 && run) atomicAdd(hist + last, run);
    return nan_seen;
}

__device__ __forceinline__ void qs_load(const uint4 *__restrict__ colv, long long v0, long long nvec,
                                        uint4 (&x)[QS_V]) {
#pragma unroll
    for (int u = 0; u < QS_V; ++u) {
        const long long v = v0 + (long long)u * QS_NT;
        x[u] = v < nvec ? __ldg(colv + v) : make_uint4(0u, 0u, 0u, 0u);
    }
}

// One sweep over the column for digit pass P, one register set (the
// one-launch select: its four passes in one kernel leave no registers for a
// second set).
template <int P>
__device__ __forceinline__ int qs_sweep1(const uint4 *__restrict__ colv, long long n, uint32_t *hist,
                                         const uint8_t *tbl12, const uint8_t *tbl8a, const uint8_t *tbl8b) {
    const long long nvec = (n + 3) >> 2;
    int nan_seen = 0;
    for (long long v0 = threadIdx.x; v0 < nvec; v0 += (long long)QS_NT * QS_V) {
        uint4 x[QS_V];
        qs_load(colv, v0, nvec, x);
        nan_seen |= qs_count<P>(x, v0, n, hist, tbl12, tbl8a, tbl8b);
    }
    return nan_seen;
}

// One sweep over the column for digit pass P: two register sets alternate,
// so the next step's loads are in flight while this step's digits are
// counted.
template <int P>
__device__ __forceinline__ int qs_sweep(const uint4 *__restrict__ colv, long long n, uint32_t *hist,
                                        const uint8_t *tbl12, const uint8_t *tbl8a, const uint8_t *tbl8b) {
    const long long nvec = (n + 3) >> 2;
    constexpr long long STEP = (long long)QS_NT * QS_V;
    int nan_seen = 0;
    uint4 xa[QS_V], xb[QS_V];
    long long v0 = threadIdx.x;
    if (v0 < nvec) qs_load(colv, v0, nvec, xa);
    while (v0 < nvec) {
        if (v0 + STEP < nvec) qs_load(colv, v0 + STEP, nvec, xb);
        nan_seen |= qs_count<P>(xa, v0, n, hist, tbl12, tbl8a, tbl8b);
        v0 += STEP;
        if (v0 >= nvec) break;
        if (v0 + STEP < nvec) qs_load(colv, v0 + STEP, nvec, xa);
        nan_seen |= qs_count<P>(xb, v0, n, hist, tbl12, tbl8a, tbl8b);
        v0 += STEP;
    }
    return nan_seen;
}

__global__ void __launch_bounds__(QS_NT, 2) k_qselect(const float *__restrict__ XT, long long n, long long ld,
                                                      const float *__restrict__ q, int nq, float *__restrict__ edges) {
    extern __shared__ __align__(16) uint32_t qs_dyn[];
    uint32_t *hist = qs_dyn;                                            // [QS_MAXT][256] (pass 0: [QS_H0])
    uint8_t *tbl12 = reinterpret_cast<uint8_t *>(qs_dyn + QS_MAXT * 256);  // 12-bit prefix -> pass-1 slot
    uint8_t *tbl8a = tbl12 + QS_H0;                                     // [pass-1 slot][8 bits] -> pass-2 slot
    uint8_t *tbl8b = tbl8a + QS_MAXT * 256;                             // [pass-2 slot][8 bits] -> pass-3 slot
    __shared__ int t_rank[QS_MAXT];
    __shared__ uint32_t t_key[QS_MAXT];     // resolved key prefix (high digits)
    __shared__ uint32_t t_resid[QS_MAXT];   // rank within the prefix's elements
    __shared__ int t_slot[QS_MAXT];
    __shared__ float t_w[QS_MAXQ];
    __shared__ int s_nslot;
    __shared__ uint32_t s_pre[QS_MAXT];

    const int f = blockIdx.x;
    const uint4 *colv = reinterpret_cast<const uint4 *>(XT + (long long)f * ld);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = QS_NT / 32;
    constexpr int SHIFT[4] = {20, 12, 4, 0};  // low bit of each pass's digit

    for (int q0 = 0; q0 < nq; q0 += QS_MAXQ) {
        const int nqs = min(QS_MAXQ, nq - q0);
        const int nt = 2 * nqs;
        if (tid < nqs) {
            const float last = (float)(n - 1);
            const float rank = __fmul_rn(q[q0 + tid], last);
            const long long lo = (long long)rank;
            const long long hi = (long long)ceilf(rank);
            t_rank[2 * tid] = (int)lo;
            t_rank[2 * tid + 1] = (int)hi;
            t_w[tid] = __fsub_rn(rank, (float)lo);
        }
        // ---- pass 0: first digit, NaN detection
        for (int t = tid; t < QS_H0; t += QS_NT) hist[t] = 0;
        __syncthreads();
        const int nan_seen = qs_sweep1<0>(colv, n, hist, tbl12, tbl8a, tbl8b);
        if (__syncthreads_or(nan_seen)) {  // torch: every rank -> n-1 (the NaN)
            for (int j = tid; j < nq; j += QS_NT) edges[(long long)f * nq + j] = __int_as_float(0x7fc00000);
            return;
        }
        for (int t = warp; t < nt; t += NW) {
            int d;
            uint32_t before;
            qs_find<QS_H0>(hist, (uint32_t)t_rank[t], d, before);
            if (lane == 0) {
                t_key[t] = (uint32_t)d << 20;
                t_resid[t] = (uint32_t)t_rank[t] - before;
            }
        }
        __syncthreads();
        // ---- passes 1..3
#pragma unroll
        for (int p = 1; p <= 3; ++p) {
            const int sh = SHIFT[p - 1];     // the resolved prefix is key >> sh
            if (tid == 0) {                  // distinct prefixes -> slots (<= 64 targets)
                int ns = 0;
                for (int t = 0; t < nt; ++t) {
                    const uint32_t pre = t_key[t] >> sh;
                    int sl = -1;
                    for (int u = 0; u < ns; ++u)
                        if (s_pre[u] == pre) { sl = u; break; }
                    if (sl < 0) { sl = ns; s_pre[ns++] = pre; }
                    t_slot[t] = sl;
                }
                s_nslot = ns;
            }
            __syncthreads();
            const int ns = s_nslot;
            if (p == 1) {
                for (int t = tid; t < QS_H0; t += QS_NT) tbl12[t] = QS_NONE;
            } else {
                uint8_t *tb = p == 2 ? tbl8a : tbl8b;
                for (int t = tid; t < QS_MAXT * 256; t += QS_NT) tb[t] = QS_NONE;
            }
            for (int t = tid; t < ns * 256; t += QS_NT) hist[t] = 0;
            __syncthreads();
            if (tid < ns) {
                const uint32_t pre = s_pre[tid];
                if (p == 1) {
                    tbl12[pre] = (uint8_t)tid;
                } else if (p == 2) {
                    tbl8a[tbl12[pre >> 8] * 256 + (pre & 0xFF)] = (uint8_t)tid;
                } else {
                    const int s1 = tbl12[pre >> 16];
                    const int s2 = tbl8a[s1 * 256 + ((pre >> 8) & 0xFF)];
                    tbl8b[s2 * 256 + (pre & 0xFF)] = (uint8_t)tid;
                }
            }
            __syncthreads();
            if (p == 1) qs_sweep1<1>(colv, n, hist, tbl12, tbl8a, tbl8b);
            else if (p == 2) qs_sweep1<2>(colv, n, hist, tbl12, tbl8a, tbl8b);
            else qs_sweep1<3>(colv, n, hist, tbl12, tbl8a, tbl8b);
            __syncthreads();
            for (int t = warp; t < nt; t += NW) {
                int d;
                uint32_t before;
                qs_find<256>(hist + t_slot[t] * 256, t_resid[t], d, before);
                if (lane == 0) {
                    t_key[t] |= (uint32_t)d << SHIFT[p];
                    t_resid[t] -= before;
                }
            }
            __syncthreads();
        }
        // ---- edges: torch's lerp with one FMA per branch
        if (tid < nqs) {
            const float a = __int_as_float((int)key2f(t_key[2 * tid]));
            const float b = __int_as_float((int)key2f(t_key[2 * tid + 1]));
            const float w = t_w[tid];
            const float d = __fsub_rn(b, a);
            const float e = (fabsf(w) < 0.5f) ? __fmaf_rn(w, d, a) : __fmaf_rn(-d, __fsub_rn(1.0f, w), b);
            edges[(long long)f * nq + q0 + tid] = e;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Row-sharded columns (several ranks): the same radix select, one digit pass
// per launch.  Each rank histograms the digit of its own rows
// (k_qs_local<P>), the histograms are summed over the ranks between passes
// (an int32 all-reduce), and every rank resolves the same digits from the
// sums (k_qs_pick<P>) -- the order statistics of the concatenated column, so
// torch.quantile's edges over it bit for bit, without moving any row.  At
// most QS_MAXQ quantiles.  Per-column state (uint32): the resolved keys of
// the 2*nq targets, their residual ranks, and a NaN flag.
constexpr int QS_STATE = 2 * QS_MAXT + 1;
constexpr int QS_HCOL = QS_MAXT * 256;  // histogram words per column, passes 1-3 (pass 0: QS_H0)

// Slots of digit pass p (1..3): the distinct resolved prefixes (key >> sh,
// sh = the low bit of pass p-1's digit) in target order.  One thread.
__device__ __forceinline__ int qs_slots(const uint32_t *key, int nt, int sh, int *slot, uint32_t *pre) {
    int ns = 0;
    for (int t = 0; t < nt; ++t) {
        const uint32_t pr = key[t] >> sh;
        int sl = -1;
        for (int u = 0; u < ns; ++u)
            if (pre[u] == pr) { sl = u; break; }
        if (sl < 0) { sl = ns; pre[ns++] = pr; }
        slot[t] = sl;
    }
    return ns;
}

template <int P>
__global__ void __launch_bounds__(QS_NT, 2) k_qs_local(const float *__restrict__ XT, long long n, long long ld,
                                                       int nq, const uint32_t *__restrict__ state,
                                                       uint32_t *__restrict__ hist_out, int *__restrict__ nan_out) {
    extern __shared__ __align__(16) uint32_t qs_dyn[];
    uint32_t *hist = qs_dyn;
    uint8_t *tbl12 = reinterpret_cast<uint8_t *>(qs_dyn + QS_MAXT * 256);
    uint8_t *tbl8a = tbl12 + QS_H0;
    uint8_t *tbl8b = tbl8a + QS_MAXT * 256;
    __shared__ uint32_t t_key[QS_MAXT], s_pre[QS_MAXT];
    __shared__ int t_slot[QS_MAXT], s_nslot;
    constexpr int SHIFT[4] = {20, 12, 4, 0};
    const int f = blockIdx.x, tid = threadIdx.x;
    const uint4 *colv = reinterpret_cast<const uint4 *>(XT + (long long)f * ld);
    if (P == 0) {
        for (int t = tid; t < QS_H0; t += QS_NT) hist[t] = 0;
        __syncthreads();
        const int nan_seen = n > 0 ? qs_sweep<0>(colv, n, hist, tbl12, tbl8a, tbl8b) : 0;
        const int any = __syncthreads_or(nan_seen);
        for (int t = tid; t < QS_H0; t += QS_NT) hist_out[(long long)f * QS_H0 + t] = hist[t];
        if (tid == 0) nan_out[f] = any;
        return;
    }
    const uint32_t *st = state + (long long)f * QS_STATE;
    if (st[2 * QS_MAXT]) return;  // NaN column: its edges are decided
    const int nt = 2 * nq;
    if (tid < nt) t_key[tid] = st[tid];
    __syncthreads();
    // the slot tables of passes 1..P, as the one-launch select builds them
    for (int p = 1; p <= P; ++p) {
        if (tid == 0) s_nslot = qs_slots(t_key, nt, SHIFT[p - 1], t_slot, s_pre);
        if (p == 1) {
            for (int t = tid; t < QS_H0; t += QS_NT) tbl12[t] = QS_NONE;
        } else {
            uint8_t *tb = p == 2 ? tbl8a : tbl8b;
            for (int t = tid; t < QS_MAXT * 256; t += QS_NT) tb[t] = QS_NONE;
        }
        __syncthreads();
        if (tid < s_nslot) {
            const uint32_t pre = s_pre[tid];
            if (p == 1) {
                tbl12[pre] = (uint8_t)tid;
            } else if (p == 2) {
                tbl8a[tbl12[pre >> 8] * 256 + (pre & 0xFF)] = (uint8_t)tid;
            } else {
                const int s1 = tbl12[pre >> 16];
                const int s2 = tbl8a[s1 * 256 + ((pre >> 8) & 0xFF)];
                tbl8b[s2 * 256 + (pre & 0xFF)] = (uint8_t)tid;
            }
        }
        __syncthreads();
    }
    const int ns = s_nslot;
    for (int t = tid; t < ns * 256; t += QS_NT) hist[t] = 0;
    __syncthreads();
    if (n > 0) qs_sweep<P>(colv, n, hist, tbl12, tbl8a, tbl8b);
    __syncthreads();
    for (int t = tid; t < ns * 256; t += QS_NT) hist_out[(long long)f * QS_HCOL + t] = hist[t];
}

template <int P>
__global__ void __launch_bounds__(256) k_qs_pick(const uint32_t *__restrict__ hist_in, const int *__restrict__ nan_in,
                                                 long long n, const float *__restrict__ q, int nq,
                                                 uint32_t *__restrict__ state, float *__restrict__ edges) {
    extern __shared__ __align__(16) uint32_t qs_row[];  // the column's summed histogram
    __shared__ uint32_t t_key[QS_MAXT], t_resid[QS_MAXT], s_pre[QS_MAXT];
    __shared__ int t_slot[QS_MAXT], s_nslot;
    constexpr int SHIFT[4] = {20, 12, 4, 0};
    const int f = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = 256 / 32;
    const int nt = 2 * nq;
    uint32_t *st = state + (long long)f * QS_STATE;
    if (P == 0) {
        if (nan_in[f]) {  // torch: every rank -> n-1 (the NaN)
            if (tid == 0) st[2 * QS_MAXT] = 1u;
            for (int j = tid; j < nq; j += 256) edges[(long long)f * nq + j] = __int_as_float(0x7fc00000);
            return;
        }
        for (int t = tid; t < QS_H0; t += 256) qs_row[t] = hist_in[(long long)f * QS_H0 + t];
        if (tid < nq) {
            const float rank = __fmul_rn(q[tid], (float)(n - 1));
            t_resid[2 * tid] = (uint32_t)(long long)rank;
            t_resid[2 * tid + 1] = (uint32_t)(long long)ceilf(rank);
        }
        __syncthreads();
        for (int t = warp; t < nt; t += NW) {
            int d;
            uint32_t before;
            qs_find<QS_H0>(qs_row, t_resid[t], d, before);
            if (lane == 0) {
                st[t] = (uint32_t)d << 20;
                st[QS_MAXT + t] = t_resid[t] - before;
            }
        }
        if (tid == 0) st[2 * QS_MAXT] = 0u;
        return;
    }
    if (st[2 * QS_MAXT]) return;
    if (tid < nt) {
        t_key[tid] = st[tid];
        t_resid[tid] = st[QS_MAXT + tid];
    }
    __syncthreads();
    if (tid == 0) s_nslot = qs_slots(t_key, nt, SHIFT[P - 1], t_slot, s_pre);
    __syncthreads();
    for (int t = tid; t < s_nslot * 256; t += 256) qs_row[t] = hist_in[(long long)f * QS_HCOL + t];
    __syncthreads();
    for (int t = warp; t < nt; t += NW) {
        int d;
        uint32_t before;
        qs_find<256>(qs_row + t_slot[t] * 256, t_resid[t], d, before);
        if (lane == 0) {
            t_key[t] |= (uint32_t)d << SHIFT[P];
            t_resid[t] -= before;
        }
    }
    __syncthreads();
    if (tid < nt) {
        st[tid] = t_key[tid];
        st[QS_MAXT + tid] = t_resid[tid];
    }
    if (P == 3 && tid < nq) {  // edges: torch's lerp with one FMA per branch
        const float rank = __fmul_rn(q[tid], (float)(n - 1));
        const float w = __fsub_rn(rank, (float)(long long)rank);
        const float a = __int_as_float((int)key2f(t_key[2 * tid]));
        const float b = __int_as_float((int)key2f(t_key[2 * tid + 1]));
        const float dd = __fsub_rn(b, a);
        edges[(long long)f * nq + tid] =
            (fabsf(w) < 0.5f) ? __fmaf_rn(w, dd, a) : __fmaf_rn(-dd, __fsub_rn(1.0f, w), b);
    }
}

}  // namespace wgb

using namespace wgb;

extern "C" int wgb_quantile_edges(const float *X, int64_t n, int32_t F, int64_t x_stride, const float *q,
                                  int32_t nq, float *XT, float *edges, void *stream) {
    WGB_CHECK_ARG(n >= 1 && F >= 1 && nq >= 1, "bad sizes n=%lld F=%d nq=%d", (long long)n, F, nq);
    WGB_CHECK_ARG(n <= (1ll << 24), "quantile() input tensor is too large");
    WGB_CHECK_ARG(x_stride >= F, "x_stride < F");
    WGB_CHECK_ARG(X && q && XT && edges, "NULL pointer");
    WGB_CHECK_ARG((reinterpret_cast<uintptr_t>(XT) & 15) == 0, "XT must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    const long long ld = (n + 3) & ~3ll;
    WGB_CUDA(launch_transpose(X, n, F, x_stride, ld, XT, st));
    WGB_CUDA(cudaFuncSetAttribute(k_qselect, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QS_SMEM));
    k_qselect<<<(unsigned)F, QS_NT, QS_SMEM, st>>>(XT, n, ld, q, nq, edges);
    WGB_LAUNCHED("k_qselect");
    return WGB_OK;
}

extern "C" int wgb_quantile_pass(int32_t pass, const float *X, int64_t n, int32_t F, int64_t x_stride, int32_t nq,
                                 float *XT, const uint32_t *state, uint32_t *hist, int32_t *nan_flags, void *stream) {
    WGB_CHECK_ARG(pass >= 0 && pass <= 3, "pass %d out of range", pass);
    WGB_CHECK_ARG(n >= 0 && F >= 1 && nq >= 1 && nq <= QS_MAXQ, "bad sizes n=%lld F=%d nq=%d (nq <= %d)",
                  (long long)n, F, nq, QS_MAXQ);
    WGB_CHECK_ARG(n <= (1ll << 24), "quantile() input tensor is too large");
    WGB_CHECK_ARG(x_stride >= F, "x_stride < F");
    WGB_CHECK_ARG(XT && state && hist && nan_flags && (pass > 0 || X || n == 0), "NULL pointer");
    WGB_CHECK_ARG((reinterpret_cast<uintptr_t>(XT) & 15) == 0, "XT must be 16-byte aligned");
    cudaStream_t st = as_stream(stream);
    const long long ld = (n + 3) & ~3ll;
    if (pass == 0 && n > 0) WGB_CUDA(launch_transpose(X, n, F, x_stride, ld, XT, st));
#define WGB_QS_LOCAL(P_)                                                                                      \
    WGB_CUDA(cudaFuncSetAttribute(k_qs_local<P_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QS_SMEM)); \
    k_qs_local<P_><<<(unsigned)F, QS_NT, QS_SMEM, st>>>(XT, n, ld, nq, state, hist, nan_flags);
    if (pass == 0) { WGB_QS_LOCAL(0) } else if (pass == 1) { WGB_QS_LOCAL(1) } else if (pass == 2) { WGB_QS_LOCAL(2) } else { WGB_QS_LOCAL(3) }
#undef WGB_QS_LOCAL
    WGB_LAUNCHED("k_qs_local");
    return WGB_OK;
}

extern "C" int wgb_quantile_pick(int32_t pass, const uint32_t *hist, const int32_t *nan_flags, int64_t n_total,
                                 const float *q, int32_t nq, int32_t F, uint32_t *state, float *edges,
                                 void *stream) {
    WGB_CHECK_ARG(pass >= 0 && pass <= 3, "pass %d out of range", pass);
    WGB_CHECK_ARG(n_total >= 1 && n_total <= (1ll << 24), "n_total=%lld outside [1, 2^24]", (long long)n_total);
    WGB_CHECK_ARG(F >= 1 && nq >= 1 && nq <= QS_MAXQ, "bad sizes F=%d nq=%d (nq <= %d)", F, nq, QS_MAXQ);
    WGB_CHECK_ARG(hist && nan_flags && q && state && edges, "NULL pointer");
    cudaStream_t st = as_stream(stream);
    const size_t sm = (size_t)(pass == 0 ? QS_H0 : QS_HCOL) * sizeof(uint32_t);
#define WGB_QS_PICK(P_)                                                                                   \
    WGB_CUDA(cudaFuncSetAttribute(k_qs_pick<P_>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));  \
    k_qs_pick<P_><<<(unsigned)F, 256, sm, st>>>(hist, nan_flags, n_total, q, nq, state, edges);
    if (pass == 0) { WGB_QS_PICK(0) } else if (pass == 1) { WGB_QS_PICK(1) } else if (pass == 2) { WGB_QS_PICK(2) } else { WGB_QS_PICK(3) }
#undef WGB_QS_PICK
    WGB_LAUNCHED("k_qs_pick");
    return WGB_OK;
}
