// Exact quantile edges of every feature column (sm_100a), replacing the
// per-column torch.quantile(X[:, f], linspace(0, 1, B+1)[1:-1]) of the
// reference's preprocess_gpu_data (warpgbm/core.py:527-538).
//
// torch.quantile (linear) sorts the column, takes rank = q * (n - 1) in fp32,
// below = trunc(rank), above = ceil(rank), w = rank - below and returns
// lerp(sorted[below], sorted[above], w); any NaN in the column sets every
// rank to n - 1 (the NaN), so all edges are NaN.  Only the 2 (B - 1) order
// statistics are needed, so instead of a sort each column does a radix
// select: four passes over the column, one 8-bit digit of the
// order-preserving key per pass, histogramming only elements whose higher
// digits match a still-active target prefix.  Keys order exactly like the
// radix sort torch uses (-0.0 before +0.0), so the selected elements -- and
// the edges, computed with torch's lerp formula and one fused multiply-add
// per branch -- are bit-identical.
namespace wgb {

constexpr int QS_NT = 512;      // threads per column CTA
constexpr int QS_U = 8;         // elements per thread per sweep step (loads in flight)
constexpr int QS_MAXQ = 32;     // quantiles per sweep (64 target ranks)
constexpr int QS_MAXT = 2 * QS_MAXQ;
constexpr size_t QS_SMEM = QS_MAXT * 256 * 4 + 2 * QS_MAXT * 256 * 2;

__device__ __forceinline__ uint32_t f2key(uint32_t b) { return b ^ ((b >> 31) ? 0xFFFFFFFFu : 0x80000000u); }
__device__ __forceinline__ uint32_t key2f(uint32_t k) { return k ^ ((k >> 31) ? 0x80000000u : 0xFFFFFFFFu); }

// [f][r] = X[r][f]: 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256) k_transpose(const float *__restrict__ X, long long n, int F, long long xs,
                                                   float *__restrict__ XT) {
    __shared__ float t[32][33];
    const long long r0 = (long long)blockIdx.x * 32;
    const int f0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows of threads
    for (int y = ty; y < 32; y += 8) {
        long long r = r0 + y;
        int f = f0 + tx;
        t[y][tx] = (r < n && f < F) ? __ldg(X + r * xs + f) : 0.0f;
    }
    __syncthreads();
    for (int y = ty; y < 32; y += 8) {
        int f = f0 + y;
        long long r = r0 + tx;
        if (f < F && r < n) XT[(long long)f * n + r] = t[tx][y];
    }
}

// warp-aggregated histogram increment; key < 0 = no increment.  Every lane
// of the warp calls it.
__device__ __forceinline__ void qs_count(uint32_t *hist, int key) {
    const unsigned m = __match_any_sync(0xffffffffu, key);
    const int lane = threadIdx.x & 31;
    if (key >= 0 && lane == __ffs(m) - 1) atomicAdd(hist + key, (uint32_t)__popc(m));
}

// Cumulative search of one 256-bucket row by one warp: bucket holding the
// resid-th element (0-based), and the count before it.
__device__ __forceinline__ void qs_find(const uint32_t *row, uint32_t resid, int &digit, uint32_t &before) {
    const int lane = threadIdx.x & 31;
    uint32_t c[8];
    uint32_t s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        c[i] = row[lane * 8 + i];
        s += c[i];
    }
    uint32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    uint32_t excl = incl - s;
    // lane whose range [excl, incl) holds resid
    const bool mine = resid >= excl && resid < incl;
    const unsigned who = __ballot_sync(0xffffffffu, mine);
    const int src = who ? __ffs(who) - 1 : 31;
    int d = 0;
    uint32_t b = 0;
    if (lane == src) {
        uint32_t acc = excl;
        d = lane * 8 + 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (resid < acc + c[i]) {
                d = lane * 8 + i;
                break;
            }
            acc += c[i];
        }
        b = acc;
    }
    digit = __shfl_sync(0xffffffffu, d, src);
    before = __shfl_sync(0xffffffffu, b, src);
}

__global__ void __launch_bounds__(QS_NT) k_qselect(const float *__restrict__ XT, long long n, const float *__restrict__ q,
                                                   int nq, float *__restrict__ edges) {
    extern __shared__ uint32_t qs_dyn[];        // hist | tbl2 | tbl3 (QS_SMEM bytes)
    uint32_t *hist = qs_dyn;                    // [QS_MAXT][256]; pass 0: per-warp rows
    short *tbl2 = reinterpret_cast<short *>(qs_dyn + QS_MAXT * 256);  // [QS_MAXT][256]
    short *tbl3 = tbl2 + QS_MAXT * 256;                               // [QS_MAXT][256]
    __shared__ short tbl1[256];
    __shared__ int t_rank[QS_MAXT];
    __shared__ uint32_t t_key[QS_MAXT];     // resolved key prefix (high digits)
    __shared__ uint32_t t_resid[QS_MAXT];   // rank within the prefix's elements
    __shared__ int t_slot[QS_MAXT];
    __shared__ float t_w[QS_MAXQ];
    __shared__ int s_nan, s_nslot;
    __shared__ uint32_t s_pre[QS_MAXT];

    const int f = blockIdx.x;
    const float *col = XT + (long long)f * n;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = QS_NT / 32;
    const uint32_t *colb = reinterpret_cast<const uint32_t *>(col);

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
        // ---- pass 0: digit 0 histogram (per warp), NaN detection
        for (int t = tid; t < NW * 256; t += QS_NT) hist[t] = 0;
        if (tid == 0) s_nan = 0;
        __syncthreads();
        int nan_seen = 0;
        for (long long base = (long long)warp * 32 * QS_U; base < n; base += (long long)QS_NT * QS_U) {
            uint32_t b[QS_U];
#pragma unroll
            for (int u = 0; u < QS_U; ++u) {
                const long long i = base + 32 * u + lane;
                b[u] = i < n ? __ldg(colb + i) : 0xFFFFFFFFu;  // marker: past the column end
            }
#pragma unroll
            for (int u = 0; u < QS_U; ++u) {
                const bool in = base + 32 * u + lane < n;
                nan_seen |= in && (b[u] & 0x7FFFFFFFu) > 0x7F800000u;
                qs_count(hist + warp * 256, in ? (int)(f2key(b[u]) >> 24) : -1);
            }
        }
        if (__syncthreads_or(nan_seen)) {  // torch: every rank -> n-1 (the NaN)
            for (int j = tid; j < nq; j += QS_NT) edges[(long long)f * nq + j] = __int_as_float(0x7fc00000);
            return;
        }
        // fold warp rows into row 0
        for (int d = tid; d < 256; d += QS_NT) {
            uint32_t s = 0;
            for (int w = 0; w < NW; ++w) s += hist[w * 256 + d];
            hist[d] = s;
        }
        __syncthreads();
        // each target: digit 0 and residual rank (one warp per target)
        for (int t = warp; t < nt; t += NW) {
            int d;
            uint32_t before;
            qs_find(hist, (uint32_t)t_rank[t], d, before);
            if (lane == 0) {
                t_key[t] = (uint32_t)d << 24;
                t_resid[t] = (uint32_t)t_rank[t] - before;
            }
        }
        __syncthreads();
        // ---- passes 1..3
        for (int p = 1; p <= 3; ++p) {
            const int sh_hi = 32 - 8 * p;        // bits above the digit of this pass
            // distinct prefixes of this level -> slots (one thread, <= 64 targets)
            if (tid == 0) {
                int ns = 0;
                for (int t = 0; t < nt; ++t) {
                    const uint32_t pre = t_key[t] >> sh_hi;
                    int s = -1;
                    for (int u = 0; u < ns; ++u)
                        if (s_pre[u] == pre) { s = u; break; }
                    if (s < 0) { s = ns; s_pre[ns++] = pre; }
                    t_slot[t] = s;
                }
                s_nslot = ns;
            }
            __syncthreads();
            const int ns = s_nslot;
            // lookup table of this level: element prefix -> slot
            if (p == 1) {
                for (int t = tid; t < 256; t += QS_NT) tbl1[t] = -1;
            } else if (p == 2) {
                for (int t = tid; t < QS_MAXT * 256; t += QS_NT) tbl2[t] = -1;
            } else {
                for (int t = tid; t < QS_MAXT * 256; t += QS_NT) tbl3[t] = -1;
            }
            for (int t = tid; t < ns * 256; t += QS_NT) hist[t] = 0;
            __syncthreads();
            if (tid < ns) {
                const uint32_t pre = s_pre[tid];
                if (p == 1) {
                    tbl1[pre & 0xFF] = (short)tid;
                } else if (p == 2) {
                    tbl2[tbl1[(pre >> 8) & 0xFF] * 256 + (pre & 0xFF)] = (short)tid;
                } else {
                    const int s1 = tbl1[(pre >> 16) & 0xFF];
                    const int s2 = tbl2[s1 * 256 + ((pre >> 8) & 0xFF)];
                    tbl3[s2 * 256 + (pre & 0xFF)] = (short)tid;
                }
            }
            __syncthreads();
            for (long long base = (long long)warp * 32 * QS_U; base < n; base += (long long)QS_NT * QS_U) {
                uint32_t b[QS_U];
#pragma unroll
                for (int u = 0; u < QS_U; ++u) {
                    const long long i = base + 32 * u + lane;
                    b[u] = i < n ? __ldg(colb + i) : 0u;
                }
#pragma unroll
                for (int u = 0; u < QS_U; ++u) {
                    int key = -1;
                    if (base + 32 * u + lane < n) {
                        const uint32_t k = f2key(b[u]);
                        int s = tbl1[k >> 24];
                        if (s >= 0 && p >= 2) s = tbl2[s * 256 + ((k >> 16) & 0xFF)];
                        if (s >= 0 && p >= 3) s = tbl3[s * 256 + ((k >> 8) & 0xFF)];
                        if (s >= 0) key = s * 256 + (int)((k >> (sh_hi - 8)) & 0xFF);
                    }
                    if (__any_sync(0xffffffffu, key >= 0)) qs_count(hist, key);  // warp-uniform
                }
            }
            __syncthreads();
            for (int t = warp; t < nt; t += NW) {
                int d;
                uint32_t before;
                qs_find(hist + t_slot[t] * 256, t_resid[t], d, before);
                if (lane == 0) {
                    t_key[t] |= (uint32_t)d << (sh_hi - 8);
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

}  // namespace wgb

using namespace wgb;

extern "C" int wgb_quantile_edges(const float *X, int64_t n, int32_t F, int64_t x_stride, const float *q,
                                  int32_t nq, float *XT, float *edges, void *stream) {
    WGB_CHECK_ARG(n >= 1 && F >= 1 && nq >= 1, "bad sizes n=%lld F=%d nq=%d", (long long)n, F, nq);
    WGB_CHECK_ARG(n <= (1ll << 24), "quantile() input tensor is too large");
    WGB_CHECK_ARG(x_stride >= F, "x_stride < F");
    WGB_CHECK_ARG(X && q && XT && edges, "NULL pointer");
    cudaStream_t st = as_stream(stream);
    dim3 tg((unsigned)((n + 31) / 32), (unsigned)((F + 31) / 32));
    k_transpose<<<tg, 256, 0, st>>>(X, n, F, x_stride, XT);
    WGB_LAUNCHED("k_transpose");
    WGB_CUDA(cudaFuncSetAttribute(k_qselect, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QS_SMEM));
    k_qselect<<<(unsigned)F, QS_NT, QS_SMEM, st>>>(XT, n, q, nq, edges);
    WGB_LAUNCHED("k_qselect");
    return WGB_OK;
}
