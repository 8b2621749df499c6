// Shared helpers of the warpgbm_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <climits>
#include <cmath>

#include "../../include/warpgbm_b200.h"

namespace wgb {

// ---------------------------------------------------------------- errors --
void set_error(const char *fmt, ...);

#define WGB_CHECK_ARG(cond, ...)                                              \
    do {                                                                      \
        if (!(cond)) {                                                        \
            ::wgb::set_error(__VA_ARGS__);                                    \
            return WGB_ERR_ARG;                                               \
        }                                                                     \
    } while (0)

#define WGB_CUDA(call)                                                        \
    do {                                                                      \
        cudaError_t e_ = (call);                                              \
        if (e_ != cudaSuccess) {                                              \
            ::wgb::set_error("%s failed: %s (%s:%d)", #call,                  \
                             cudaGetErrorString(e_), __FILE__, __LINE__);     \
            return WGB_ERR_CUDA;                                              \
        }                                                                     \
    } while (0)

#define WGB_LAUNCHED(name)                                                    \
    do {                                                                      \
        cudaError_t e_ = cudaGetLastError();                                  \
        if (e_ != cudaSuccess) {                                              \
            ::wgb::set_error("launch of %s failed: %s", name,                 \
                             cudaGetErrorString(e_));                         \
            return WGB_ERR_CUDA;                                              \
        }                                                                     \
    } while (0)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch: the kernels of a tree level are launched
// with programmatic stream serialisation, so each one's launch is prepared
// while its predecessor on the stream finishes; every such kernel first
// waits (griddepcontrol.wait) until that predecessor has completed and its
// writes are visible.  Launched without the attribute, the wait returns at
// once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

#define WGB_PDL(name, ...)                                                                 \
    do {                                                                                   \
        cudaError_t e_ = ::wgb::launch_pdl(__VA_ARGS__);                                   \
        if (e_ != cudaSuccess) {                                                           \
            ::wgb::set_error("launch of %s failed: %s", name, cudaGetErrorString(e_));     \
            return WGB_ERR_CUDA;                                                           \
        }                                                                                  \
    } while (0)

// ------------------------------------------------------------ constants --
constexpr int HIST_R = 2048;        // rows per histogram chunk (cell packing needs <= 2048)
// Packing of a histogram cell into two 32-bit shared words for <= HIST_R rows:
//   A += (1 << HIST_CNT_SHIFT) + (q & HIST_LO_MASK),  B += q >> HIST_LO_BITS
// count = A >> HIST_CNT_SHIFT, sum q = B * 2^HIST_LO_BITS + (A & (2^HIST_CNT_SHIFT - 1)).
// |q| <= 2^29 - 32 (fp32 residuals), so 2048 rows keep A below 2^32 and B in int32.
constexpr int HIST_CNT_SHIFT = 20;
constexpr int HIST_LO_BITS = 9;
constexpr uint32_t HIST_LO_MASK = (1u << HIST_LO_BITS) - 1u;
constexpr uint32_t HIST_A_SUM_MASK = (1u << HIST_CNT_SHIFT) - 1u;
#define HIST_ERA_R(has_era) ((has_era) ? HIST_R : 1)
constexpr int HIST_THREADS = 256;

// Where a histogram build adds its cells: cell (slot, era e, position kp,
// bin b) of the sums is g[(kp / ks) * slice_stride + (slot - slot0) *
// slot_elems + (e * ks + kp % ks) * (B + 1) + b], the count the same offset
// from c.  The histogram pool is the case ks = k, slice_stride = 0, slot0 =
// 0; a sliced fit's staging buffer holds one region of the level's slots per
// slice of ks positions.
struct HistOut {
    long long *g, *c;
    long long slot_elems, slice_stride;
    int ks, slot0;
};
constexpr int SPLIT_WARPS = 8;     // features per single-era split block (one warp each)
constexpr int PART_TILE = 2048;     // positions per partition tile
constexpr int PART_THREADS = 256;

// --------------------------------------------------------- fixed point --
// Residual quantisation: q = rint(g * 2^s), s = 29 - e where max|g| = m*2^e,
// m in [0.5, 1).  With fp32 residuals m <= 1 - 2^-24, so |q| <= 2^29 - 32:
// int64 totals hold 2^33 rows and the histogram kernel's two 32-bit shared
// words per cell stay exact for HIST_R rows.
__host__ __device__ inline int quant_shift(float maxabs) {
    if (!(maxabs > 0.0f) || isinf(maxabs)) return 0;
    int e;
    frexpf(maxabs, &e);
    int s = 29 - e;
    if (s > 126) s = 126;
    if (s < -99) s = -99;
    return s;
}

// wgb_node.built: bit 0 = histogram built from rows, bits 8.. = the node's
// tree within the batch of trees grown together (its class offset)
__host__ __device__ inline int node_flags(bool built, int tree) { return (tree << 8) | (built ? 1 : 0); }
__host__ __device__ inline bool node_built(int flags) { return (flags & 1) != 0; }
__host__ __device__ inline int node_tree(int flags) { return flags >> 8; }

// 2^s as float for s in [-126, 127]
__device__ __forceinline__ float pow2f(int s) { return __int_as_float((127 + s) << 23); }

// Leaf value = mean residual of the node's rows from the exact sums
// (fp32 ops: float(sum_q) * 2^-s, times 1/float(n)).
__device__ __forceinline__ float canon_leaf(long long sumq, long long count, float inv) {
    float sf = __fmul_rn(__ll2float_rn(sumq), inv);
    float fac = __fdiv_rn(1.0f, __ll2float_rn(count));
    return __fmul_rn(sf, fac);
}

// best_split_kernel.cu:42-50 with one IEEE rounding per operation.
struct SplitEval {
    float gain;
    float dir;
};
__device__ __forceinline__ SplitEval eval_split(float GL, float HL, float GT, float HT, float mcw,
                                                float eps) {
    SplitEval r{0.0f, 0.0f};
    float GR = __fsub_rn(GT, GL);
    float HR = __fsub_rn(HT, HL);
    if (HL >= mcw && HR >= mcw) {
        float dl = __fadd_rn(HL, eps), dr = __fadd_rn(HR, eps), dt = __fadd_rn(HT, eps);
        float t1 = __fdiv_rn(__fmul_rn(GL, GL), dl);
        float t2 = __fdiv_rn(__fmul_rn(GR, GR), dr);
        float t3 = __fdiv_rn(__fmul_rn(GT, GT), dt);
        r.gain = __fsub_rn(__fadd_rn(t1, t2), t3);
        float lv = __fdiv_rn(GL, dl), rv = __fdiv_rn(GR, dr);
        r.dir = (lv > rv) ? 1.0f : -1.0f;
    }
    return r;
}

// The same with the parent term t3 = (GT*GT) / (HT + eps) computed once per
// feature (it does not depend on the split point; identical value).
__device__ __forceinline__ float parent_term(float GT, float HT, float eps) {
    return __fdiv_rn(__fmul_rn(GT, GT), __fadd_rn(HT, eps));
}
__device__ __forceinline__ SplitEval eval_split_pt(float GL, float HL, float GT, float HT, float t3, float mcw,
                                                   float eps) {
    SplitEval r{0.0f, 0.0f};
    float GR = __fsub_rn(GT, GL);
    float HR = __fsub_rn(HT, HL);
    if (HL >= mcw && HR >= mcw) {
        float dl = __fadd_rn(HL, eps), dr = __fadd_rn(HR, eps);
        float t1 = __fdiv_rn(__fmul_rn(GL, GL), dl);
        float t2 = __fdiv_rn(__fmul_rn(GR, GR), dr);
        r.gain = __fsub_rn(__fadd_rn(t1, t2), t3);
        float lv = __fdiv_rn(GL, dl), rv = __fdiv_rn(GR, dr);
        r.dir = (lv > rv) ? 1.0f : -1.0f;
    }
    return r;
}

// Arg-max key of the directional era split (core.py:577-594): higher
// agreement first (max over every candidate), then higher masked criterion
// (-inf where crit <= min_split_gain), then the lower flat index.
struct Key {
    int A;
    float c;
    int idx;
};
__device__ __forceinline__ bool key_better(const Key &a, const Key &b) {
    if (a.A != b.A) return a.A > b.A;
    if (a.c != b.c) return a.c > b.c;
    return a.idx < b.idx;
}
__device__ __forceinline__ Key key_none() { return Key{-1, -INFINITY, INT_MAX}; }

__device__ __forceinline__ Key warp_key_max(Key k) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Key t;
        t.A = __shfl_xor_sync(0xffffffffu, k.A, o);
        t.c = __shfl_xor_sync(0xffffffffu, k.c, o);
        t.idx = __shfl_xor_sync(0xffffffffu, k.idx, o);
        if (key_better(t, k)) k = t;
    }
    return k;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int warp_min(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide minimum (every thread gets the result).  Contains barriers.
__device__ __forceinline__ int block_min(int v, int *scratch /* >= 33 ints */) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_min(v);
    if (lane == 0) scratch[w] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        int m = INT_MAX;
        for (int i = 0; i < nw; ++i) m = min(m, scratch[i]);
        scratch[32] = m;
    }
    __syncthreads();
    int r = scratch[32];
    __syncthreads();
    return r;
}

// First index in a[0, n) (ascending) whose value is >= v; n if none.
__device__ __forceinline__ int lower_bound_int(const int *a, int n, int v) {
    int lo = 0, hi = n;
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (a[mid] < v) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// Exclusive prefix sum over the block (blockDim.x a multiple of 32, at most
// 1024); `total` receives the block's sum.  Every thread calls it.
__device__ __forceinline__ int block_scan_excl(int v, int *scratch /* >= 33 ints */, int &total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) scratch[w] = incl;
    __syncthreads();
    if (w == 0) {
        const int t = lane < nw ? scratch[lane] : 0;
        int ti = t;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, ti, o);
            if (lane >= o) ti += u;
        }
        scratch[lane] = ti - t;
        if (lane == 31) scratch[32] = ti;
    }
    __syncthreads();
    const int r = scratch[w] + incl - v;
    total = scratch[32];
    __syncthreads();
    return r;
}

}  // namespace wgb
