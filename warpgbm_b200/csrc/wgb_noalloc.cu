// wgb_compute_histogram3_noalloc: the histogram of wgb_compute_histogram3
// for callers that are not allowed to allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc or any allocator on the
// path that builds a histogram: an engine that hands the library a fixed
// memory budget and forbids it to grow, a real-time loop that must not
// stall on the allocator, or code that runs where allocation is not allowed.
// The regular entry point takes its int64 accumulators from the
// stream-ordered pool; this one uses a fixed block of device memory that is
// part of the library image instead.  Its limits:
//   * the block is WGB_NOALLOC_SCRATCH_BYTES (64 MiB); every GPU on which the
//     library's kernels are loaded keeps it reserved until the process exits;
//   * a call needs num_eras * k * (num_bins + 1) * 16 bytes of histogram
//     cells plus F_master * 4 + ceil(n / 2048) * 16 + 96 bytes, each part
//     rounded up to 256 bytes; larger calls are rejected with WGB_ERR_ARG
//     before any work is queued;
//   * all calls share the block: two calls that can overlap on the GPU (on
//     different streams, or on the same device from different threads
//     without ordering) race on it.  Calls issued on one stream are ordered
//     and safe; every call clears the cells it uses before it starts.
//   * the first call on a device resolves the block's device address with
//     cudaGetSymbolAddress (once per device, with that device current);
//     make that first call before capturing a stream.
#include <mutex>

namespace wgb {

constexpr size_t WGB_NOALLOC_SCRATCH_BYTES = 64ull << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[WGB_NOALLOC_SCRATCH_BYTES];

struct NoallocAddr {
    static constexpr int MAXDEV = 64;
    void *ptr[MAXDEV] = {};
    std::mutex m;
};
static NoallocAddr g_noalloc_addr;

static inline size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace wgb

using namespace wgb;

extern "C" int wgb_compute_histogram3_noalloc(const int8_t *bin_indices, int64_t num_rows, int64_t F_master,
                                              const float *residuals, const int32_t *sample_indices, int64_t n,
                                              const int32_t *feature_indices, int32_t k,
                                              const int32_t *era_indices, float *grad_hist, float *hess_hist,
                                              int32_t num_eras, int32_t num_bins, int32_t threads_per_block,
                                              int32_t rows_per_thread, void *stream) {
    WGB_CHECK_ARG(threads_per_block > 0 && threads_per_block % 32 == 0,
                  "threads_per_block should be a positive multiple of 32");
    WGB_CHECK_ARG(rows_per_thread >= 1 && rows_per_thread <= 16, "rows_per_thread must be in [1, 16]");
    WGB_CHECK_ARG(num_bins >= 2 && num_bins <= 127, "num_bins must be in [2, 127]");
    WGB_CHECK_ARG(num_eras >= 1 && k >= 0 && n >= 0 && num_rows >= 0 && F_master >= 1, "bad sizes");
    WGB_CHECK_ARG(n < (1ll << 31), "too many samples");
    if (n == 0 || k == 0) return WGB_OK;

    // carve the fixed block: cells, counts, kpos, chunk list, scalars, node
    const long long se = (long long)num_eras * k * (num_bins + 1);
    const int nchunk = (int)((n + HIST_R - 1) / HIST_R);
    const size_t off_hc = round256((size_t)se * 8);
    const size_t off_kpos = off_hc + round256((size_t)se * 8);
    const size_t off_chunks = off_kpos + round256((size_t)F_master * 4);
    const size_t off_small = off_chunks + round256((size_t)nchunk * sizeof(int4));
    const size_t off_nd = off_small + 256;
    const size_t need = off_nd + round256(sizeof(wgb_node));
    WGB_CHECK_ARG(need <= WGB_NOALLOC_SCRATCH_BYTES,
                  "wgb_compute_histogram3_noalloc needs %zu bytes of scratch (num_eras*k*(num_bins+1) = %lld "
                  "cells); its fixed block holds %zu bytes -- use wgb_compute_histogram3",
                  need, se, (size_t)WGB_NOALLOC_SCRATCH_BYTES);

    int dev;
    WGB_CUDA(cudaGetDevice(&dev));
    WGB_CHECK_ARG(dev >= 0 && dev < NoallocAddr::MAXDEV, "device index %d out of range", dev);
    unsigned char *base;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_addr.m);
        if (!g_noalloc_addr.ptr[dev]) {
            void *p = nullptr;
            WGB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));  // the device is current here
            g_noalloc_addr.ptr[dev] = p;
        }
        base = static_cast<unsigned char *>(g_noalloc_addr.ptr[dev]);
    }
    long long *hg = reinterpret_cast<long long *>(base);
    long long *hc = reinterpret_cast<long long *>(base + off_hc);
    int *kpos = reinterpret_cast<int *>(base + off_kpos);
    int4 *chunks = reinterpret_cast<int4 *>(base + off_chunks);
    int *small = reinterpret_cast<int *>(base + off_small);
    wgb_node *nd = reinterpret_cast<wgb_node *>(base + off_nd);
    int *nchunks = small, *shift = small + 1, *nn = small + 2;
    float *maxabs = reinterpret_cast<float *>(small + 3);

    cudaStream_t st = as_stream(stream);
    // the block keeps the previous call's contents: clear what must start at 0
    WGB_CUDA(cudaMemsetAsync(hg, 0, sizeof(long long) * se, st));
    WGB_CUDA(cudaMemsetAsync(hc, 0, sizeof(long long) * se, st));
    WGB_CUDA(cudaMemsetAsync(kpos, 0xff, sizeof(int) * F_master, st));
    WGB_CUDA(cudaMemsetAsync(small, 0, 256, st));
    k_kpos<<<(k + 255) / 256, 256, 0, st>>>(feature_indices, k, (int)F_master, kpos);
    k_max_abs_rows<<<grid_cap(n, 256), 256, 0, st>>>(residuals, sample_indices, n, num_rows, maxabs);
    k_single_node<<<1, 1, 0, st>>>(maxabs, shift, nd, (int)n, nn);
    k_chunk_plan<<<1, 1024, 0, st>>>(nd, nn, chunks, nchunks, nchunk, 0);
    WGB_LAUNCHED("wgb_compute_histogram3_noalloc setup");
    cudaError_t le = launch_hist(nchunk, bin_indices, F_master, (int)F_master, sample_indices, nullptr, residuals,
                                 shift, num_eras > 1 ? era_indices : nullptr, kpos, k, num_eras, num_bins, 0, false,
                                 chunks, nchunks, nd, HistOut{hg, hc, se, 0, k, 0}, num_rows, st);
    if (le != cudaSuccess) {
        set_error("k_hist launch failed: %s", cudaGetErrorString(le));
        return WGB_ERR_CUDA;
    }
    k_hist_to_float<<<grid_cap((long long)num_eras * k * num_bins, 256), 256, 0, st>>>(
        hg, hc, (long long)num_eras * k, num_bins, shift, grad_hist, hess_hist);
    WGB_LAUNCHED("k_hist_to_float");
    return WGB_OK;
}
