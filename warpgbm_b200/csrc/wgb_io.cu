// Pipelined host -> device copy from pageable memory (numpy arrays).
//
// A copy from pageable memory with cudaMemcpyAsync is staged by the driver
// through one small pinned buffer at a fraction of the link bandwidth.  Here
// a persistent pool of host threads copies the source, chunk by chunk, into
// a ring of pinned staging buffers while the DMA engine moves the previous
// chunk to the device with one plain cudaMemcpyAsync per chunk.  Part of the
// ingest path of fit(): the float matrix of the reference's
// preprocess_gpu_data (warpgbm/core.py:487-538) crosses the link once, at
// close to full PCIe bandwidth.
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace wgb {

class CopyPool {
   public:
    static CopyPool &get() {
        static CopyPool pool;
        return pool;
    }

    // memcpy(dst, src, n) split over the worker threads; returns when done.
    void parallel_copy(void *dst, const void *src, size_t n) {
        const size_t nt = workers_.size() + 1;
        const size_t part = (n + nt - 1) / nt;
        {
            std::unique_lock<std::mutex> lk(m_);
            dst_ = static_cast<char *>(dst);
            src_ = static_cast<const char *>(src);
            n_ = n;
            part_ = part;
            pending_ = workers_.size();
            ++gen_;
        }
        cv_.notify_all();
        // the caller takes the last slice
        size_t off = part * (nt - 1);
        if (off < n) memcpy(dst_ + off, src_ + off, n - off);
        std::unique_lock<std::mutex> lk(m_);
        done_cv_.wait(lk, [&] { return pending_ == 0; });
    }

   private:
    CopyPool() {
        unsigned hw = std::thread::hardware_concurrency();
        unsigned nt = hw > 1 ? (hw > 16 ? 16 : hw) : 1;
        for (unsigned i = 0; i + 1 < nt; ++i) workers_.emplace_back([this, i] { run(i); });
    }
    ~CopyPool() {
        {
            std::unique_lock<std::mutex> lk(m_);
            stop_ = true;
            ++gen_;
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
    }
    void run(size_t idx) {
        size_t seen = 0;
        for (;;) {
            char *d;
            const char *s;
            size_t n, part;
            {
                std::unique_lock<std::mutex> lk(m_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                if (stop_) return;
                d = dst_;
                s = src_;
                n = n_;
                part = part_;
            }
            size_t off = part * idx;
            if (off < n) memcpy(d + off, s + off, (off + part <= n ? part : n - off));
            std::unique_lock<std::mutex> lk(m_);
            if (--pending_ == 0) done_cv_.notify_one();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex m_;
    std::condition_variable cv_, done_cv_;
    char *dst_ = nullptr;
    const char *src_ = nullptr;
    size_t n_ = 0, part_ = 0, pending_ = 0, gen_ = 0;
    bool stop_ = false;
};

struct Staging {
    static constexpr int NBUF = 3;
    static constexpr size_t CHUNK = 64ull << 20;
    void *buf[NBUF] = {nullptr, nullptr, nullptr};
    cudaEvent_t ev[NBUF];
    int device = -1;
    std::mutex m;
};

static Staging g_stage;

}  // namespace wgb

using namespace wgb;

extern "C" int wgb_h2d(void *dst, const void *src, int64_t bytes, void *stream) {
    WGB_CHECK_ARG(bytes >= 0, "negative size");
    if (bytes == 0) return WGB_OK;
    WGB_CHECK_ARG(dst && src, "NULL pointer");
    cudaStream_t st = as_stream(stream);
    std::lock_guard<std::mutex> lk(g_stage.m);
    int dev;
    WGB_CUDA(cudaGetDevice(&dev));
    if (g_stage.device != dev) {
        if (g_stage.device >= 0) {
            for (int i = 0; i < Staging::NBUF; ++i) {
                cudaEventSynchronize(g_stage.ev[i]);
                cudaEventDestroy(g_stage.ev[i]);
                cudaFreeHost(g_stage.buf[i]);
                g_stage.buf[i] = nullptr;
            }
            g_stage.device = -1;
        }
        // everything is created into locals and kept only once all of it
        // exists: a failure part way frees what was made and leaves the
        // staging unset, so the next call starts clean
        void *buf[Staging::NBUF] = {nullptr, nullptr, nullptr};
        cudaEvent_t ev[Staging::NBUF] = {nullptr, nullptr, nullptr};
        cudaError_t e = cudaSuccess;
        for (int i = 0; i < Staging::NBUF && e == cudaSuccess; ++i) {
            e = cudaHostAlloc(&buf[i], Staging::CHUNK, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventRecord(ev[i], st);
        }
        if (e != cudaSuccess) {
            for (int i = 0; i < Staging::NBUF; ++i) {
                if (ev[i]) cudaEventDestroy(ev[i]);
                if (buf[i]) cudaFreeHost(buf[i]);
            }
            set_error("pinned staging setup failed: %s", cudaGetErrorString(e));
            return WGB_ERR_CUDA;
        }
        for (int i = 0; i < Staging::NBUF; ++i) {
            g_stage.buf[i] = buf[i];
            g_stage.ev[i] = ev[i];
        }
        g_stage.device = dev;
    }
    CopyPool &pool = CopyPool::get();
    const char *s = static_cast<const char *>(src);
    char *d = static_cast<char *>(dst);
    int64_t off = 0;
    int b = 0;
    while (off < bytes) {
        const size_t n = (size_t)((bytes - off) < (int64_t)Staging::CHUNK ? (bytes - off) : Staging::CHUNK);
        WGB_CUDA(cudaEventSynchronize(g_stage.ev[b]));  // the DMA out of this buffer has finished
        pool.parallel_copy(g_stage.buf[b], s + off, n);
        WGB_CUDA(cudaMemcpyAsync(d + off, g_stage.buf[b], n, cudaMemcpyHostToDevice, st));
        WGB_CUDA(cudaEventRecord(g_stage.ev[b], st));
        off += (int64_t)n;
        b = (b + 1) % Staging::NBUF;
    }
    return WGB_OK;
}
