// hostio.cu -- jst_copy_h2d / jst_copy_d2h: host <-> device copies through
// pinned, double-buffered staging (include/jstorch_gemm.h).
//
// Reference: Tensor::from_array / from_buffer (native/core/tensor.cpp:740-750)
// is a synchronous cudaMemcpy from the JS heap (pageable), and to_array
// (:775-800) synchronises the whole device, copies synchronously, and then
// napi.cpp:17-30 builds nested JS arrays element by element.
//
// Here, per device, two pinned staging chunks alternate: the host copy of
// chunk i+1 (pageable -> pinned, split over a few worker threads) runs while
// the DMA of chunk i is in flight.
//   * h2d returns once the source has been read; the last DMAs may still be
//     running on the stream (they read only the staging chunks), so the data
//     is ready in stream order, not at return;
//   * d2h waits for its stream only (not the whole device) and returns when
//     the destination holds the data;
//   * a source or destination that is already page-locked is copied by one
//     direct DMA.
#include <cuda_runtime.h>
#include <unistd.h>

#include <algorithm>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "gemm_internal.h"

namespace jst {
namespace io {

namespace {

constexpr size_t kStageChunkBytes = 8u << 20;  // per staging chunk

// CUDA error -> exception inside this file; the C entry points turn it into a status.
struct CudaFail {
    const char* what;
    cudaError_t err;
};

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw CudaFail{what, e};
    }
}

struct Stage {
    std::mutex mu;
    float* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool used[2] = {false, false};  // ev[i] has been recorded since the buffer was last free
};

constexpr int kMaxDevices = 64;
Stage g_stage[kMaxDevices];

Stage& stage_for_current_device() {
    int dev = 0;
    ck(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) throw CudaFail{"device index out of range", cudaErrorInvalidDevice};
    return g_stage[dev];
}

void ensure(Stage& st) {
    for (int i = 0; i < 2; ++i) {
        if (!st.buf[i]) ck(cudaMallocHost(reinterpret_cast<void**>(&st.buf[i]), kStageChunkBytes), "pinned staging");
        if (!st.ev[i]) ck(cudaEventCreateWithFlags(&st.ev[i], cudaEventDisableTiming), "event create");
    }
}

// Wait until the DMA that last used staging chunk i is done.
void drain(Stage& st, int i) {
    if (st.used[i]) {
        ck(cudaEventSynchronize(st.ev[i]), "staging wait");
        st.used[i] = false;
    }
}

bool is_pinned(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

// Below this size the driver's own staging of a pageable copy is as fast.
constexpr size_t kDirectBytes = 256u << 10;

// Persistent workers for the pageable <-> pinned memcpy: one thread copies
// about 10 GB/s, a PCIe 5 x16 DMA runs several times that, and a fresh
// destination also takes its first-touch page faults inside the copy.
class CopyPool {
  public:
    CopyPool() : pid_(getpid()) {
        const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
        nworkers_ = (int)std::min(7u, hw > 2 ? hw / 2 - 1 : 0u);
        for (int i = 0; i < nworkers_; ++i) threads_.emplace_back([this, i] { loop(i); });
    }
    ~CopyPool() {
        {
            std::lock_guard<std::mutex> lk(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }
    // memcpy(dst, src, n) split over the workers and the calling thread
    void copy(void* dst, const void* src, size_t n) {
        constexpr size_t kMinPart = 1u << 20;
        const int parts = (int)std::min<size_t>((size_t)nworkers_ + 1, std::max<size_t>(1, n / kMinPart));
        if (parts <= 1 || getpid() != pid_) {  // a forked child has no workers
            std::memcpy(dst, src, n);
            return;
        }
        std::unique_lock<std::mutex> call(call_mu_);  // one split copy at a time
        {
            std::lock_guard<std::mutex> lk(mu_);
            dst_ = static_cast<char*>(dst);
            src_ = static_cast<const char*>(src);
            n_ = n;
            parts_ = parts;
            pending_ = parts - 1;
            ++gen_;
        }
        cv_.notify_all();
        part(0);
        std::unique_lock<std::mutex> lk(mu_);
        done_cv_.wait(lk, [this] { return pending_ == 0; });
    }

  private:
    void part(int k) {
        const size_t per = (n_ / parts_ + 63) & ~size_t(63);
        const size_t off = std::min(n_, per * (size_t)k);
        const size_t end = k == parts_ - 1 ? n_ : std::min(n_, off + per);
        if (end > off) std::memcpy(dst_ + off, src_ + off, end - off);
    }
    void loop(int i) {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lk(mu_);
            cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
            if (stop_) return;
            seen = gen_;
            const int k = i + 1;
            if (k >= parts_) continue;
            lk.unlock();
            part(k);
            lk.lock();
            if (--pending_ == 0) done_cv_.notify_one();
        }
    }

    pid_t pid_;
    int nworkers_ = 0;
    std::vector<std::thread> threads_;
    std::mutex mu_, call_mu_;
    std::condition_variable cv_, done_cv_;
    bool stop_ = false;
    uint64_t gen_ = 0;
    char* dst_ = nullptr;
    const char* src_ = nullptr;
    size_t n_ = 0;
    int parts_ = 1, pending_ = 0;
};

CopyPool& copy_pool() {
    static CopyPool pool;
    return pool;
}

}  // namespace

void h2d(void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return;
    if (is_pinned(src)) {
        // Direct DMA; wait for it, because the caller may reuse its buffer on return.
        ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "H2D copy");
        ck(cudaStreamSynchronize(s), "H2D wait");
        return;
    }
    if (bytes <= kDirectBytes) {
        ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "H2D copy");
        return;
    }
    Stage& st = stage_for_current_device();
    std::lock_guard<std::mutex> lk(st.mu);
    ensure(st);
    const char* from = reinterpret_cast<const char*>(src);
    char* to = reinterpret_cast<char*>(dst);
    int i = 0;
    for (size_t off = 0; off < bytes; off += kStageChunkBytes, i ^= 1) {
        const size_t n = std::min(kStageChunkBytes, bytes - off);
        drain(st, i);
        copy_pool().copy(st.buf[i], from + off, n);
        ck(cudaMemcpyAsync(to + off, st.buf[i], n, cudaMemcpyHostToDevice, s), "H2D copy");
        ck(cudaEventRecord(st.ev[i], s), "event record");
        st.used[i] = true;
    }
}

void d2h(void* dst, const void* src, size_t bytes, cudaStream_t s) {
    if (bytes == 0) return;
    if (is_pinned(dst) || bytes <= kDirectBytes) {
        ck(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "D2H copy");
        ck(cudaStreamSynchronize(s), "D2H wait");
        return;
    }
    Stage& st = stage_for_current_device();
    std::lock_guard<std::mutex> lk(st.mu);
    ensure(st);
    drain(st, 0);
    drain(st, 1);
    const char* from = reinterpret_cast<const char*>(src);
    char* to = reinterpret_cast<char*>(dst);
    const size_t nchunks = (bytes + kStageChunkBytes - 1) / kStageChunkBytes;
    auto issue = [&](size_t c) {
        const size_t off = c * kStageChunkBytes;
        const size_t n = std::min(kStageChunkBytes, bytes - off);
        const int b = (int)(c & 1);
        ck(cudaMemcpyAsync(st.buf[b], from + off, n, cudaMemcpyDeviceToHost, s), "D2H copy");
        ck(cudaEventRecord(st.ev[b], s), "event record");
        st.used[b] = true;
    };
    issue(0);
    if (nchunks > 1) issue(1);
    for (size_t c = 0; c < nchunks; ++c) {
        const int b = (int)(c & 1);
        drain(st, b);
        const size_t off = c * kStageChunkBytes;
        copy_pool().copy(to + off, st.buf[b], std::min(kStageChunkBytes, bytes - off));
        if (c + 2 < nchunks) issue(c + 2);
    }
}

void release() {
    for (int d = 0; d < kMaxDevices; ++d) {
        Stage& st = g_stage[d];
        std::lock_guard<std::mutex> lk(st.mu);
        for (int i = 0; i < 2; ++i) {
            if (st.ev[i]) {
                cudaEventSynchronize(st.ev[i]);
                cudaEventDestroy(st.ev[i]);
                st.ev[i] = nullptr;
            }
            if (st.buf[i]) {
                cudaFreeHost(st.buf[i]);
                st.buf[i] = nullptr;
            }
            st.used[i] = false;
        }
    }
}

}  // namespace io

int hostio_release() {
    io::release();
    return JST_OK;
}

}  // namespace jst

extern "C" {

int jst_copy_h2d(void* dst_device, const void* src_host, size_t bytes, jst_stream_t stream) {
    if (bytes && (!dst_device || !src_host)) return jst::set_status(JST_ERR_ARG, "jst_copy_h2d: null pointer");
    try {
        jst::io::h2d(dst_device, src_host, bytes, reinterpret_cast<cudaStream_t>(stream));
    } catch (const jst::io::CudaFail& f) {
        return jst::set_status(f.err == cudaErrorMemoryAllocation ? JST_ERR_NOMEM : JST_ERR_CUDA, f.what);
    }
    return jst::set_status(JST_OK, nullptr);
}

int jst_copy_d2h(void* dst_host, const void* src_device, size_t bytes, jst_stream_t stream) {
    if (bytes && (!dst_host || !src_device)) return jst::set_status(JST_ERR_ARG, "jst_copy_d2h: null pointer");
    try {
        jst::io::d2h(dst_host, src_device, bytes, reinterpret_cast<cudaStream_t>(stream));
    } catch (const jst::io::CudaFail& f) {
        return jst::set_status(f.err == cudaErrorMemoryAllocation ? JST_ERR_NOMEM : JST_ERR_CUDA, f.what);
    }
    return jst::set_status(JST_OK, nullptr);
}

}  // extern "C"
