// hostio.cpp -- pinned, double-buffered host <-> device copies (see hostio.h).
#include "hostio.h"

#include <algorithm>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <unistd.h>

namespace jst {
namespace core {

namespace {

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
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
    if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("hostio: device index out of range");
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

void h2d(float* dst, const float* src, int64_t count, cudaStream_t s) {
    if (count <= 0) return;
    const size_t bytes = (size_t)count * sizeof(float);
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

void d2h(float* dst, const float* src, int64_t count, cudaStream_t s) {
    if (count <= 0) return;
    const size_t bytes = (size_t)count * sizeof(float);
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

void hostio_release() {
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

}  // namespace core
}  // namespace jst
