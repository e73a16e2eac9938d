// profile.cu -- launch counting and optional CUDA-event timing of every kernel
// this library launches (the reference has no tracing at all).
//
// When enabled, each launch site records one event before and one after its
// kernel on the kernel's own stream; jst_profile_read() waits for them and
// returns per-kernel launch counts and summed device time.  Disabled, a launch
// costs one relaxed atomic increment.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "gemm_internal.h"

namespace jst {

namespace {
struct Pending {
    int kernel;
    cudaEvent_t ev0, ev1;
};
struct Stat {
    int64_t launches = 0;
    double total_ms = 0.0;
};
std::atomic<int64_t> g_launches{0};
std::atomic<int> g_enabled{0};
std::mutex g_mu;
std::vector<Pending> g_pending;
std::vector<cudaEvent_t> g_free_events;
Stat g_stats[KERNEL_ID_COUNT];

const char* kKernelNames[KERNEL_ID_COUNT] = {"tc_gemm", "split_rows", "split_transpose", "ffma_gemm",
                                             "fill_epilogue", "conv_im2col", "splitk_reduce", "gru_gate"};

cudaEvent_t take_event() {
    if (!g_free_events.empty()) {
        cudaEvent_t e = g_free_events.back();
        g_free_events.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}
}  // namespace

ProfScope::ProfScope(cudaStream_t s, int kernel) : s_(s), kernel_(kernel) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (!g_enabled.load(std::memory_order_relaxed)) return;
    // launches being captured into a CUDA graph are not timed (their events
    // would become graph nodes)
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    ev0_ = take_event();
    ev1_ = take_event();
    if (ev0_) cudaEventRecord(static_cast<cudaEvent_t>(ev0_), s_);
}

ProfScope::~ProfScope() {
    if (!ev0_ || !ev1_) return;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaEventRecord(static_cast<cudaEvent_t>(ev1_), s_);
    g_pending.push_back({kernel_, static_cast<cudaEvent_t>(ev0_), static_cast<cudaEvent_t>(ev1_)});
}

}  // namespace jst

extern "C" {

int64_t jst_launch_count(void) { return jst::g_launches.load(); }

int jst_profile_enable(int on) {
    std::lock_guard<std::mutex> lk(jst::g_mu);
    for (auto& p : jst::g_pending) {
        jst::g_free_events.push_back(p.ev0);
        jst::g_free_events.push_back(p.ev1);
    }
    jst::g_pending.clear();
    for (auto& s : jst::g_stats) s = jst::Stat{};
    jst::g_enabled.store(on ? 1 : 0);
    return JST_OK;
}

int jst_profile_read(jst_kernel_stat* out, int max_entries) {
    std::lock_guard<std::mutex> lk(jst::g_mu);
    int rc = JST_OK;
    for (auto& p : jst::g_pending) {
        float ms = 0.f;
        if (cudaEventSynchronize(p.ev1) != cudaSuccess || cudaEventElapsedTime(&ms, p.ev0, p.ev1) != cudaSuccess) {
            cudaGetLastError();
            rc = JST_ERR_CUDA;
        }
        jst::g_stats[p.kernel].launches += 1;
        jst::g_stats[p.kernel].total_ms += ms;
        jst::g_free_events.push_back(p.ev0);
        jst::g_free_events.push_back(p.ev1);
    }
    jst::g_pending.clear();
    int n = 0;
    for (int k = 0; k < jst::KERNEL_ID_COUNT; ++k) {
        if (jst::g_stats[k].launches == 0) continue;
        if (out && n < max_entries) {
            std::memset(&out[n], 0, sizeof(out[n]));
            std::strncpy(out[n].name, jst::kKernelNames[k], sizeof(out[n].name) - 1);
            out[n].launches = jst::g_stats[k].launches;
            out[n].total_ms = jst::g_stats[k].total_ms;
        }
        ++n;
    }
    if (rc != JST_OK) return -rc;
    return n;
}

}  // extern "C"
