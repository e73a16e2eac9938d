// gemm_api.cu -- the C ABI of libjstorch_gemm.so (declared in
// include/jstorch_gemm.h): argument validation, kernel selection, workspace,
// status reporting, the reference-compatible launchers and the host-array
// torch.matmul entry point.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "gemm_internal.h"

namespace jst {

// ---------------------------------------------------------------- status
static thread_local int t_status = JST_OK;
static thread_local char t_msg[256] = "";

int set_status(int status, const char* msg) {
    t_status = status;
    if (status != JST_OK) {
        std::snprintf(t_msg, sizeof(t_msg), "%s", msg ? msg : "");
    }
    return status;
}

static int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return JST_OK;
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    return set_status(e == cudaErrorMemoryAllocation ? JST_ERR_NOMEM : JST_ERR_CUDA, buf);
}

// ---------------------------------------------------------------- devices
struct DeviceState {
    bool init = false;
    bool ok = false;
    uint32_t* err_word = nullptr;
    cudaMemPool_t pool = nullptr;
};
static std::mutex g_dev_mu;
static DeviceState g_dev[64];

// Validates that the current device is a compute-capability 10.x part and
// sets up its error word and workspace pool once.
static int current_device(int* out_dev) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return set_status(JST_ERR_NO_DEVICE, "no CUDA device available");
    }
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceState& st = g_dev[dev];
    if (!st.init) {
        st.init = true;
        int major = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        if (major != 10) {
            cudaGetLastError();
            return set_status(JST_ERR_NO_DEVICE, "libjstorch_gemm is built for sm_100a (B200) only");
        }
        if (cudaMalloc(&st.err_word, sizeof(uint32_t)) != cudaSuccess ||
            cudaMemset(st.err_word, 0, sizeof(uint32_t)) != cudaSuccess) {
            cudaGetLastError();
            return set_status(JST_ERR_NOMEM, "cannot allocate the device error word");
        }
        cudaMemPoolProps props;
        std::memset(&props, 0, sizeof(props));
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        if (cudaMemPoolCreate(&st.pool, &props) != cudaSuccess) {
            cudaGetLastError();
            return set_status(JST_ERR_CUDA, "cudaMemPoolCreate failed");
        }
        uint64_t keep = ~0ull;  // cache freed workspace inside the pool
        cudaMemPoolSetAttribute(st.pool, cudaMemPoolAttrReleaseThreshold, &keep);
        st.ok = true;
    }
    if (!st.ok) return set_status(JST_ERR_NO_DEVICE, "device unusable by libjstorch_gemm (see first error)");
    *out_dev = dev;
    return JST_OK;
}

uint32_t* device_error_word() {
    int dev = 0;
    cudaGetDevice(&dev);
    return (dev >= 0 && dev < 64) ? g_dev[dev].err_word : nullptr;
}

// ---------------------------------------------------------------- dispatch
static bool use_tc(const GemmArgs& a) {
    // The split pass costs one read of each operand plus two plane writes, and
    // the tensor-core kernel needs many 128 x 256 tiles to fill 148 SMs.
    // Measured on B200 (fp32 in / out): FFMA is as fast or faster up to about
    // 2^28 multiply-adds (512^3, the nn.Linear layers of the MLP config); the
    // tensor-core kernel wins from 2^30 (64 x 512x512x64 batched, 2048^3 and up).
    const double macs = (double)a.M * a.N * a.K * a.batch;
    if (a.K < 32) return false;
    if (a.M >= 64 && a.N >= 64) return macs >= 1073741824.0;
    // A narrow side of 16..63 pads the tensor-core tile (128 rows, 64 columns
    // at least) to a quarter or half full, but the FFMA kernel's tiles are
    // padded as well and its peak is a quarter of the 3xTF32 rate, so large
    // products still belong on the tensor cores (a 3x3 convolution with 32
    // output channels, M = 32 over 32 x 3136 x 2304: FFMA 7.9 TFLOP/s).
    return a.M >= 16 && a.N >= 16 && macs >= 4294967296.0;
}

static int validate(const jst_gemm_desc* d, GemmArgs* a) {
    if (!d) return set_status(JST_ERR_ARG, "null descriptor");
    if (d->M < 0 || d->N < 0 || d->K < 0) return set_status(JST_ERR_ARG, "negative dimension");
    if (d->batch < 1) return set_status(JST_ERR_ARG, "batch must be >= 1");
    if (d->transA != 0 && d->transA != 1) return set_status(JST_ERR_ARG, "transA must be 0 or 1");
    if (d->transB != 0 && d->transB != 1) return set_status(JST_ERR_ARG, "transB must be 0 or 1");
    const int e = d->epilogue;
    if (!(e >= JST_EPI_NONE && e <= JST_EPI_MASK) && e != JST_EPI_BIAS_ROW && e != JST_EPI_BIAS_ROW_RELU)
        return set_status(JST_ERR_ARG, "unknown epilogue");
    if (d->epilogue == JST_EPI_MASK && (!d->aux || d->ld_aux < d->N || (d->batch > 1 && d->stride_aux < 0)))
        return set_status(JST_ERR_ARG, "mask epilogue needs aux with ld_aux >= N");
    if (d->kernel < JST_KERNEL_AUTO || d->kernel > JST_KERNEL_FFMA) return set_status(JST_ERR_ARG, "unknown kernel");
    const bool row_bias = e == JST_EPI_BIAS_ROW || e == JST_EPI_BIAS_ROW_RELU;
    const bool has_bias = e == JST_EPI_BIAS || e == JST_EPI_BIAS_RELU || row_bias;
    if (has_bias && !d->bias) return set_status(JST_ERR_ARG, "bias epilogue without a bias pointer");
    const int64_t a_rows = d->transA ? d->K : d->M, a_cols = d->transA ? d->M : d->K;
    const int64_t b_rows = d->transB ? d->N : d->K, b_cols = d->transB ? d->K : d->N;
    if (d->M > 0 && d->N > 0) {
        if (!d->C) return set_status(JST_ERR_ARG, "null C");
        if (d->ldc < d->N) return set_status(JST_ERR_ARG, "ldc < N");
        if (d->batch > 1 && d->strideC < (int64_t)(d->M - 1) * d->ldc + d->N)
            return set_status(JST_ERR_ARG, "strideC overlaps batches of C");
        if (d->K > 0) {
            if (!d->A || !d->B) return set_status(JST_ERR_ARG, "null A or B");
            if (d->lda < std::max<int64_t>(a_cols, 1)) return set_status(JST_ERR_ARG, "lda too small");
            if (d->ldb < std::max<int64_t>(b_cols, 1)) return set_status(JST_ERR_ARG, "ldb too small");
            if (d->strideA < 0 || d->strideB < 0) return set_status(JST_ERR_ARG, "negative batch stride");
            (void)a_rows; (void)b_rows;
        }
    }
    a->transA = d->transA; a->transB = d->transB;
    a->M = d->M; a->N = d->N; a->K = d->K; a->batch = d->batch;
    a->A = d->A; a->lda = d->lda; a->strideA = d->strideA;
    a->B = d->B; a->ldb = d->ldb; a->strideB = d->strideB;
    a->C = d->C; a->ldc = d->ldc; a->strideC = d->strideC;
    a->bias = has_bias ? d->bias : nullptr;
    a->bias_row = row_bias ? 1 : 0;
    a->relu = (e == JST_EPI_RELU || e == JST_EPI_BIAS_RELU || e == JST_EPI_BIAS_ROW_RELU) ? 1 : 0;
    a->aux = d->epilogue == JST_EPI_MASK ? d->aux : nullptr;
    a->ld_aux = d->ld_aux;
    a->stride_aux = d->stride_aux;
    return JST_OK;
}

int validate_gemm_desc(const jst_gemm_desc* d, GemmArgs* a) { return validate(d, a); }

int workspace_alloc(size_t bytes, cudaStream_t s, void** out) {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    if (!bytes) bytes = 16;
    // Inside a stream capture the allocation becomes a graph memory node of the
    // graph's own pool; outside, it comes from this library's pool.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    rc = cuda_status(cudaStreamIsCapturing(s, &cs), "capture query");
    if (rc) return rc;
    if (cs == cudaStreamCaptureStatusActive) return cuda_status(cudaMallocAsync(out, bytes, s), "workspace allocation");
    return cuda_status(cudaMallocFromPoolAsync(out, bytes, g_dev[dev].pool, s), "workspace allocation");
}

int workspace_free(void* p, cudaStream_t s) { return cuda_status(cudaFreeAsync(p, s), "workspace release"); }

static int gemm(const jst_gemm_desc* d) {
    GemmArgs a;
    int rc = validate(d, &a);
    if (rc) return rc;
    int dev = 0;
    rc = current_device(&dev);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(d->stream);
    if (a.M == 0 || a.N == 0) return set_status(JST_OK, nullptr);
    if (a.K == 0) {
        rc = fill_epilogue_run(a, s);
        return rc ? rc : set_status(JST_OK, nullptr);
    }
    const int k = d->kernel == JST_KERNEL_AUTO ? (use_tc(a) ? JST_KERNEL_TC3XTF32 : JST_KERNEL_FFMA) : d->kernel;
    if (k == JST_KERNEL_FFMA) {
        rc = ffma_gemm_run(a, s);
        return rc ? rc : set_status(JST_OK, nullptr);
    }
    // tensor-core path: stream-ordered workspace from this library's pool
    const size_t bytes = tc_workspace_bytes(a);
    void* ws = nullptr;
    rc = workspace_alloc(bytes, s, &ws);
    if (rc) return rc;
    rc = tc_gemm_run(a, ws, s);
    const int frc = workspace_free(ws, s);
    if (rc) return rc;
    rc = frc;
    return rc ? rc : set_status(JST_OK, nullptr);
}

// ---------------------------------------------------------------- host staging
struct HostStage {
    std::mutex mu;
    int dev = -1;
    cudaStream_t stream = nullptr;  // compute stream of synchronous calls
    cudaStream_t h2d = nullptr;     // copy streams of the pipelined path
    cudaStream_t d2h = nullptr;
    std::vector<cudaEvent_t> ev;
    float* d_buf = nullptr;  // A | B | C
    size_t d_cap = 0;        // floats
    // Recorded on the caller's stream when a call's last use of d_buf is
    // enqueued; the next call's stream waits for it, so calls on different
    // streams take turns on the staging buffer instead of racing on it.
    cudaEvent_t released = nullptr;
    bool released_recorded = false;
};
static HostStage g_host[64];

// Large host-array products: C is cut into a grid of blocks (about 4 x 4,
// at least 1024 x 1024), A into the matching row blocks and B into column
// panels.  The host->device copies alternate between A blocks and B panels
// (proportionally), each block's GEMM starts as soon as its row block and its
// panel are on the device, and each C block goes back to the host as soon as
// it is done -- so compute starts after about a quarter of each operand has
// arrived and the device->host traffic runs under the host->device traffic
// instead of after it.  B panels and C blocks move as pitched 2-D copies.
// All three streams are ordered after the caller's earlier work on st, and st
// is ordered after the last C block has reached the host buffer.
static int host_matmul_pipelined(HostStage& h, const float* a, const float* b, float* c, int M, int K, int N,
                                 float* dA, float* dB, float* dC, cudaStream_t st) {
    int rc;
    if (!h.h2d) {
        rc = cuda_status(cudaStreamCreateWithFlags(&h.h2d, cudaStreamNonBlocking), "stream create");
        if (rc) return rc;
        rc = cuda_status(cudaStreamCreateWithFlags(&h.d2h, cudaStreamNonBlocking), "stream create");
        if (rc) return rc;
    }
    const int64_t Kp = (K + 3) & ~3;
    auto split_dim = [](int n, int align) {
        int64_t blk = std::max<int64_t>(1024, ((int64_t)(n + 3) / 4 + align - 1) / align * align);
        std::vector<std::pair<int, int>> v;  // (start, extent)
        for (int64_t x = 0; x < n; x += blk) v.push_back({(int)x, (int)std::min<int64_t>(blk, n - x)});
        return v;
    };
    const auto rb = split_dim(M, 128), cb = split_dim(N, 256);
    const int gr = (int)rb.size(), gc = (int)cb.size();
    const size_t nev = 3 + (size_t)gr + gc + (size_t)gr * gc;
    while (h.ev.size() < nev) {
        cudaEvent_t e;
        rc = cuda_status(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event create");
        if (rc) return rc;
        h.ev.push_back(e);
    }
    cudaEvent_t ev_entry = h.ev[0], ev_done = h.ev[2];
    auto ev_a = [&](int i) { return h.ev[3 + i]; };
    auto ev_b = [&](int j) { return h.ev[3 + gr + j]; };
    auto ev_c = [&](int i, int j) { return h.ev[3 + gr + gc + (size_t)i * gc + j]; };
    const size_t a_plane = (size_t)M * Kp, b_plane = (size_t)N * Kp;
    void* ws = nullptr;
    rc = workspace_alloc((2 * a_plane + 2 * b_plane) * sizeof(float), st, &ws);
    if (rc) return rc;
    float* a_hi = static_cast<float*>(ws);
    float* a_lo = a_hi + a_plane;
    float* b_hi = a_lo + a_plane;
    float* b_lo = b_hi + b_plane;
    uint32_t* err = device_error_word();
    const size_t pitch = (size_t)N * sizeof(float);

    rc = cuda_status(cudaEventRecord(ev_entry, st), "event record");
    if (!rc) rc = cuda_status(cudaStreamWaitEvent(h.h2d, ev_entry, 0), "stream wait");
    if (!rc) rc = cuda_status(cudaStreamWaitEvent(h.d2h, ev_entry, 0), "stream wait");
    // enqueue order of the host->device copies (A block i or B panel j), proportional
    std::vector<std::pair<char, int>> loads;
    for (int ia = 0, ib = 0; ia < gr || ib < gc;) {
        if (ib >= gc || (ia < gr && (int64_t)ia * gc <= (int64_t)ib * gr)) loads.push_back({'A', ia++});
        else loads.push_back({'B', ib++});
    }
    // inputs and compute first: with pageable host memory each H2D copy blocks
    // the host, and the C copies must not be queued ahead of them
    std::vector<std::pair<int, int>> order;  // blocks that just became computable
    std::vector<std::pair<int, int>> done;   // blocks in compute order
    int na = 0, nb = 0;
    for (size_t l = 0; l < loads.size() && !rc; ++l) {
        if (loads[l].first == 'A') {
            const int i = loads[l].second;
            const int r0 = rb[i].first, rows = rb[i].second;
            rc = cuda_status(cudaMemcpyAsync(dA + (int64_t)r0 * K, a + (int64_t)r0 * K, (size_t)rows * K * sizeof(float),
                                             cudaMemcpyHostToDevice, h.h2d), "H2D A block");
            if (!rc) rc = cuda_status(cudaEventRecord(ev_a(i), h.h2d), "event record");
            if (!rc) rc = cuda_status(cudaStreamWaitEvent(st, ev_a(i), 0), "stream wait");
            if (!rc) rc = tc_split(dA + (int64_t)r0 * K, 1, K, 0, rows, K, 1, a_hi + r0 * Kp, a_lo + r0 * Kp, st);
            ++na;
            for (int j = 0; j < nb && !rc; ++j) order.push_back({i, j});
        } else {
            const int j = loads[l].second;
            const int c0 = cb[j].first, cols = cb[j].second;
            rc = cuda_status(cudaMemcpy2DAsync(dB + c0, pitch, b + c0, pitch, (size_t)cols * sizeof(float), K,
                                               cudaMemcpyHostToDevice, h.h2d), "H2D B panel");
            if (!rc) rc = cuda_status(cudaEventRecord(ev_b(j), h.h2d), "event record");
            if (!rc) rc = cuda_status(cudaStreamWaitEvent(st, ev_b(j), 0), "stream wait");
            if (!rc) rc = tc_split(dB + c0, 0, N, 0, cols, K, 1, b_hi + c0 * Kp, b_lo + c0 * Kp, st);
            ++nb;
            for (int i = 0; i < na && !rc; ++i) order.push_back({i, j});
        }
        // the blocks that just became computable
        while (!rc && !order.empty()) {
            const int i = order.front().first, j = order.front().second;
            order.erase(order.begin());
            const int r0 = rb[i].first, rows = rb[i].second, c0 = cb[j].first, cols = cb[j].second;
            rc = tc_gemm_planes(a_hi + r0 * Kp, a_lo + r0 * Kp, b_hi + c0 * Kp, b_lo + c0 * Kp, rows, cols, K, 1,
                                dC + (int64_t)r0 * N + c0, N, 0, nullptr, 0, err, st);
            if (!rc) rc = cuda_status(cudaEventRecord(ev_c(i, j), st), "event record");
            if (rc) break;
            done.push_back({i, j});
        }
    }
    for (size_t q = 0; q < done.size() && !rc; ++q) {
        const int i = done[q].first, j = done[q].second;
        const int r0 = rb[i].first, rows = rb[i].second, c0 = cb[j].first, cols = cb[j].second;
        rc = cuda_status(cudaStreamWaitEvent(h.d2h, ev_c(i, j), 0), "stream wait");
        if (!rc)
            rc = cuda_status(cudaMemcpy2DAsync(c + (int64_t)r0 * N + c0, pitch, dC + (int64_t)r0 * N + c0, pitch,
                                               (size_t)cols * sizeof(float), rows, cudaMemcpyDeviceToHost, h.d2h),
                             "D2H C block");
    }
    if (!rc) rc = cuda_status(cudaEventRecord(ev_done, h.d2h), "event record");
    if (!rc) rc = cuda_status(cudaStreamWaitEvent(st, ev_done, 0), "stream wait");
    const int frc = workspace_free(ws, st);
    return rc ? rc : frc;
}

// Host-array GEMM: stage a and b to device buffers cached per device, run the
// GEMM, copy C back.  sync: on the library's own stream, waiting for the
// result; otherwise everything is enqueued on `user_stream` (0 = the legacy
// default stream) and the call returns.
static int host_matmul(const float* a, const float* b, float* c, int M, int K, int N, cudaStream_t user_stream,
                       bool sync) {
    if (M < 0 || K < 0 || N < 0) return set_status(JST_ERR_ARG, "negative dimension");
    if ((M > 0 && K > 0 && !a) || (K > 0 && N > 0 && !b) || (M > 0 && N > 0 && !c))
        return set_status(JST_ERR_ARG, "null host pointer");
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    HostStage& h = g_host[dev];
    std::lock_guard<std::mutex> lk(h.mu);
    if (sync && !h.stream) {
        rc = cuda_status(cudaStreamCreateWithFlags(&h.stream, cudaStreamNonBlocking), "stream create");
        if (rc) return rc;
    }
    cudaStream_t st = sync ? h.stream : user_stream;
    jst_stream_t jst_st = reinterpret_cast<jst_stream_t>(st);
    // synchronous calls stage operands of at least 16 MiB through jst_copy_h2d / _d2h (below)
    auto staged = [sync](size_t n) { return sync && n * sizeof(float) >= (size_t(16) << 20); };
    const size_t na = (size_t)M * K, nb = (size_t)K * N, nc = (size_t)M * N;
    // keep each plane 16-byte aligned inside the staging buffer
    auto up4 = [](size_t n) { return (n + 3) & ~size_t(3); };
    const size_t need = up4(na) + up4(nb) + up4(nc);
    if (need > h.d_cap) {
        if (h.d_buf) {
            cudaDeviceSynchronize();  // the old buffer may still be in use on some stream
            cudaFree(h.d_buf);
        }
        h.d_buf = nullptr;
        h.d_cap = 0;
        rc = cuda_status(cudaMalloc(&h.d_buf, std::max<size_t>(need, 4) * sizeof(float)), "device staging");
        if (rc) return rc;
        h.d_cap = need;
    }
    float* dA = h.d_buf;
    float* dB = dA + up4(na);
    float* dC = dB + up4(nb);
    if (!h.released) {
        rc = cuda_status(cudaEventCreateWithFlags(&h.released, cudaEventDisableTiming), "event create");
        if (rc) return rc;
    }
    if (h.released_recorded) {  // the previous call (any stream) is done with the staging buffer first
        rc = cuda_status(cudaStreamWaitEvent(st, h.released, 0), "stream wait");
        if (rc) return rc;
    }
    {
        jst_gemm_desc probe;
        jst_gemm_desc_init(&probe, M, N, K, dA, dB, dC);
        GemmArgs pa{};
        validate(&probe, &pa);
        if (M >= 2048 && K > 0 && N > 0 && use_tc(pa)) {
            rc = host_matmul_pipelined(h, a, b, c, M, K, N, dA, dB, dC, st);
            if (rc) return rc;
            goto done;
        }
    }
    // Synchronous calls move large operands through the pinned double-buffered
    // staging of jst_copy_h2d / jst_copy_d2h (pageable host arrays: the host
    // copy of one chunk overlaps the DMA of the other; page-locked: one
    // direct DMA).  Below 16 MiB the driver's own pageable copy is faster
    // (512^3: 0.28 against 0.33 ms per call); the stream-ordered form keeps
    // cudaMemcpyAsync semantics.
    if (na) {
        rc = staged(na) ? jst_copy_h2d(dA, a, na * sizeof(float), jst_st)
                        : cuda_status(cudaMemcpyAsync(dA, a, na * sizeof(float), cudaMemcpyHostToDevice, st), "H2D A");
        if (rc) return rc;
    }
    if (nb) {
        rc = staged(nb) ? jst_copy_h2d(dB, b, nb * sizeof(float), jst_st)
                        : cuda_status(cudaMemcpyAsync(dB, b, nb * sizeof(float), cudaMemcpyHostToDevice, st), "H2D B");
        if (rc) return rc;
    }
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, dA, dB, dC);
    d.stream = jst_st;
    rc = gemm(&d);
    if (rc) return rc;
    if (nc) {
        rc = staged(nc) ? jst_copy_d2h(c, dC, nc * sizeof(float), jst_st)
                        : cuda_status(cudaMemcpyAsync(c, dC, nc * sizeof(float), cudaMemcpyDeviceToHost, st), "D2H C");
        if (rc) return rc;
    }
done:
    rc = cuda_status(cudaEventRecord(h.released, st), "event record");
    if (rc) return rc;
    h.released_recorded = true;
    if (!sync) return set_status(JST_OK, nullptr);
    rc = cuda_status(cudaStreamSynchronize(st), "matmul synchronise");
    if (rc) return rc;
    uint32_t* w = g_dev[dev].err_word;
    uint32_t e = 0;
    if (w && cudaMemcpy(&e, w, sizeof(e), cudaMemcpyDeviceToHost) == cudaSuccess && e != 0) {
        cudaMemset(w, 0, sizeof(uint32_t));
        return set_status(JST_ERR_TIMEOUT, "a GEMM kernel pipeline wait timed out");
    }
    return set_status(JST_OK, nullptr);
}

}  // namespace jst

// ==================================================================== C ABI
extern "C" {

const char* jst_last_error(void) { return jst::t_msg; }
int jst_get_last_status(void) { return jst::t_status; }

void jst_gemm_desc_init(jst_gemm_desc* d, int M, int N, int K, const float* A, const float* B, float* C) {
    if (!d) return;
    std::memset(d, 0, sizeof(*d));
    d->M = M; d->N = N; d->K = K;
    d->A = A; d->lda = K; d->strideA = (int64_t)M * K;
    d->B = B; d->ldb = N; d->strideB = (int64_t)K * N;
    d->C = C; d->ldc = N; d->strideC = (int64_t)M * N;
    d->batch = 1;
    d->epilogue = JST_EPI_NONE;
    d->kernel = JST_KERNEL_AUTO;
    d->stream = nullptr;
}

int jst_gemm_ex(const jst_gemm_desc* d) { return jst::gemm(d); }

int jst_gemm_select_kernel(const jst_gemm_desc* d) {
    jst::GemmArgs a{};
    if (jst::validate(d, &a)) return -1;
    if (d->kernel != JST_KERNEL_AUTO) return d->kernel;
    return jst::use_tc(a) ? JST_KERNEL_TC3XTF32 : JST_KERNEL_FFMA;
}

// native/ops/matmul.cu:28-37 -- row-major NN, beta = 0
void launch_matmul(const float* a, const float* b, float* c, int M, int K, int N, jst_stream_t s) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, a, b, c);
    d.stream = s;
    jst::gemm(&d);
}

// native/ops/matmul.cu:40-50 -- packed strided batch
void launch_bmm(const float* a, const float* b, float* c, int B, int M, int K, int N, jst_stream_t s) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, a, b, c);
    d.batch = B;
    d.stream = s;
    jst::gemm(&d);
}

// native/ops/matmul.cu:54-67 -- out = x * w^T (+ bias), w stored [out_f, in_f]
void launch_linear(const float* x, const float* w, const float* bias, float* out, int B, int in_f, int out_f,
                   jst_stream_t s) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, B, out_f, in_f, x, w, out);
    d.transB = 1;
    d.ldb = in_f;
    d.strideB = (int64_t)out_f * in_f;
    d.bias = bias;
    d.epilogue = bias ? JST_EPI_BIAS : JST_EPI_NONE;
    d.stream = s;
    jst::gemm(&d);
}

int jst_matmul_host(const float* a, const float* b, float* c, int M, int K, int N) {
    return jst::host_matmul(a, b, c, M, K, N, nullptr, true);
}

int jst_matmul_host_async(const float* a, const float* b, float* c, int M, int K, int N, jst_stream_t stream) {
    return jst::host_matmul(a, b, c, M, K, N, reinterpret_cast<cudaStream_t>(stream), false);
}

int jst_device_error(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 0;
    }
    cudaDeviceSynchronize();
    uint32_t e = 0;
    if (jst::g_dev[dev].err_word) {
        cudaMemcpy(&e, jst::g_dev[dev].err_word, sizeof(e), cudaMemcpyDeviceToHost);
        if (e) cudaMemset(jst::g_dev[dev].err_word, 0, sizeof(uint32_t));
    }
    uint32_t en = 0;  // jst_gemm_tc_noalloc keeps its own word
    jst::noalloc_take_error(dev, &en);
    cudaGetLastError();
    return (int)(e | en);
}

int jst_test_set_device_error(int word) {
    int dev = 0;
    if (word == 0) {
        int rc = jst::current_device(&dev);
        if (rc) return rc;
        const uint32_t one = 1;
        if (cudaMemcpy(jst::g_dev[dev].err_word, &one, sizeof(one), cudaMemcpyHostToDevice) != cudaSuccess) {
            cudaGetLastError();
            return jst::set_status(JST_ERR_CUDA, "writing the device error word failed");
        }
        return jst::set_status(JST_OK, nullptr);
    }
    if (word != 1) return jst::set_status(JST_ERR_ARG, "jst_test_set_device_error: word must be 0 or 1");
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return jst::set_status(JST_ERR_NO_DEVICE, "no CUDA device available");
    }
    const int rc = jst::noalloc_set_error(dev, 1);
    return rc ? rc : jst::set_status(JST_OK, nullptr);
}

void jst_release_caches(void) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    for (int i = 0; i < 64; ++i) {
        std::lock_guard<std::mutex> lk(jst::g_host[i].mu);
        if (!jst::g_host[i].d_buf && !jst::g_dev[i].pool) continue;
        cudaSetDevice(i);
        cudaDeviceSynchronize();
        if (jst::g_host[i].d_buf) cudaFree(jst::g_host[i].d_buf);
        jst::g_host[i].d_buf = nullptr;
        jst::g_host[i].d_cap = 0;
        if (jst::g_dev[i].pool) cudaMemPoolTrimTo(jst::g_dev[i].pool, 0);
    }
    cudaSetDevice(cur);
    jst::hostio_release();
}

}  // extern "C"
