// dist.cu -- libjstorch_dist.so: row-sharded and batch-sharded GEMMs over
// NCCL, one process per GPU (C ABI in include/jstorch_dist.h).
//
// Row-sharded GEMM (configuration 5 of the benchmark):
//   1. B is broadcast in place from the root (ncclBroadcast, NVLS where NCCL
//      picks it);
//   2. A_local and B are split once into hi / lo TF32 planes;
//   3. for each row block of A_local the tensor-core kernel writes its C rows
//      straight into their global place in C_full; an event hands the block
//      to a communication stream that all-gathers it in place while the next
//      block computes.  With block-cyclic row ownership (block i of rank r is
//      global block i * nranks + r) the blocks of one round are contiguous in
//      C_full, so each round is a single in-place ncclAllGather.
// No kernel reads another GPU's memory; all data moves through NCCL.
//
// Host-side failure handling: the communicator is created non-blocking and
// every NCCL call is polled against a host deadline; on expiry the
// communicator is aborted and JST_ERR_TIMEOUT returned (a peer that died or
// never joined ends the call with an error, not a hang).
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/jstorch_dist.h"
#include "gemm_internal.h"

struct jst_comm {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int nranks = 1;
    int device = 0;
    double timeout_s = 60.0;
    bool broken = false;
    cudaStream_t comm_stream = nullptr;
    std::vector<cudaEvent_t> events;
};

namespace jst {
namespace {

int nccl_error(jst_comm* c, ncclResult_t r, const char* what) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s: %s%s%s", what, ncclGetErrorString(r), c && c->nccl ? " / " : "",
                  c && c->nccl ? ncclGetLastError(c->nccl) : "");
    if (c) c->broken = true;
    return set_status(JST_ERR_NCCL, buf);
}

// Wait (on the host) until the communicator has no operation in progress.
int nccl_settle(jst_comm* c, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return JST_OK;
    if (r != ncclInProgress) return nccl_error(c, r, what);
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (true) {
        if (ncclCommGetAsyncError(c->nccl, &st) != ncclSuccess) return nccl_error(c, st, what);
        if (st != ncclInProgress) break;
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > c->timeout_s) {
            ncclCommAbort(c->nccl);
            c->nccl = nullptr;
            c->broken = true;
            char buf[160];
            std::snprintf(buf, sizeof(buf), "%s: no progress within %.1f s (peer missing?); communicator aborted",
                          what, c->timeout_s);
            return set_status(JST_ERR_TIMEOUT, buf);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
    return st == ncclSuccess ? JST_OK : nccl_error(c, st, what);
}

int ready(jst_comm* c) {
    if (!c) return set_status(JST_ERR_ARG, "null communicator");
    if (c->broken || !c->nccl) return set_status(JST_ERR_NCCL, "communicator is broken (earlier error or timeout)");
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device)
        return set_status(JST_ERR_ARG, "current device differs from the communicator's device");
    return JST_OK;
}

int ensure_events(jst_comm* c, size_t n) {
    while (c->events.size() < n) {
        cudaEvent_t e;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            return set_status(JST_ERR_CUDA, "cudaEventCreate failed");
        }
        c->events.push_back(e);
    }
    return JST_OK;
}

}  // namespace
}  // namespace jst

extern "C" {

int jst_comm_get_unique_id(unsigned char id[JST_COMM_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == JST_COMM_ID_BYTES, "ncclUniqueId size");
    if (!id) return jst::set_status(JST_ERR_ARG, "null id");
    ncclUniqueId u;
    ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return jst::nccl_error(nullptr, r, "ncclGetUniqueId");
    std::memcpy(id, &u, sizeof(u));
    return jst::set_status(JST_OK, nullptr);
}

int jst_comm_init(jst_comm** out, int nranks, int rank, const unsigned char id[JST_COMM_ID_BYTES], double timeout_s) {
    using namespace jst;
    if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks || !(timeout_s > 0))
        return set_status(JST_ERR_ARG, "jst_comm_init: bad argument");
    *out = nullptr;
    auto* c = new jst_comm();
    c->rank = rank;
    c->nranks = nranks;
    c->timeout_s = timeout_s;
    if (cudaGetDevice(&c->device) != cudaSuccess) {
        cudaGetLastError();
        delete c;
        return set_status(JST_ERR_NO_DEVICE, "no CUDA device");
    }
    if (cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        delete c;
        return set_status(JST_ERR_CUDA, "stream create failed");
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, u, rank, &cfg);
    int rc = (c->nccl == nullptr && r != ncclSuccess && r != ncclInProgress) ? nccl_error(c, r, "ncclCommInitRank")
                                                                            : nccl_settle(c, r, "ncclCommInitRank");
    if (rc) {
        if (c->nccl) ncclCommAbort(c->nccl);
        cudaStreamDestroy(c->comm_stream);
        delete c;
        return rc;
    }
    *out = c;
    return set_status(JST_OK, nullptr);
}

int jst_comm_sync(jst_comm* c, jst_stream_t stream) {
    using namespace jst;
    if (!c) return set_status(JST_ERR_ARG, "null communicator");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) {
            cudaGetLastError();
            return set_status(JST_ERR_CUDA, cudaGetErrorString(e));
        }
        if (c->nccl) {
            ncclResult_t st = ncclSuccess;
            if (ncclCommGetAsyncError(c->nccl, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress)
                return nccl_error(c, st, "collective failed");
        }
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > c->timeout_s) {
            if (c->nccl) ncclCommAbort(c->nccl);  // ends collectives still waiting for a peer
            c->nccl = nullptr;
            c->broken = true;
            return set_status(JST_ERR_TIMEOUT, "stream did not complete within the communicator deadline; aborted");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    return set_status(JST_OK, nullptr);
}

int jst_comm_rank(const jst_comm* c) { return c ? c->rank : -1; }
int jst_comm_size(const jst_comm* c) { return c ? c->nranks : -1; }

int jst_comm_destroy(jst_comm* c) {
    using namespace jst;
    if (!c) return set_status(JST_OK, nullptr);
    int rc = JST_OK;
    if (c->nccl) {
        if (c->broken) {
            ncclCommAbort(c->nccl);
        } else {
            cudaStreamSynchronize(c->comm_stream);
            ncclResult_t r = ncclCommFinalize(c->nccl);
            rc = nccl_settle(c, r, "ncclCommFinalize");
            if (c->nccl) {
                if (rc) ncclCommAbort(c->nccl);
                else ncclCommDestroy(c->nccl);
            }
        }
    }
    for (auto e : c->events) cudaEventDestroy(e);
    if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
    delete c;
    return rc ? rc : set_status(JST_OK, nullptr);
}

int jst_gemm_rowsharded(jst_comm* c, const float* A_local, int M_local, int K, float* B, int N, int root,
                        float* C_full, int chunk_rows, jst_stream_t stream) {
    using namespace jst;
    int rc = ready(c);
    if (rc) return rc;
    if (M_local < 0 || K < 1 || N < 1 || root < 0 || root >= c->nranks || chunk_rows < 1 ||
        (M_local % chunk_rows) != 0 || !B || !C_full || (M_local > 0 && !A_local))
        return set_status(JST_ERR_ARG, "jst_gemm_rowsharded: bad argument");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int nchunks = M_local / chunk_rows;
    rc = ensure_events(c, (size_t)nchunks + 1);
    if (rc) return rc;

    // 1. B from the root to every rank, in place, on the compute stream
    rc = nccl_settle(c, ncclBroadcast(B, B, (size_t)K * N, ncclFloat, root, c->nccl, s), "ncclBroadcast(B)");
    if (rc) return rc;
    if (M_local == 0) return set_status(JST_OK, nullptr);

    // 2. split planes of A_local and B, once
    const size_t Kp = (size_t)((K + 3) & ~3);
    const size_t a_plane = (size_t)M_local * Kp, b_plane = (size_t)N * Kp;
    void* ws = nullptr;
    rc = workspace_alloc((2 * a_plane + 2 * b_plane) * sizeof(float), s, &ws);
    if (rc) return rc;
    float* a_hi = static_cast<float*>(ws);
    float* a_lo = a_hi + a_plane;
    float* b_hi = a_lo + a_plane;
    float* b_lo = b_hi + b_plane;
    rc = tc_split(A_local, 1, K, 0, M_local, K, 1, a_hi, a_lo, s);
    if (!rc) rc = tc_split(B, 0, N, 0, N, K, 1, b_hi, b_lo, s);

    // 3. per row block: GEMM into C_full, then its in-place all-gather on the comm stream
    for (int i = 0; i < nchunks && !rc; ++i) {
        const int64_t grow = ((int64_t)i * c->nranks + c->rank) * chunk_rows;  // first global row of the block
        float* cblk = C_full + grow * N;
        rc = tc_gemm_planes(a_hi + (size_t)i * chunk_rows * Kp, a_lo + (size_t)i * chunk_rows * Kp, b_hi, b_lo,
                            chunk_rows, N, K, 1, cblk, N, 0, nullptr, 0, device_error_word(), s);
        if (rc) break;
        if (cudaEventRecord(c->events[i], s) != cudaSuccess || cudaStreamWaitEvent(c->comm_stream, c->events[i], 0) !=
                                                                     cudaSuccess) {
            cudaGetLastError();
            rc = set_status(JST_ERR_CUDA, "event hand-off failed");
            break;
        }
        float* round0 = C_full + (int64_t)i * c->nranks * chunk_rows * N;
        rc = nccl_settle(c, ncclAllGather(cblk, round0, (size_t)chunk_rows * N, ncclFloat, c->nccl, c->comm_stream),
                         "ncclAllGather(C)");
    }
    // the compute stream continues once every all-gather is done
    if (cudaEventRecord(c->events[nchunks], c->comm_stream) != cudaSuccess ||
        cudaStreamWaitEvent(s, c->events[nchunks], 0) != cudaSuccess) {
        cudaGetLastError();
        if (!rc) rc = set_status(JST_ERR_CUDA, "event hand-off failed");
    }
    const int frc = workspace_free(ws, s);
    if (rc) return rc;
    return frc ? frc : set_status(JST_OK, nullptr);
}

int jst_bmm_batchsharded(jst_comm* c, const float* A_local, const float* B_local, int batch_local, int M, int K,
                         int N, float* C_full, jst_stream_t stream) {
    using namespace jst;
    int rc = ready(c);
    if (rc) return rc;
    if (batch_local < 1 || M < 0 || K < 0 || N < 0 || !C_full)
        return set_status(JST_ERR_ARG, "jst_bmm_batchsharded: bad argument");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t per = (int64_t)batch_local * M * N;
    float* mine = C_full + (int64_t)c->rank * per;
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, A_local, B_local, mine);
    d.batch = batch_local;
    d.stream = stream;
    rc = jst_gemm_ex(&d);
    if (rc) return rc;
    if (per == 0) return set_status(JST_OK, nullptr);
    rc = nccl_settle(c, ncclAllGather(mine, C_full, (size_t)per, ncclFloat, c->nccl, s), "ncclAllGather(C)");
    return rc ? rc : set_status(JST_OK, nullptr);
}

}  // extern "C"
