// dist.cu -- libjstorch_dist.so: row-sharded and batch-sharded GEMMs over
// NCCL, one process per GPU (C ABI in include/jstorch_dist.h).
//
// Row-sharded GEMM (configuration 5 of the benchmark):
//   1. B is broadcast in place from the root (ncclBroadcast, NVLS where NCCL
//      picks it) on the communication stream, while the row blocks of A_local
//      are split into hi / lo TF32 planes on the compute streams;
//   2. B is split once it has arrived;
//   3. for each row block of A_local the tensor-core kernel writes its C rows
//      straight into their global place in C_full (blocks alternate between two
//      compute streams so the tail wave of one overlaps the next); an event
//      hands the block to the communication stream, which all-gathers it in
//      place while later blocks compute.  With block-cyclic row ownership
//      (block i of rank r is global block i * nranks + r) the blocks of one
//      round are contiguous in C_full, so each round is one in-place
//      ncclAllGather.
// No kernel reads another GPU's memory.  C travels by NCCL all-gathers, by
// copy-engine writes into registered peer buffers (jst_comm_register), or by
// multimem stores into a multicast-backed buffer (jst_symm_alloc).
//
// Host-side failure handling: the communicator is created non-blocking and
// every NCCL call is polled against a host deadline; on expiry the
// communicator is aborted and JST_ERR_TIMEOUT returned (a peer that died or
// never joined ends the call with an error, not a hang).
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "dist_internal.h"

namespace jst {

int nccl_error(jst_comm* c, ncclResult_t r, const char* what) {
    char buf[256];
    std::snprintf(buf, sizeof(buf), "%s: %s%s%s", what, ncclGetErrorString(r), c && c->nccl ? " / " : "",
                  c && c->nccl ? ncclGetLastError(c->nccl) : "");
    if (c) c->broken = true;
    return set_status(JST_ERR_NCCL, buf);
}

// Wait (on the host) until the communicator has no operation in progress.
// Polls with a yield for the first 2 ms (an enqueue usually settles within
// tens of microseconds, and the caller's next launches wait for it), then
// every 200 us up to the communicator's deadline.
int nccl_settle(jst_comm* c, ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return JST_OK;
    if (r != ncclInProgress) return nccl_error(c, r, what);
    const auto t0 = std::chrono::steady_clock::now();
    ncclResult_t st = ncclInProgress;
    while (true) {
        if (ncclCommGetAsyncError(c->nccl, &st) != ncclSuccess) return nccl_error(c, st, what);
        if (st != ncclInProgress) break;
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el < 2e-3) {
            std::this_thread::yield();
            continue;
        }
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

void trace_mark(jst_comm* c, const char* label, cudaStream_t s) {
    if (!c->trace) return;
    if (c->trace_n == c->trace_ev.size()) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) {
            cudaGetLastError();
            return;
        }
        c->trace_ev.push_back(e);
        c->trace_label.push_back(nullptr);
    }
    c->trace_label[c->trace_n] = label;
    cudaEventRecord(c->trace_ev[c->trace_n], s);
    ++c->trace_n;
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
    if (cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&c->compute2, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
        delete c;
        return set_status(JST_ERR_CUDA, "stream create failed");
    }
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    std::memcpy(c->id, id, JST_COMM_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&c->nccl, nranks, u, rank, &cfg);
    int rc = (c->nccl == nullptr && r != ncclSuccess && r != ncclInProgress) ? nccl_error(c, r, "ncclCommInitRank")
                                                                            : nccl_settle(c, r, "ncclCommInitRank");
    if (rc) {
        if (c->nccl) ncclCommAbort(c->nccl);
        cudaStreamDestroy(c->comm_stream);
        cudaStreamDestroy(c->compute2);
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

int jst_comm_trace(jst_comm* c, int on) {
    if (!c) return jst::set_status(JST_ERR_ARG, "null communicator");
    c->trace = on != 0;
    c->trace_n = 0;
    return jst::set_status(JST_OK, nullptr);
}

int jst_comm_trace_read(jst_comm* c, char* labels, double* ms, int max_entries) {
    if (!c || !labels || !ms) return -jst::set_status(JST_ERR_ARG, "jst_comm_trace_read: bad argument");
    const int n = (int)std::min<size_t>(c->trace_n, (size_t)max_entries);
    for (int i = 0; i < n; ++i) {
        float t = 0.f;
        if (cudaEventSynchronize(c->trace_ev[i]) != cudaSuccess ||
            cudaEventElapsedTime(&t, c->trace_ev[0], c->trace_ev[i]) != cudaSuccess)
            cudaGetLastError();
        std::snprintf(labels + 32 * i, 32, "%s", c->trace_label[i] ? c->trace_label[i] : "");
        ms[i] = t;
    }
    return n;
}

int jst_comm_rank(const jst_comm* c) { return c ? c->rank : -1; }
// The rank count NCCL reports for the communicator (the requested count once
// the communicator is gone).
int jst_comm_size(const jst_comm* c) {
    if (!c) return -1;
    int n = c->nranks;
    if (c->nccl && !c->broken && ncclCommCount(c->nccl, &n) != ncclSuccess) n = c->nranks;
    return n;
}

int jst_comm_destroy(jst_comm* c) {
    using namespace jst;
    if (!c) return set_status(JST_OK, nullptr);
    int rc = JST_OK;
    // buffers still registered are released first, while the barrier works
    for (auto* sy : std::vector<jst_symm*>(c->symms)) jst_symm_free(sy);
    for (auto* r : std::vector<jst_reg*>(c->regs)) jst_comm_deregister(r);
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
    if (c->barrier_word) cudaFree(c->barrier_word);
    if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
    if (c->compute2) cudaStreamDestroy(c->compute2);
    for (auto st : c->copy_streams) cudaStreamDestroy(st);
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
    // events: entry, broadcast done, B split done, all done, one per block, one per copy stream
    rc = ensure_events(c, (size_t)nchunks + 4 + 8);
    if (rc) return rc;
    cudaEvent_t ev_entry = c->events[0], ev_bcast = c->events[1], ev_bsplit = c->events[2],
                ev_done = c->events[3];
    auto ev_blk = [&](int i) { return c->events[4 + i]; };
    auto cuda_ok = [&](cudaError_t e) {
        if (e == cudaSuccess) return true;
        cudaGetLastError();
        rc = set_status(JST_ERR_CUDA, "stream / event hand-off failed");
        return false;
    };
    // Row blocks alternate between the caller's stream and a second compute
    // stream, so one block's last wave of tiles overlaps the next block's
    // first; the collectives run in order on the communication stream.
    cudaStream_t cs[2] = {s, c->compute2};
    c->trace_n = 0;
    trace_mark(c, "entry", s);
    if (!cuda_ok(cudaEventRecord(ev_entry, s)) || !cuda_ok(cudaStreamWaitEvent(c->compute2, ev_entry, 0)) ||
        !cuda_ok(cudaStreamWaitEvent(c->comm_stream, ev_entry, 0)))
        return rc;

    // 1. B from the root to every rank, in place, on the communication stream
    rc = nccl_settle(c, ncclBroadcast(B, B, (size_t)K * N, ncclFloat, root, c->nccl, c->comm_stream),
                     "ncclBroadcast(B)");
    if (rc) return rc;
    trace_mark(c, "broadcast B done", c->comm_stream);
    if (!cuda_ok(cudaEventRecord(ev_bcast, c->comm_stream))) return rc;

    const size_t Kp = (size_t)((K + 3) & ~3);
    const size_t a_plane = (size_t)M_local * Kp, b_plane = (size_t)N * Kp;
    void* ws = nullptr;
    if (M_local > 0) {
        rc = workspace_alloc((2 * a_plane + 2 * b_plane) * sizeof(float), s, &ws);
        if (rc) return rc;
        if (!cuda_ok(cudaEventRecord(ev_entry, s)) || !cuda_ok(cudaStreamWaitEvent(c->compute2, ev_entry, 0))) {
            workspace_free(ws, s);
            return rc;
        }
    }
    float* a_hi = static_cast<float*>(ws);
    float* a_lo = a_hi + a_plane;
    float* b_hi = a_lo + a_plane;
    float* b_lo = b_hi + b_plane;

    // 2. split each block of A_local on its own stream (overlaps the broadcast)
    for (int i = 0; i < nchunks && !rc; ++i)
        rc = tc_split(A_local + (size_t)i * chunk_rows * K, 1, K, 0, chunk_rows, K, 1, a_hi + (size_t)i * chunk_rows * Kp,
                      a_lo + (size_t)i * chunk_rows * Kp, cs[i & 1]);
    // 3. split B once it has arrived; both compute streams wait for it
    if (!rc && nchunks > 0) {
        if (cuda_ok(cudaStreamWaitEvent(s, ev_bcast, 0))) rc = tc_split(B, 0, N, 0, N, K, 1, b_hi, b_lo, s);
        trace_mark(c, "split B done", s);
        if (!rc && cuda_ok(cudaEventRecord(ev_bsplit, s))) cuda_ok(cudaStreamWaitEvent(c->compute2, ev_bsplit, 0));
    }
    // 4. per block: GEMM into its place in C_full, then its in-place
    // all-gather -- or, with a multicast-backed C_full, the GEMM's epilogue
    // stores the block once through the multicast view into every rank's copy
    const size_t c_bytes = (size_t)M_local * c->nranks * N * sizeof(float);
    jst_symm* sy = find_symm(c, C_full, c_bytes);
    jst_reg* reg = sy ? nullptr : find_reg(c, C_full, c_bytes);
    const int ncopy = reg ? (int)std::min<size_t>(c->copy_streams.size(), 8) : 0;
    for (int i = 0; i < nchunks && !rc; ++i) {
        const int64_t grow = ((int64_t)i * c->nranks + c->rank) * chunk_rows;  // first global row of the block
        float* cblk = C_full + grow * N;
        float* cdst = sy ? symm_multicast_ptr(sy, symm_offset(sy, cblk)) : cblk;
        rc = tc_gemm_planes(a_hi + (size_t)i * chunk_rows * Kp, a_lo + (size_t)i * chunk_rows * Kp, b_hi, b_lo,
                            chunk_rows, N, K, 1, cdst, N, 0, nullptr, 0, device_error_word(), cs[i & 1], sy ? 1 : 0);
        if (rc) break;
        trace_mark(c, "gemm block done", cs[i & 1]);
        if (!cuda_ok(cudaEventRecord(ev_blk(i), cs[i & 1])) ||
            !cuda_ok(cudaStreamWaitEvent(c->comm_stream, ev_blk(i), 0)))
            break;
        if (sy) continue;
        if (reg) {  // copy engines push the block into every other rank's C_full
            const size_t blk_bytes = (size_t)chunk_rows * N * sizeof(float);
            for (int k = 1; k < c->nranks && !rc; ++k) {
                const int q = (c->rank + k) % c->nranks;  // stagger destinations across ranks
                cudaStream_t cp = c->copy_streams[(size_t)(k - 1) % ncopy];
                if (!cuda_ok(cudaStreamWaitEvent(cp, ev_blk(i), 0))) break;
                if (!cuda_ok(cudaMemcpyAsync(reg_peer_ptr(reg, q, cblk), cblk, blk_bytes, cudaMemcpyDeviceToDevice,
                                             cp)))
                    break;
            }
            continue;
        }
        float* round0 = C_full + (int64_t)i * c->nranks * chunk_rows * N;
        rc = nccl_settle(c, ncclAllGather(cblk, round0, (size_t)chunk_rows * N, ncclFloat, c->nccl, c->comm_stream),
                         "ncclAllGather(C)");
        trace_mark(c, "all-gather round done", c->comm_stream);
    }
    // copy path: the communication stream waits for every copy stream
    for (int k = 0; k < ncopy && !rc; ++k) {
        cudaEvent_t e = c->events[4 + (size_t)nchunks + k];
        if (!cuda_ok(cudaEventRecord(e, c->copy_streams[k])) || !cuda_ok(cudaStreamWaitEvent(c->comm_stream, e, 0)))
            break;
    }
    // fused and copy paths: every rank's blocks have landed everywhere once
    // every rank has passed its last GEMM / copy (a 1-float all-reduce)
    if (!rc && (sy || reg) && nchunks > 0) {
        if (!c->barrier_word && cudaMalloc(&c->barrier_word, sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            rc = set_status(JST_ERR_NOMEM, "barrier word allocation failed");
        }
        if (!rc)
            rc = nccl_settle(c, ncclAllReduce(c->barrier_word, c->barrier_word, 1, ncclFloat, ncclSum, c->nccl,
                                              c->comm_stream),
                             "ncclAllReduce(barrier)");
    }
    // the caller's stream continues once every collective (hence every block) is done
    trace_mark(c, "all done", c->comm_stream);
    if (cuda_ok(cudaEventRecord(ev_done, c->comm_stream))) cuda_ok(cudaStreamWaitEvent(s, ev_done, 0));
    const int frc = ws ? workspace_free(ws, s) : JST_OK;
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
