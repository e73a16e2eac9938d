// dist_internal.h -- communicator state shared by dist.cu and symm.cu.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <vector>

#include "../../include/jstorch_dist.h"
#include "gemm_internal.h"

struct jst_symm;
struct jst_reg;

struct jst_comm {
    ncclComm_t nccl = nullptr;
    int rank = 0;
    int nranks = 1;
    int device = 0;
    double timeout_s = 60.0;
    bool broken = false;
    cudaStream_t comm_stream = nullptr;
    cudaStream_t compute2 = nullptr;  // second compute stream of the row-sharded GEMM
    std::vector<cudaEvent_t> events;
    unsigned char id[JST_COMM_ID_BYTES] = {};  // the communicator id (identical on every rank)
    unsigned symm_serial = 0;                  // multicast buffers created so far (same on every rank)
    float* barrier_word = nullptr;             // 1-float device buffer for host-visible barriers
    std::vector<jst_symm*> symms;              // live multicast-backed buffers of this communicator
    std::vector<jst_reg*> regs;                // buffers registered for copy-engine delivery
    std::vector<cudaStream_t> copy_streams;    // copy-engine streams of the registered path
    // optional timeline of the last sharded call (jst_comm_trace)
    bool trace = false;
    std::vector<cudaEvent_t> trace_ev;
    std::vector<const char*> trace_label;
    size_t trace_n = 0;
};


namespace jst {
int nccl_error(jst_comm* c, ncclResult_t r, const char* what);
// Wait (on the host) until the communicator has no operation in progress.
int nccl_settle(jst_comm* c, ncclResult_t r, const char* what);
int ready(jst_comm* c);
int ensure_events(jst_comm* c, size_t n);
// All ranks reach this point (a 1-float all-reduce on `s`, waited for on the
// host within the communicator's deadline).
int comm_barrier(jst_comm* c, cudaStream_t s);
// With tracing on, record a timing event labelled `label` on stream s.
void trace_mark(jst_comm* c, const char* label, cudaStream_t s);
// The multicast buffer containing [p, p + bytes) on this rank, or nullptr.
jst_symm* find_symm(jst_comm* c, const void* p, size_t bytes);
// Device address through which a store reaches offset `off` of `sy` on every rank.
float* symm_multicast_ptr(jst_symm* sy, size_t off);
size_t symm_offset(jst_symm* sy, const void* p);
// The registered buffer containing [p, p + bytes) on this rank, or nullptr;
// peer_ptr gives where the same offset lives in rank r's buffer (mapped here).
jst_reg* find_reg(jst_comm* c, const void* p, size_t bytes);
void* reg_peer_ptr(jst_reg* r, int rank, const void* local_p);
}  // namespace jst
