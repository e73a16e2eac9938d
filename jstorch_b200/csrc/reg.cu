// reg.cu -- buffers registered with every rank of a communicator
// (jst_comm_register), so the row-sharded GEMM can push each finished C block
// into the other ranks' copies with the copy engines: no collective kernel
// competes with the GEMM for SMs.
//
// Registration is collective: each rank takes a CUDA IPC handle of the
// allocation containing its buffer (plus the buffer's offset in it); the
// records are all-gathered through the communicator and every rank maps the
// other ranks' allocations (cudaIpcOpenMemHandle).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "dist_internal.h"

struct jst_reg {
    jst_comm* comm = nullptr;
    char* local = nullptr;  // this rank's buffer
    size_t bytes = 0;
    std::vector<char*> peer;       // rank r's buffer as mapped here (peer[rank] = local)
    std::vector<void*> peer_base;  // opened IPC mappings (nullptr for this rank)
};

namespace jst {
namespace {

struct IpcRecord {
    cudaIpcMemHandle_t handle;
    uint64_t offset;  // buffer start minus allocation start
    uint64_t bytes;
};

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn get_address_range() {
    static GetAddressRangeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<GetAddressRangeFn>(p);
    });
    return fn;
}

void unmap(jst_reg* r) {
    for (void* b : r->peer_base)
        if (b) cudaIpcCloseMemHandle(b);
    r->peer_base.clear();
}

}  // namespace

jst_reg* find_reg(jst_comm* c, const void* p, size_t bytes) {
    const char* a = static_cast<const char*>(p);
    for (auto* r : c->regs)
        if (a >= r->local && a + bytes <= r->local + r->bytes) return r;
    return nullptr;
}

void* reg_peer_ptr(jst_reg* r, int rank, const void* local_p) {
    return r->peer[rank] + (static_cast<const char*>(local_p) - r->local);
}

}  // namespace jst

extern "C" {

int jst_comm_register(jst_comm* c, void* ptr, size_t bytes, jst_reg** out) {
    using namespace jst;
    int rc = ready(c);
    if (rc) return rc;
    if (!ptr || !bytes || !out) return set_status(JST_ERR_ARG, "jst_comm_register: bad argument");
    *out = nullptr;
    auto range = get_address_range();
    if (!range) return set_status(JST_ERR_UNSUPPORTED, "cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t alloc = 0;
    if (range(&base, &alloc, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return set_status(JST_ERR_ARG, "jst_comm_register: pointer is not device memory");
    if (reinterpret_cast<CUdeviceptr>(ptr) + bytes > base + alloc)
        return set_status(JST_ERR_ARG, "jst_comm_register: buffer extends past its allocation");

    IpcRecord mine{};
    if (cudaIpcGetMemHandle(&mine.handle, reinterpret_cast<void*>(base)) != cudaSuccess) {
        cudaGetLastError();
        return set_status(JST_ERR_UNSUPPORTED, "cudaIpcGetMemHandle failed (memory not from cudaMalloc?)");
    }
    mine.offset = reinterpret_cast<CUdeviceptr>(ptr) - base;
    mine.bytes = bytes;
    // all-gather the records through the communicator (device staging)
    const size_t rec = sizeof(IpcRecord);
    char* dev = nullptr;
    if (cudaMalloc(&dev, rec * (size_t)c->nranks) != cudaSuccess) {
        cudaGetLastError();
        return set_status(JST_ERR_NOMEM, "registration staging allocation failed");
    }
    std::vector<IpcRecord> all((size_t)c->nranks);
    rc = cudaMemcpyAsync(dev + rec * c->rank, &mine, rec, cudaMemcpyHostToDevice, c->comm_stream) == cudaSuccess
             ? JST_OK
             : set_status(JST_ERR_CUDA, "registration copy failed");
    if (!rc)
        rc = nccl_settle(c, ncclAllGather(dev + rec * c->rank, dev, rec, ncclChar, c->nccl, c->comm_stream),
                         "ncclAllGather(registration)");
    if (!rc) rc = jst_comm_sync(c, reinterpret_cast<jst_stream_t>(c->comm_stream));
    if (!rc && cudaMemcpy(all.data(), dev, rec * (size_t)c->nranks, cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = set_status(JST_ERR_CUDA, "registration copy failed");
    cudaFree(dev);
    if (rc) return rc;

    auto* r = new jst_reg();
    r->comm = c;
    r->local = static_cast<char*>(ptr);
    r->bytes = bytes;
    r->peer.assign((size_t)c->nranks, nullptr);
    r->peer_base.assign((size_t)c->nranks, nullptr);
    for (int q = 0; q < c->nranks && !rc; ++q) {
        if (all[q].bytes != bytes) {
            rc = set_status(JST_ERR_ARG, "jst_comm_register: ranks registered different sizes");
            break;
        }
        if (q == c->rank) {
            r->peer[q] = r->local;
            continue;
        }
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[q].handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            rc = set_status(JST_ERR_UNSUPPORTED, "cudaIpcOpenMemHandle failed");
            break;
        }
        r->peer_base[q] = p;
        r->peer[q] = static_cast<char*>(p) + all[q].offset;
    }
    // copy-engine streams, created once per communicator
    while (!rc && c->copy_streams.size() < 4) {
        cudaStream_t st;
        if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            rc = set_status(JST_ERR_CUDA, "stream create failed");
            break;
        }
        c->copy_streams.push_back(st);
    }
    // every rank has mapped every buffer before anyone writes into one
    if (!rc) rc = comm_barrier(c, c->comm_stream);
    if (rc) {
        unmap(r);
        delete r;
        return rc;
    }
    c->regs.push_back(r);
    *out = r;
    return set_status(JST_OK, nullptr);
}

int jst_comm_deregister(jst_reg* r) {
    using namespace jst;
    if (!r) return set_status(JST_OK, nullptr);
    jst_comm* c = r->comm;
    int rc = JST_OK;
    // nobody may still be writing into another rank's buffer
    if (!c->broken && c->nccl) rc = comm_barrier(c, c->comm_stream);
    else cudaDeviceSynchronize();
    unmap(r);
    c->regs.erase(std::remove(c->regs.begin(), c->regs.end(), r), c->regs.end());
    delete r;
    return rc ? rc : set_status(JST_OK, nullptr);
}

}  // extern "C"
