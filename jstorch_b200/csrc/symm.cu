// symm.cu -- multicast-backed buffers (jst_symm) for the fused GEMM +
// all-gather of the row-sharded path (C ABI in include/jstorch_dist.h).
//
// Each rank creates physical device memory (cuMemCreate, POSIX-fd shareable),
// rank 0 creates one multicast object for the team and hands its file
// descriptor to the other ranks over an abstract unix-domain socket
// (SCM_RIGHTS) whose name is derived from the communicator id; every rank adds
// its device, binds its memory and maps two virtual ranges: the ordinary
// (unicast) view of its own copy and the multicast view, through which a store
// reaches every rank's copy.  The CUDA driver entry points are looked up at
// run time (cudaGetDriverEntryPoint), so the library does not link libcuda.
#include <cuda.h>
#include <cuda_runtime.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <poll.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>

#include "dist_internal.h"

struct jst_symm {
    jst_comm* comm = nullptr;
    size_t size = 0;  // bytes mapped (rounded up to the granularities)
    CUmemGenericAllocationHandle mem = 0;
    CUmemGenericAllocationHandle mc = 0;
    CUdeviceptr uc = 0;    // this rank's copy
    CUdeviceptr mcva = 0;  // multicast view
    bool bound = false;
};

namespace jst {
namespace {

struct Drv {
    decltype(&::cuGetErrorString) getErrorString = nullptr;
    decltype(&::cuDeviceGetAttribute) deviceGetAttribute = nullptr;
    decltype(&::cuMemCreate) memCreate = nullptr;
    decltype(&::cuMemRelease) memRelease = nullptr;
    decltype(&::cuMemGetAllocationGranularity) memGetAllocationGranularity = nullptr;
    decltype(&::cuMemAddressReserve) memAddressReserve = nullptr;
    decltype(&::cuMemAddressFree) memAddressFree = nullptr;
    decltype(&::cuMemMap) memMap = nullptr;
    decltype(&::cuMemUnmap) memUnmap = nullptr;
    decltype(&::cuMemSetAccess) memSetAccess = nullptr;
    decltype(&::cuMemExportToShareableHandle) memExportToShareableHandle = nullptr;
    decltype(&::cuMemImportFromShareableHandle) memImportFromShareableHandle = nullptr;
    decltype(&::cuMulticastCreate) multicastCreate = nullptr;
    decltype(&::cuMulticastAddDevice) multicastAddDevice = nullptr;
    decltype(&::cuMulticastBindMem) multicastBindMem = nullptr;
    decltype(&::cuMulticastUnbind) multicastUnbind = nullptr;
    decltype(&::cuMulticastGetGranularity) multicastGetGranularity = nullptr;
    bool ok = false;
};

const Drv& drv() {
    static Drv d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto get = [](const char* name, void** fn) {
            cudaDriverEntryPointQueryResult q;
            return cudaGetDriverEntryPoint(name, fn, cudaEnableDefault, &q) == cudaSuccess &&
                   q == cudaDriverEntryPointSuccess && *fn;
        };
        bool ok = true;
#define JST_DRV(field, name) ok = get(name, reinterpret_cast<void**>(&d.field)) && ok
        JST_DRV(getErrorString, "cuGetErrorString");
        JST_DRV(deviceGetAttribute, "cuDeviceGetAttribute");
        JST_DRV(memCreate, "cuMemCreate");
        JST_DRV(memRelease, "cuMemRelease");
        JST_DRV(memGetAllocationGranularity, "cuMemGetAllocationGranularity");
        JST_DRV(memAddressReserve, "cuMemAddressReserve");
        JST_DRV(memAddressFree, "cuMemAddressFree");
        JST_DRV(memMap, "cuMemMap");
        JST_DRV(memUnmap, "cuMemUnmap");
        JST_DRV(memSetAccess, "cuMemSetAccess");
        JST_DRV(memExportToShareableHandle, "cuMemExportToShareableHandle");
        JST_DRV(memImportFromShareableHandle, "cuMemImportFromShareableHandle");
        JST_DRV(multicastCreate, "cuMulticastCreate");
        JST_DRV(multicastAddDevice, "cuMulticastAddDevice");
        JST_DRV(multicastBindMem, "cuMulticastBindMem");
        JST_DRV(multicastUnbind, "cuMulticastUnbind");
        JST_DRV(multicastGetGranularity, "cuMulticastGetGranularity");
#undef JST_DRV
        d.ok = ok;
    });
    return d;
}

int drv_status(CUresult r, const char* what) {
    if (r == CUDA_SUCCESS) return JST_OK;
    const char* s = nullptr;
    if (drv().getErrorString) drv().getErrorString(r, &s);
    char buf[200];
    std::snprintf(buf, sizeof(buf), "%s: %s", what, s ? s : "CUDA driver error");
    return set_status(r == CUDA_ERROR_NOT_SUPPORTED ? JST_ERR_UNSUPPORTED : JST_ERR_CUDA, buf);
}

// ---- file-descriptor hand-off from rank 0 over an abstract unix socket
void socket_name(const jst_comm* c, unsigned serial, sockaddr_un* addr, socklen_t* len) {
    std::memset(addr, 0, sizeof(*addr));
    addr->sun_family = AF_UNIX;
    char name[96];
    int n = std::snprintf(name, sizeof(name), "jstorch-symm-");
    for (int i = 0; i < 16; ++i) n += std::snprintf(name + n, sizeof(name) - n, "%02x", c->id[i + 8]);
    n += std::snprintf(name + n, sizeof(name) - n, "-%u", serial);
    std::memcpy(addr->sun_path + 1, name, (size_t)n);  // leading NUL: abstract namespace
    *len = (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + n);
}

int send_fd(int sock, int fd) {
    char byte = 'F';
    iovec iov{&byte, 1};
    char ctrl[CMSG_SPACE(sizeof(int))];
    std::memset(ctrl, 0, sizeof(ctrl));
    msghdr msg{};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    msg.msg_control = ctrl;
    msg.msg_controllen = sizeof(ctrl);
    cmsghdr* cm = CMSG_FIRSTHDR(&msg);
    cm->cmsg_level = SOL_SOCKET;
    cm->cmsg_type = SCM_RIGHTS;
    cm->cmsg_len = CMSG_LEN(sizeof(int));
    std::memcpy(CMSG_DATA(cm), &fd, sizeof(int));
    return sendmsg(sock, &msg, 0) == 1 ? 0 : -1;
}

int recv_fd(int sock, int* fd) {
    char byte = 0;
    iovec iov{&byte, 1};
    char ctrl[CMSG_SPACE(sizeof(int))];
    msghdr msg{};
    msg.msg_iov = &iov;
    msg.msg_iovlen = 1;
    msg.msg_control = ctrl;
    msg.msg_controllen = sizeof(ctrl);
    if (recvmsg(sock, &msg, 0) != 1) return -1;
    cmsghdr* cm = CMSG_FIRSTHDR(&msg);
    if (!cm || cm->cmsg_type != SCM_RIGHTS) return -1;
    std::memcpy(fd, CMSG_DATA(cm), sizeof(int));
    return 0;
}

// Rank 0: accept nranks-1 connections (bounded by the deadline) and pass fd.
int serve_fd(const jst_comm* c, unsigned serial, int fd, int listener) {
    const auto t0 = std::chrono::steady_clock::now();
    for (int served = 0; served < c->nranks - 1;) {
        pollfd p{listener, POLLIN, 0};
        const double left = c->timeout_s - std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (left <= 0) return set_status(JST_ERR_TIMEOUT, "multicast handle hand-off: a rank did not connect");
        if (poll(&p, 1, (int)std::min(left * 1000.0, 1000.0)) <= 0) continue;
        int s = accept(listener, nullptr, nullptr);
        if (s < 0) continue;
        const int r = send_fd(s, fd);
        close(s);
        if (r) return set_status(JST_ERR_CUDA, "multicast handle hand-off: sendmsg failed");
        ++served;
    }
    (void)serial;
    return JST_OK;
}

int fetch_fd(const jst_comm* c, unsigned serial, int* fd) {
    sockaddr_un addr;
    socklen_t len;
    socket_name(c, serial, &addr, &len);
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        int s = socket(AF_UNIX, SOCK_STREAM, 0);
        if (s < 0) return set_status(JST_ERR_CUDA, "socket() failed");
        if (connect(s, reinterpret_cast<sockaddr*>(&addr), len) == 0) {
            const int r = recv_fd(s, fd);
            close(s);
            return r ? set_status(JST_ERR_CUDA, "multicast handle hand-off: recvmsg failed") : JST_OK;
        }
        close(s);
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > c->timeout_s)
            return set_status(JST_ERR_TIMEOUT, "multicast handle hand-off: rank 0 never listened");
        std::this_thread::sleep_for(std::chrono::milliseconds(2));
    }
}

void release(jst_symm* sy) {
    const Drv& d = drv();
    if (sy->mcva) {
        d.memUnmap(sy->mcva, sy->size);
        d.memAddressFree(sy->mcva, sy->size);
    }
    if (sy->uc) {
        d.memUnmap(sy->uc, sy->size);
        d.memAddressFree(sy->uc, sy->size);
    }
    if (sy->bound) d.multicastUnbind(sy->mc, sy->comm->device, 0, sy->size);
    if (sy->mem) d.memRelease(sy->mem);
    if (sy->mc) d.memRelease(sy->mc);
}

}  // namespace

int comm_barrier(jst_comm* c, cudaStream_t s) {
    if (!c->barrier_word) {
        if (cudaMalloc(&c->barrier_word, sizeof(float)) != cudaSuccess) {
            cudaGetLastError();
            return set_status(JST_ERR_NOMEM, "barrier word allocation failed");
        }
    }
    int rc = nccl_settle(c, ncclAllReduce(c->barrier_word, c->barrier_word, 1, ncclFloat, ncclSum, c->nccl, s),
                         "barrier all-reduce");
    return rc ? rc : jst_comm_sync(c, reinterpret_cast<jst_stream_t>(s));
}

jst_symm* find_symm(jst_comm* c, const void* p, size_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    for (auto* sy : c->symms)
        if (a >= sy->uc && a + bytes <= sy->uc + sy->size) return sy;
    return nullptr;
}

size_t symm_offset(jst_symm* sy, const void* p) { return reinterpret_cast<uintptr_t>(p) - sy->uc; }

float* symm_multicast_ptr(jst_symm* sy, size_t off) { return reinterpret_cast<float*>(sy->mcva + off); }

}  // namespace jst

extern "C" {

int jst_symm_alloc(jst_comm* c, size_t bytes, jst_symm** out, void** local) {
    using namespace jst;
    int rc = ready(c);
    if (rc) return rc;
    if (!out || !local || bytes == 0) return set_status(JST_ERR_ARG, "jst_symm_alloc: bad argument");
    *out = nullptr;
    *local = nullptr;
    const Drv& d = drv();
    if (!d.ok) return set_status(JST_ERR_UNSUPPORTED, "CUDA driver lacks the multicast entry points");
    int mc_ok = 0;
    rc = drv_status(d.deviceGetAttribute(&mc_ok, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, c->device),
                    "cuDeviceGetAttribute");
    if (rc) return rc;
    if (!mc_ok) return set_status(JST_ERR_UNSUPPORTED, "device has no NVLink-switch multicast support");

    const unsigned serial = c->symm_serial++;
    auto* sy = new jst_symm();
    sy->comm = c;
    CUmemAllocationProp prop{};
    prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    prop.location.id = c->device;
    prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    CUmulticastObjectProp mprop{};
    mprop.numDevices = (unsigned)c->nranks;
    mprop.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t g_mem = 0, g_mc = 0;
    mprop.size = bytes;
    rc = drv_status(d.memGetAllocationGranularity(&g_mem, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED),
                    "cuMemGetAllocationGranularity");
    if (!rc)
        rc = drv_status(d.multicastGetGranularity(&g_mc, &mprop, CU_MULTICAST_GRANULARITY_RECOMMENDED),
                        "cuMulticastGetGranularity");
    if (rc) {
        delete sy;
        return rc;
    }
    const size_t g = std::max(g_mem, g_mc);
    sy->size = (bytes + g - 1) / g * g;
    mprop.size = sy->size;

    rc = drv_status(d.memCreate(&sy->mem, sy->size, &prop, 0), "cuMemCreate");
    // rank 0 creates the multicast object and hands its descriptor out
    if (!rc && c->rank == 0) {
        rc = drv_status(d.multicastCreate(&sy->mc, &mprop), "cuMulticastCreate");
        int fd = -1;
        if (!rc)
            rc = drv_status(d.memExportToShareableHandle(&fd, sy->mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                            "cuMemExportToShareableHandle");
        if (!rc && c->nranks > 1) {
            int listener = socket(AF_UNIX, SOCK_STREAM, 0);
            sockaddr_un addr;
            socklen_t len;
            socket_name(c, serial, &addr, &len);
            if (listener < 0 || bind(listener, reinterpret_cast<sockaddr*>(&addr), len) != 0 ||
                listen(listener, c->nranks) != 0)
                rc = set_status(JST_ERR_CUDA, "multicast handle hand-off: cannot listen");
            else
                rc = serve_fd(c, serial, fd, listener);
            if (listener >= 0) close(listener);
        }
        if (fd >= 0) close(fd);
    } else if (!rc) {
        int fd = -1;
        rc = fetch_fd(c, serial, &fd);
        if (!rc)
            rc = drv_status(d.memImportFromShareableHandle(&sy->mc, reinterpret_cast<void*>((intptr_t)fd),
                                                           CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
                            "cuMemImportFromShareableHandle");
        if (fd >= 0) close(fd);
    }
    if (!rc) rc = drv_status(d.multicastAddDevice(sy->mc, c->device), "cuMulticastAddDevice");
    // every device must be in the team before memory is bound or mapped
    if (!rc) rc = comm_barrier(c, c->comm_stream);
    if (!rc) {
        rc = drv_status(d.multicastBindMem(sy->mc, 0, sy->mem, 0, sy->size, 0), "cuMulticastBindMem");
        sy->bound = rc == JST_OK;
    }
    CUmemAccessDesc acc{};
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = c->device;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    if (!rc) rc = drv_status(d.memAddressReserve(&sy->uc, sy->size, g, 0, 0), "cuMemAddressReserve");
    if (!rc) rc = drv_status(d.memMap(sy->uc, sy->size, 0, sy->mem, 0), "cuMemMap");
    if (!rc) rc = drv_status(d.memSetAccess(sy->uc, sy->size, &acc, 1), "cuMemSetAccess");
    if (!rc) rc = drv_status(d.memAddressReserve(&sy->mcva, sy->size, g, 0, 0), "cuMemAddressReserve");
    if (!rc) rc = drv_status(d.memMap(sy->mcva, sy->size, 0, sy->mc, 0), "cuMemMap(multicast)");
    if (!rc) rc = drv_status(d.memSetAccess(sy->mcva, sy->size, &acc, 1), "cuMemSetAccess(multicast)");
    // every rank is bound and mapped before anyone stores through the team
    if (!rc) rc = comm_barrier(c, c->comm_stream);
    if (rc) {
        release(sy);
        delete sy;
        return rc;
    }
    c->symms.push_back(sy);
    *out = sy;
    *local = reinterpret_cast<void*>(sy->uc);
    return set_status(JST_OK, nullptr);
}

int jst_symm_free(jst_symm* sy) {
    using namespace jst;
    if (!sy) return set_status(JST_OK, nullptr);
    jst_comm* c = sy->comm;
    int rc = JST_OK;
    // nobody may still be storing into a peer's copy
    if (!c->broken && c->nccl) rc = comm_barrier(c, c->comm_stream);
    else cudaDeviceSynchronize();
    release(sy);
    c->symms.erase(std::remove(c->symms.begin(), c->symms.end(), sy), c->symms.end());
    delete sy;
    return rc ? rc : set_status(JST_OK, nullptr);
}

}  // extern "C"
