// allocator.cpp -- per-device caching allocator (see allocator.h).
#include "allocator.h"

#include <cuda_runtime.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace jst {
namespace core {

namespace {
constexpr size_t kAlign = 512;                      // allocator.hpp:23
constexpr size_t kSegment = size_t(256) << 20;      // allocator.hpp:24

size_t align_up(size_t n) { return (n + kAlign - 1) & ~(kAlign - 1); }

struct Pool {
    std::mutex mu;
    std::unordered_map<size_t, std::vector<void*>> bins;
    std::vector<void*> segments;
    uintptr_t bump = 0;
    size_t remaining = 0;
    size_t reserved = 0;
    size_t cached = 0;

    void* allocate(size_t bytes) {
        const size_t size = align_up(bytes ? bytes : kAlign);
        std::lock_guard<std::mutex> lk(mu);
        auto it = bins.find(size);
        if (it != bins.end() && !it->second.empty()) {
            void* p = it->second.back();
            it->second.pop_back();
            cached -= size;
            return p;
        }
        if (remaining < size) {
            const size_t seg = size > kSegment ? size : kSegment;
            void* p = nullptr;
            cudaError_t e = cudaMalloc(&p, seg);
            if (e != cudaSuccess || !p) {
                cudaGetLastError();
                throw std::runtime_error(std::string("cudaMalloc failed for segment: ") + cudaGetErrorString(e));
            }
            segments.push_back(p);
            reserved += seg;
            bump = reinterpret_cast<uintptr_t>(p);
            remaining = seg;
        }
        void* p = reinterpret_cast<void*>(bump);
        bump += size;
        remaining -= size;
        return p;
    }

    void release(void* p, size_t bytes) {
        const size_t size = align_up(bytes ? bytes : kAlign);
        std::lock_guard<std::mutex> lk(mu);
        bins[size].push_back(p);
        cached += size;
    }

    void trim() {
        std::lock_guard<std::mutex> lk(mu);
        bins.clear();
        cached = 0;
        bump = 0;
        remaining = 0;
    }
};

Pool g_pools[64];

Pool& pool_of(int dev) {
    if (dev < 0 || dev >= 64) throw std::runtime_error("device index out of range");
    return g_pools[dev];
}
}  // namespace

Block::~Block() {
    if (ptr) pool_of(device).release(ptr, bytes);
}

std::shared_ptr<Block> device_alloc(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error("no CUDA device");
    }
    auto b = std::make_shared<Block>();
    b->ptr = pool_of(dev).allocate(bytes);
    b->bytes = bytes;
    b->device = dev;
    return b;
}

void trim_all() {
    cudaDeviceSynchronize();
    for (auto& p : g_pools) p.trim();
}

size_t reserved_bytes(int device) { return pool_of(device).reserved; }
size_t cached_bytes(int device) { return pool_of(device).cached; }

}  // namespace core
}  // namespace jst
