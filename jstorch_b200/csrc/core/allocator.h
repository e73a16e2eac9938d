// allocator.h -- device caching allocator of the host core.
//
// Restates the reference's CudaAllocator (native/core/allocator.hpp:22-101:
// 512-byte aligned blocks bump-allocated from 256 MiB segments, freed blocks
// kept in exact-size bins for O(1) reuse, segments returned only at exit or
// trim) with two changes for a multi-GPU, multi-threaded host:
//   * one pool per device, selected by the current device at allocation time
//     (the reference's single pool ignores devices);
//   * a mutex around every pool (the reference relies on JS being
//     single-threaded, allocator.hpp:15).
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>

namespace jst {
namespace core {

// A device block: freed back to its device's pool when the last owner drops it.
struct Block {
    void* ptr = nullptr;
    size_t bytes = 0;
    int device = 0;
    ~Block();
};

// Allocate `bytes` on the current device (throws std::runtime_error on failure).
std::shared_ptr<Block> device_alloc(size_t bytes);

// Drop the cached free blocks and reset the bump pointers of every device
// pool after a device synchronise (reference: CudaAllocator::trim, :84-89).
void trim_all();

// Bytes currently reserved in segments / cached in free bins, per device.
size_t reserved_bytes(int device);
size_t cached_bytes(int device);

}  // namespace core
}  // namespace jst
