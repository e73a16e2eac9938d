// hostio.h -- host <-> device transfers of the host core (Tensor.fromBuffer /
// toArray), staged through pinned memory.
//
// Reference: Tensor::from_array / from_buffer (native/core/tensor.cpp:740-750)
// is a synchronous cudaMemcpy from the JS heap (pageable), and to_array
// (:775-800) synchronises the whole device, copies synchronously, and then
// napi.cpp:17-30 builds nested JS arrays element by element.
//
// Here, per device, two pinned staging chunks alternate: the host copy of
// chunk i+1 (pageable -> pinned) runs while the DMA of chunk i is in flight.
//   * h2d returns once the source has been read; the last DMAs may still be
//     running on `s` (they read only the staging chunks), so the tensor is
//     ready in stream order, not at return;
//   * d2h waits for `s` only (not the whole device) and returns when `dst`
//     holds the data;
//   * a source or destination that is already page-locked (registered or
//     allocated pinned) is copied by one direct DMA.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace jst {
namespace core {

constexpr size_t kStageChunkBytes = 8u << 20;  // per staging chunk

void h2d(float* dst_dev, const float* src_host, int64_t count, cudaStream_t s);
void d2h(float* dst_host, const float* src_dev, int64_t count, cudaStream_t s);

// Release the pinned staging chunks of every device.
void hostio_release();

}  // namespace core
}  // namespace jst
