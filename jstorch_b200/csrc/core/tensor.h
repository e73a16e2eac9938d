// tensor.h -- fp32 device tensor of the host core (the part of the
// reference's jstorch::Tensor, native/core/tensor.hpp, that the matmul path
// uses), calling libjstorch_gemm.so through its C ABI for every product.
//
// Differences from the reference that matter on this path:
//   * matmul passes a transposed 2-D view straight to the NT / TN kernels
//     instead of materialising it with contiguous() (tensor.cpp:631), so the
//     nn.Linear forward (x . W^T) and both backward GEMMs move no extra bytes;
//   * 3-D x 3-D checks that K and the batch sizes agree (the reference does not);
//   * shapes and strides are 64-bit.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "allocator.h"

namespace jst {
namespace core {

using Shape = std::vector<int64_t>;

int64_t numel(const Shape& s);
Shape contiguous_strides(const Shape& s);
std::string shape_str(const Shape& s);

class Tensor {
  public:
    Tensor() = default;
    explicit Tensor(const Shape& shape);  // uninitialised, contiguous, current device

    // factories (tensor.cpp:530-535, 740-758)
    static Tensor from_buffer(const float* host, int64_t count, const Shape& shape);
    static Tensor full(const Shape& shape, float value);
    static Tensor zeros(const Shape& shape) { return full(shape, 0.0f); }
    static Tensor randn(const Shape& shape);  // seed counter starting at 42, as tensor.cpp:755

    // host read-back honouring strides (tensor.cpp:775-800)
    std::vector<float> to_array() const;
    // the same into a caller buffer of size() floats (a Float32Array's storage)
    void to_host(float* dst) const;

    const Shape& shape() const { return shape_; }
    const Shape& strides() const { return strides_; }
    int ndim() const { return (int)shape_.size(); }
    int64_t size() const { return numel(shape_); }
    int device() const { return block_ ? block_->device : 0; }
    bool defined() const { return (bool)block_; }
    bool is_contiguous() const;
    float* data() const { return block_ ? static_cast<float*>(block_->ptr) + offset_ : nullptr; }

    // views (tensor.cpp:190-260)
    Tensor transpose() const;  // 2-D only
    Tensor transpose(int d0, int d1) const;
    Tensor view(const Shape& s) const;
    Tensor reshape(const Shape& s) const;
    Tensor slice(int dim, int64_t start, int64_t end) const;  // tensor.cpp:243-258
    Tensor squeeze(int axis) const;
    Tensor unsqueeze(int axis) const;

    Tensor contiguous() const;  // strided copy on the device (misc.cu:216-231)

    // the matmul path
    Tensor matmul(const Tensor& other) const;                      // tensor.cpp:630-654
    Tensor linear(const Tensor& weight, const Tensor* bias) const;  // tensor.cpp:658-671
    Tensor add(const Tensor& other) const;  // same shape, or [..., N] + [N] (binary.cu)
    Tensor relu() const;                    // kernels.cuh:50
    Tensor relu_backward(const Tensor& x) const;  // this * (x > 0)  (autograd.hpp:132)
    Tensor sum(int dim, bool keepdim) const;      // dim 0 of 2-D; other dims via transpose

  private:
    std::shared_ptr<Block> block_;
    int64_t offset_ = 0;
    Shape shape_, strides_;
};

// current stream of the core (the reference enqueues everything on stream 0)
cudaStream_t core_stream();
void set_core_stream(cudaStream_t s);

// Bytes the allocator holds; clear_cache mirrors Tensor::clear_cache (tensor.cpp:1024-1029).
void clear_cache();

}  // namespace core
}  // namespace jst
