// core_kernels.h -- launchers of the host core's auxiliary kernels (kernels.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace jst {
namespace core {

constexpr int kMaxDims = 8;

struct StridedDesc {
    int ndim;
    int64_t shape[kMaxDims];
    int64_t stride[kMaxDims];  // source strides in elements
};

void strided_copy(const float* src, float* dst, const StridedDesc& d, int64_t total, cudaStream_t s);
// number of strided copies (Tensor::contiguous materialisations) so far
int64_t strided_copy_count();
void fill(float* dst, float v, int64_t n, cudaStream_t s);
void add(const float* a, const float* b, float* c, int64_t n, cudaStream_t s);
void add_rowvec(const float* a, const float* v, float* c, int64_t rows, int64_t cols, cudaStream_t s);
void relu(const float* a, float* c, int64_t n, cudaStream_t s);
void relu_backward(const float* g, const float* x, float* out, int64_t n, cudaStream_t s);
void sum_rows(const float* a, float* out, int64_t rows, int64_t cols, cudaStream_t s);
void randn(float* dst, int64_t n, uint64_t seed, cudaStream_t s);

}  // namespace core
}  // namespace jst
