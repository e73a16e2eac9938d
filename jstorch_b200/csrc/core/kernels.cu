// kernels.cu -- the non-GEMM device work of the host core's matmul path.
//
// These are the reference's auxiliary kernels on that path, rewritten for
// B200: 64-bit index math, float4 where layout allows, grids sized in
// multiples of the 148 SMs.
//   strided_copy   Tensor::contiguous (reference misc.cu:216-231, 326-337)
//   fill           Tensor::full / zeros (tensor.cpp:530-535)
//   add            same-shape add, gradient accumulation (binary.cu:16-31)
//   add_rowvec     [R, N] + [N] bias broadcast (binary.cu:34-56 AddOp path)
//   relu           relu forward (kernels.cuh:50)
//   relu_backward  g * (x > 0) in one pass (autograd.hpp:132 runs full, gt, mul)
//   sum_rows       sum over dim 0 of [R, N] -> [N]: the bias gradient
//                  (autograd.hpp:326-327 via reduce.cu:275-287)
//   randn          normal(0, 1) values from (seed, index) only
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "core_kernels.h"

namespace jst {
namespace core {

namespace {
constexpr int kThreads = 256;

int grid_for(int64_t n, int per_thread = 1) {
    const int64_t want = (n + (int64_t)kThreads * per_thread - 1) / ((int64_t)kThreads * per_thread);
    const int64_t cap = 148 * 32;
    return (int)(want < 1 ? 1 : (want > cap ? cap : want));
}

__global__ void strided_copy_kernel(const float* __restrict__ src, float* __restrict__ dst, StridedDesc d,
                                    int64_t total) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t rem = i, off = 0;
        for (int k = d.ndim - 1; k >= 0; --k) {
            const int64_t c = rem % d.shape[k];
            rem /= d.shape[k];
            off += c * d.stride[k];
        }
        dst[i] = src[off];
    }
}

__global__ void fill_kernel(float* __restrict__ dst, float v, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = v;
}

// n4: number of leading float4 groups (0 when a pointer is not 16-byte aligned)
__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c,
                           int64_t n, int64_t n4) {
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float4* c4 = reinterpret_cast<float4*>(c);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 x = a4[i], y = b4[i];
        c4[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
    }
    for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) c[i] = a[i] + b[i];
}

__global__ void add_rowvec_kernel(const float* __restrict__ a, const float* __restrict__ v, float* __restrict__ c,
                                  int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        c[i] = a[i] + __ldg(v + (i % cols));
}

__global__ void relu_kernel(const float* __restrict__ a, float* __restrict__ c, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        c[i] = fmaxf(a[i], 0.0f);
}

__global__ void relu_backward_kernel(const float* __restrict__ g, const float* __restrict__ x,
                                     float* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = x[i] > 0.0f ? g[i] : 0.0f;
}

// One thread per column, rows split over blockDim.y (32) warp-rows and
// combined in shared memory in a fixed order: reads are coalesced along the
// columns, and a [256, N] gradient takes 8 loads per thread.
__global__ void sum_rows_kernel(const float* __restrict__ a, float* __restrict__ out, int64_t rows, int64_t cols) {
    __shared__ float part[32][33];
    const int64_t col = blockIdx.x * 32 + threadIdx.x;
    float s = 0.0f;
    if (col < cols)
        for (int64_t r = threadIdx.y; r < rows; r += blockDim.y) s += a[r * cols + col];
    part[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    if (threadIdx.y == 0 && col < cols) {
        float t = 0.0f;
        for (int k = 0; k < (int)blockDim.y; ++k) t += part[k][threadIdx.x];
        out[col] = t;
    }
}

// SplitMix64 finaliser of (seed, index) -> two uniforms -> Box-Muller normal.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void randn_kernel(float* __restrict__ dst, int64_t n, uint64_t seed) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t r = mix64(seed * 0x100000001B3ull ^ mix64((uint64_t)i));
        const float u1 = ((uint32_t)(r >> 40) + 1u) * (1.0f / 16777217.0f);  // (0, 1]
        const float u2 = (uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);   // [0, 1)
        dst[i] = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
    }
}
}  // namespace

static std::atomic<int64_t> g_strided_copies{0};
int64_t strided_copy_count() { return g_strided_copies.load(); }

void strided_copy(const float* src, float* dst, const StridedDesc& d, int64_t total, cudaStream_t s) {
    if (total <= 0) return;
    g_strided_copies.fetch_add(1, std::memory_order_relaxed);
    strided_copy_kernel<<<grid_for(total), kThreads, 0, s>>>(src, dst, d, total);
}

void fill(float* dst, float v, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    fill_kernel<<<grid_for(n), kThreads, 0, s>>>(dst, v, n);
}

void add(const float* a, const float* b, float* c, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    const bool al = ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                      reinterpret_cast<uintptr_t>(c)) & 15) == 0;
    add_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(a, b, c, n, al ? n / 4 : 0);
}

void add_rowvec(const float* a, const float* v, float* c, int64_t rows, int64_t cols, cudaStream_t s) {
    if (rows * cols <= 0) return;
    add_rowvec_kernel<<<grid_for(rows * cols), kThreads, 0, s>>>(a, v, c, rows, cols);
}

void relu(const float* a, float* c, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    relu_kernel<<<grid_for(n), kThreads, 0, s>>>(a, c, n);
}

void relu_backward(const float* g, const float* x, float* out, int64_t n, cudaStream_t s) {
    if (n <= 0) return;
    relu_backward_kernel<<<grid_for(n), kThreads, 0, s>>>(g, x, out, n);
}

void sum_rows(const float* a, float* out, int64_t rows, int64_t cols, cudaStream_t s) {
    if (cols <= 0) return;
    sum_rows_kernel<<<(unsigned)((cols + 31) / 32), dim3(32, 32), 0, s>>>(a, out, rows, cols);
}

void randn(float* dst, int64_t n, uint64_t seed, cudaStream_t s) {
    if (n <= 0) return;
    randn_kernel<<<grid_for(n), kThreads, 0, s>>>(dst, n, seed);
}

}  // namespace core
}  // namespace jst
