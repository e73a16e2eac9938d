// splitk.cu -- the reduce step of split-K GEMMs (both kernels).
//
// A split-K GEMM writes S partial products, part[s][batch][M][N] packed, each
// over one slice of K.  This kernel adds them in slice order (so the result
// is the same on every run) and applies the GEMM's epilogue: column or row
// bias, ReLU, the ReLU-backward mask.
#include <cuda_runtime.h>

#include <algorithm>

#include "gemm_internal.h"
#include "ptx.cuh"

namespace jst {
namespace {

// One thread per W consecutive columns of a row: W = 4 (float4) when N % 4 == 0.
template <int W>
__global__ void splitk_reduce_kernel(const SplitKReduce r) {
    ptx::griddep_wait();  // launched as a programmatic dependent of the GEMM that wrote the partials
    const int nw = r.N / W;
    const int64_t total = (int64_t)r.batch * r.M * nw;
    const int64_t plane = (int64_t)r.batch * r.M * r.N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int cw = (int)(i % nw);
        const int64_t br = i / nw;
        const int row = (int)(br % r.M);
        const int b = (int)(br / r.M);
        const int col = cw * W;
        const int64_t off = ((int64_t)b * r.M + row) * r.N + col;
        float v[W];
#pragma unroll
        for (int j = 0; j < W; ++j) v[j] = 0.0f;
        for (int sl = 0; sl < r.slices; ++sl) {
            const float* src = r.part + sl * plane + off;
            if constexpr (W == 4) {
                const float4 x = __ldg(reinterpret_cast<const float4*>(src));
                v[0] += x.x; v[1] += x.y; v[2] += x.z; v[3] += x.w;
            } else {
                v[0] += __ldg(src);
            }
        }
        float* crow = r.C + (int64_t)b * r.strideC + (int64_t)row * r.ldc;
        const float* arow = r.aux ? r.aux + (int64_t)b * r.stride_aux + (int64_t)row * r.ld_aux : nullptr;
        const float rb = (r.bias && r.bias_row) ? __ldg(r.bias + row) : 0.0f;
#pragma unroll
        for (int j = 0; j < W; ++j) {
            float x = v[j];
            if (r.bias) x += r.bias_row ? rb : __ldg(r.bias + col + j);
            if (r.relu) x = fmaxf(x, 0.0f);
            if (arow && !(__ldg(arow + col + j) > 0.0f)) x = 0.0f;
            v[j] = x;
        }
        if constexpr (W == 4) {
            if (r.vecC) {
                *reinterpret_cast<float4*>(crow + col) = make_float4(v[0], v[1], v[2], v[3]);
                continue;
            }
        }
#pragma unroll
        for (int j = 0; j < W; ++j) crow[col + j] = v[j];
    }
}

}  // namespace

int splitk_reduce_run(const SplitKReduce& r, cudaStream_t s) {
    if (r.M == 0 || r.N == 0 || r.batch == 0) return JST_OK;
    const bool w4 = (r.N & 3) == 0;
    const int64_t total = (int64_t)r.batch * r.M * (w4 ? r.N / 4 : r.N);
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    {
        ProfScope prof(s, KID_SPLITK_REDUCE);
        if (w4) launch_dependent(splitk_reduce_kernel<4>, dim3(blocks), dim3(256), 0, s, r);
        else launch_dependent(splitk_reduce_kernel<1>, dim3(blocks), dim3(256), 0, s, r);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, "split-K reduce launch failed");
}

SplitKReduce splitk_reduce_args(const GemmArgs& a, const float* part, int slices) {
    SplitKReduce r;
    r.part = part;
    r.slices = slices;
    r.batch = a.batch;
    r.M = a.M;
    r.N = a.N;
    r.C = a.C;
    r.ldc = a.ldc;
    r.strideC = a.strideC;
    r.bias = a.bias;
    r.bias_row = a.bias_row;
    r.relu = a.relu;
    r.aux = a.aux;
    r.ld_aux = a.ld_aux;
    r.stride_aux = a.stride_aux;
    r.vecC = ((reinterpret_cast<uintptr_t>(a.C) & 15) == 0) && (a.ldc % 4 == 0) && (a.strideC % 4 == 0);
    return r;
}

}  // namespace jst
