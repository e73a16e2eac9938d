// gemm_ffma.cu -- fp32 FFMA (SIMT) GEMM for small and skinny shapes.
//
// Exact fp32 arithmetic (one fma per product, fp32 accumulation), all four layouts (op(A) = A or A^T, op(B) = B or B^T, the NN/NT/TN
// forms of native/ops/matmul.cu:28-67 and of GradTensor::matmul_'s backward,
// native/core/autograd.hpp:433-441), strided batches and the fused bias / ReLU
// epilogue (matmul.cu:18-23, kernels.cuh:50).
//
// Register-blocked outer-product kernel: a CTA owns a BM x BN tile of C; each
// thread owns (4*RM) x (4*RN) outputs laid out as RM x RN blocks of 4 x 4 that
// sit BM/RM rows and BN/RN columns apart, so the shared-memory reads of a warp
// are conflict-free float4 loads.  Tiles of A and B are staged k-major in
// shared memory (double buffered; the next tile is fetched into registers
// while the current one is multiplied).  Global loads are float4 whenever
// the operand's leading dimension and base allow it, scalar and bounds-checked
// elsewhere; tiles wholly inside M x N with aligned operands skip the
// per-element checks for every full k-slab.
//
// Split K: when the tiles of C cannot fill the SMs (the M = 256 layers of an
// MLP, 512^3), K is cut into S slices of whole BK steps; CTA (tile, slice)
// writes its partial tile to a stream-ordered workspace and the split-K
// reduce (splitk.cu) adds the S partials in slice order and applies the
// epilogue.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "gemm_internal.h"
#include "ptx.cuh"

namespace jst {
namespace ffma {

struct Params {
    int M, N, K;
    const float* A; int64_t lda, strideA;
    const float* B; int64_t ldb, strideB;
    float* C; int64_t ldc, strideC;
    const float* bias;
    int bias_row;  // bias[row] instead of bias[col]
    int relu;
    const float* aux;
    int64_t ld_aux, stride_aux;
    int vecA, vecB, vecC;
    int kslices, kchunk;  // split K: S slices of kchunk (a multiple of BK); S = 1: no split
    float* part;          // S > 1: partial tiles, [S][batch][M][N] packed
};

// Two CTAs per SM: the register cap (128 for 256 threads) keeps 16 warps
// resident to hide the shared-memory and global-load latency.
template <int BM, int BN, int BK, int RM, int RN, bool TA, bool TB>
__global__ void __launch_bounds__((BM / (4 * RM)) * (BN / (4 * RN)), 2)
    ffma_gemm_kernel(const Params p) {
    constexpr int TX = BN / (4 * RN);
    constexpr int TY = BM / (4 * RM);
    constexpr int NT = TX * TY;
    constexpr int PAD = 4;
    constexpr int A4 = BM * BK / 4;  // float4 slots per A tile
    constexpr int B4 = BN * BK / 4;
    constexpr int LA = (A4 + NT - 1) / NT;
    constexpr int LB = (B4 + NT - 1) / NT;

    __shared__ __align__(16) float As[2][BK][BM + PAD];
    __shared__ __align__(16) float Bs[2][BK][BN + PAD];

    // launched as a programmatic dependent: wait for the previous kernel's
    // writes, then let the next kernel (the split-K reduce) be scheduled
    ptx::griddep_wait();
    ptx::griddep_launch_dependents();

    const int tid = threadIdx.x;
    const int tx = tid % TX;
    const int ty = tid / TX;
    const int m0 = blockIdx.y * BM;
    const int n0 = blockIdx.x * BN;
    const int b = blockIdx.z / p.kslices;
    const int slice = blockIdx.z - b * p.kslices;
    const int kbeg = slice * p.kchunk;
    const int kend = min(p.K, kbeg + p.kchunk);
    const float* A = p.A + (int64_t)b * p.strideA;
    const float* B = p.B + (int64_t)b * p.strideB;
    float* C = p.C + (int64_t)b * p.strideC;

    float ra[LA][4], rb[LB][4];

    // Interior tiles of float4-aligned operands load whole k-slabs with no
    // per-element bounds checks (a uniform branch per slab).
    const bool interior = p.vecA && p.vecB && m0 + BM <= p.M && n0 + BN <= p.N;

    // Fetch the k-slab starting at k0 into registers.
    auto fetch = [&](int k0) {
        if (interior && k0 + BK <= kend) {
#pragma unroll
            for (int l = 0; l < LA; ++l) {
                const int f = tid + l * NT;
                if (f >= A4) break;
                const int r = !TA ? f / (BK / 4) : f / (BM / 4);
                const int c = !TA ? (f % (BK / 4)) * 4 : (f % (BM / 4)) * 4;
                const float* src = A + (int64_t)((!TA ? m0 : k0) + r) * p.lda + (!TA ? k0 : m0) + c;
                const float4 v = __ldg(reinterpret_cast<const float4*>(src));
                ra[l][0] = v.x; ra[l][1] = v.y; ra[l][2] = v.z; ra[l][3] = v.w;
            }
#pragma unroll
            for (int l = 0; l < LB; ++l) {
                const int f = tid + l * NT;
                if (f >= B4) break;
                const int r = !TB ? f / (BN / 4) : f / (BK / 4);
                const int c = !TB ? (f % (BN / 4)) * 4 : (f % (BK / 4)) * 4;
                const float* src = B + (int64_t)((!TB ? k0 : n0) + r) * p.ldb + (!TB ? n0 : k0) + c;
                const float4 v = __ldg(reinterpret_cast<const float4*>(src));
                rb[l][0] = v.x; rb[l][1] = v.y; rb[l][2] = v.z; rb[l][3] = v.w;
            }
            return;
        }
#pragma unroll
        for (int l = 0; l < LA; ++l) {
            const int f = tid + l * NT;
            int r, c;  // r: index along the contiguous-4 run's row, c: start of the run
            if (!TA) { r = f / (BK / 4); c = (f % (BK / 4)) * 4; }   // row m, cols k..k+3
            else     { r = f / (BM / 4); c = (f % (BM / 4)) * 4; }   // row k, cols m..m+3
            const int gr = (!TA ? m0 : k0) + r;
            const int gc = (!TA ? k0 : m0) + c;
            const int rlim = !TA ? p.M : p.K;
            const int clim = !TA ? p.K : p.M;
            if (f < A4 && gr < rlim) {
                const float* src = A + (int64_t)gr * p.lda + gc;
                if (p.vecA && gc + 3 < clim) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(src));
                    ra[l][0] = v.x; ra[l][1] = v.y; ra[l][2] = v.z; ra[l][3] = v.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) ra[l][j] = (gc + j < clim) ? __ldg(src + j) : 0.0f;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) ra[l][j] = 0.0f;
            }
        }
#pragma unroll
        for (int l = 0; l < LB; ++l) {
            const int f = tid + l * NT;
            int r, c;
            if (!TB) { r = f / (BN / 4); c = (f % (BN / 4)) * 4; }   // row k, cols n..n+3
            else     { r = f / (BK / 4); c = (f % (BK / 4)) * 4; }   // row n, cols k..k+3
            const int gr = (!TB ? k0 : n0) + r;
            const int gc = (!TB ? n0 : k0) + c;
            const int rlim = !TB ? p.K : p.N;
            const int clim = !TB ? p.N : p.K;
            if (f < B4 && gr < rlim) {
                const float* src = B + (int64_t)gr * p.ldb + gc;
                if (p.vecB && gc + 3 < clim) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(src));
                    rb[l][0] = v.x; rb[l][1] = v.y; rb[l][2] = v.z; rb[l][3] = v.w;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) rb[l][j] = (gc + j < clim) ? __ldg(src + j) : 0.0f;
                }
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) rb[l][j] = 0.0f;
            }
        }
    };

    auto stash = [&](int buf) {
#pragma unroll
        for (int l = 0; l < LA; ++l) {
            const int f = tid + l * NT;
            if (f >= A4) continue;
            if (!TA) {
                const int m = f / (BK / 4), k = (f % (BK / 4)) * 4;
#pragma unroll
                for (int j = 0; j < 4; ++j) As[buf][k + j][m] = ra[l][j];
            } else {
                const int k = f / (BM / 4), m = (f % (BM / 4)) * 4;
                *reinterpret_cast<float4*>(&As[buf][k][m]) = make_float4(ra[l][0], ra[l][1], ra[l][2], ra[l][3]);
            }
        }
#pragma unroll
        for (int l = 0; l < LB; ++l) {
            const int f = tid + l * NT;
            if (f >= B4) continue;
            if (!TB) {
                const int k = f / (BN / 4), n = (f % (BN / 4)) * 4;
                *reinterpret_cast<float4*>(&Bs[buf][k][n]) = make_float4(rb[l][0], rb[l][1], rb[l][2], rb[l][3]);
            } else {
                const int n = f / (BK / 4), k = (f % (BK / 4)) * 4;
#pragma unroll
                for (int j = 0; j < 4; ++j) Bs[buf][k + j][n] = rb[l][j];
            }
        }
    };

    float acc[4 * RM][4 * RN];
#pragma unroll
    for (int i = 0; i < 4 * RM; ++i)
#pragma unroll
        for (int j = 0; j < 4 * RN; ++j) acc[i][j] = 0.0f;

    // kbeg is a multiple of BK and slices end on a BK step or at K, so the
    // bounds checks against K in fetch() also keep each slice to its own range
    const int nk = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
    if (nk > 0) {
        fetch(kbeg);
        stash(0);
    }
    __syncthreads();
    for (int t = 0; t < nk; ++t) {
        const int buf = t & 1;
        if (t + 1 < nk) fetch(kbeg + (t + 1) * BK);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float a[4 * RM], bv[4 * RN];
#pragma unroll
            for (int r = 0; r < RM; ++r) {
                const float4 v = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4 + r * (BM / RM)]);
                a[r * 4 + 0] = v.x; a[r * 4 + 1] = v.y; a[r * 4 + 2] = v.z; a[r * 4 + 3] = v.w;
            }
#pragma unroll
            for (int c = 0; c < RN; ++c) {
                const float4 v = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4 + c * (BN / RN)]);
                bv[c * 4 + 0] = v.x; bv[c * 4 + 1] = v.y; bv[c * 4 + 2] = v.z; bv[c * 4 + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < 4 * RM; ++i)
#pragma unroll
                for (int j = 0; j < 4 * RN; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
        }
        if (t + 1 < nk) stash(buf ^ 1);
        __syncthreads();
    }

    if (p.kslices > 1) {  // partial tile to the workspace; the reduce kernel applies the epilogue
        float* P = p.part + ((int64_t)slice * (gridDim.z / p.kslices) + b) * ((int64_t)p.M * p.N);
        const bool vec = (p.N & 3) == 0;
#pragma unroll
        for (int r = 0; r < RM; ++r)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = m0 + ty * 4 + r * (BM / RM) + i;
                if (row >= p.M) continue;
                float* prow = P + (int64_t)row * p.N;
#pragma unroll
                for (int c = 0; c < RN; ++c) {
                    const int col = n0 + tx * 4 + c * (BN / RN);
                    const float* v = &acc[r * 4 + i][c * 4];
                    if (vec && col + 3 < p.N) {
                        *reinterpret_cast<float4*>(prow + col) = make_float4(v[0], v[1], v[2], v[3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (col + j < p.N) prow[col + j] = v[j];
                    }
                }
            }
        return;
    }

    // epilogue: bias, ReLU, store
#pragma unroll
    for (int r = 0; r < RM; ++r) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = m0 + ty * 4 + r * (BM / RM) + i;
            if (row >= p.M) continue;
            float* crow = C + (int64_t)row * p.ldc;
            const float* arow = p.aux ? p.aux + (int64_t)b * p.stride_aux + (int64_t)row * p.ld_aux : nullptr;
#pragma unroll
            for (int c = 0; c < RN; ++c) {
                const int col = n0 + tx * 4 + c * (BN / RN);
                float v[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float x = acc[r * 4 + i][c * 4 + j];
                    if (p.bias && col + j < p.N) x += __ldg(p.bias + (p.bias_row ? row : col + j));
                    if (p.relu) x = fmaxf(x, 0.0f);
                    if (arow && col + j < p.N && !(__ldg(arow + col + j) > 0.0f)) x = 0.0f;
                    v[j] = x;
                }
                if (p.vecC && col + 3 < p.N) {
                    *reinterpret_cast<float4*>(crow + col) = make_float4(v[0], v[1], v[2], v[3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (col + j < p.N) crow[col + j] = v[j];
                }
            }
        }
    }
}

template <int BM, int BN, int BK, int RM, int RN>
static void launch_cfg(const Params& p, int batch, bool TA, bool TB, cudaStream_t s) {
    constexpr int threads = (BM / (4 * RM)) * (BN / (4 * RN));
    dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM, batch * p.kslices);
    ProfScope prof(s, KID_FFMA_GEMM);
    // a programmatic dependent of whatever precedes it on the stream (the
    // kernel waits for it before its first load)
    if (!TA && !TB) launch_dependent(ffma_gemm_kernel<BM, BN, BK, RM, RN, false, false>, grid, dim3(threads), 0, s, p);
    else if (!TA && TB) launch_dependent(ffma_gemm_kernel<BM, BN, BK, RM, RN, false, true>, grid, dim3(threads), 0, s, p);
    else if (TA && !TB) launch_dependent(ffma_gemm_kernel<BM, BN, BK, RM, RN, true, false>, grid, dim3(threads), 0, s, p);
    else launch_dependent(ffma_gemm_kernel<BM, BN, BK, RM, RN, true, true>, grid, dim3(threads), 0, s, p);
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

}  // namespace ffma

int ffma_gemm_run(const GemmArgs& a, cudaStream_t s) {
    using namespace ffma;
    Params p;
    p.M = a.M; p.N = a.N; p.K = a.K;
    p.A = a.A; p.lda = a.lda; p.strideA = a.strideA;
    p.B = a.B; p.ldb = a.ldb; p.strideB = a.strideB;
    p.C = a.C; p.ldc = a.ldc; p.strideC = a.strideC;
    p.bias = a.bias; p.bias_row = a.bias_row; p.relu = a.relu;
    p.aux = a.aux; p.ld_aux = a.ld_aux; p.stride_aux = a.stride_aux;
    p.vecA = aligned16(a.A) && (a.lda % 4 == 0) && (a.strideA % 4 == 0);
    p.vecB = aligned16(a.B) && (a.ldb % 4 == 0) && (a.strideB % 4 == 0);
    p.vecC = aligned16(a.C) && (a.ldc % 4 == 0) && (a.strideC % 4 == 0);
    if (a.batch > 65535) return set_status(JST_ERR_ARG, "ffma: batch > 65535");
    p.kslices = 1;
    p.kchunk = a.K;
    p.part = nullptr;
    // Large tiles once there are enough of them to fill the 148 SMs; 64 x 64
    // tiles (4 x 4 per thread) otherwise.
    const long long big_tiles = (long long)((a.M + 127) / 128) * ((a.N + 127) / 128) * a.batch;
    if (big_tiles >= 148) {
        launch_cfg<128, 128, 16, 2, 2>(p, a.batch, a.transA, a.transB, s);
        if (cudaPeekAtLastError() != cudaSuccess) return set_status(JST_ERR_CUDA, "ffma_gemm_kernel launch failed");
        return JST_OK;
    }
    const SplitK sk = ffma_split_k(a);
    p.kslices = sk.slices;
    p.kchunk = sk.chunk;
    void* ws = nullptr;
    if (p.kslices > 1) {
        const int rc = workspace_alloc(ffma_workspace_bytes(a), s, &ws);
        if (rc) return rc;
        p.part = static_cast<float*>(ws);
    }
    launch_cfg<64, 64, 16, 1, 1>(p, a.batch, a.transA, a.transB, s);
    if (cudaPeekAtLastError() != cudaSuccess) {
        if (ws) workspace_free(ws, s);
        return set_status(JST_ERR_CUDA, "ffma_gemm_kernel launch failed");
    }
    if (p.kslices > 1) {
        const int rc = splitk_reduce_run(splitk_reduce_args(a, p.part, p.kslices), s);
        const int frc = workspace_free(ws, s);
        if (rc) return rc;
        if (frc) return frc;
    }
    return JST_OK;
}

// Split K for the 64 x 64 configuration: as many (tile, slice) CTAs as fit in
// one wave at two per SM (a second, partial wave would cost a whole tile
// time), slices of at least 64 along K, at most 16 slices.
SplitK ffma_split_k(const GemmArgs& a) {
    SplitK r{1, a.K};
    const long long big_tiles = (long long)((a.M + 127) / 128) * ((a.N + 127) / 128) * a.batch;
    if (big_tiles >= 148) return r;
    const long long tiles = (long long)((a.M + 63) / 64) * ((a.N + 63) / 64) * a.batch;
    const long long want = 2LL * 148 / tiles;
    const long long kmax = a.K / 64;
    long long S = std::min<long long>(std::min<long long>(want, kmax), 16);
    if (S <= 1 || a.batch * S > 65535) return r;
    int chunk = (int)((a.K + S - 1) / S);
    chunk = (chunk + 15) / 16 * 16;  // whole BK = 16 steps
    r.slices = (a.K + chunk - 1) / chunk;
    r.chunk = chunk;
    if (r.slices <= 1) r = SplitK{1, a.K};
    return r;
}

size_t ffma_workspace_bytes(const GemmArgs& a) {
    const SplitK sk = ffma_split_k(a);
    return sk.slices > 1 ? (size_t)sk.slices * a.batch * a.M * a.N * sizeof(float) : 0;
}

// ------------------------------------------------------------ K == 0 fill
__global__ void fill_epilogue_kernel(float* C, int M, int N, int64_t ldc, int64_t strideC, const float* bias,
                                     int bias_row, int relu) {
    const int b = blockIdx.z;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)M * N;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / N), c = (int)(i % N);
        float v = bias ? bias[bias_row ? r : c] : 0.0f;
        if (relu) v = fmaxf(v, 0.0f);
        C[(int64_t)b * strideC + (int64_t)r * ldc + c] = v;
    }
}

int fill_epilogue_run(const GemmArgs& a, cudaStream_t s) {
    const int64_t total = (int64_t)a.M * a.N;
    if (total == 0) return JST_OK;
    const int blocks = (int)((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
    ProfScope prof(s, KID_FILL);
    fill_epilogue_kernel<<<dim3(blocks, 1, a.batch), 256, 0, s>>>(a.C, a.M, a.N, a.ldc, a.strideC, a.bias, a.bias_row, a.relu);
    if (cudaPeekAtLastError() != cudaSuccess) return set_status(JST_ERR_CUDA, "fill kernel launch failed");
    return JST_OK;
}

}  // namespace jst
