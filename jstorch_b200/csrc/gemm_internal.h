// gemm_internal.h -- shared declarations between the kernels and the C ABI.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/jstorch_gemm.h"

namespace jst {

// Normalised, validated GEMM request (see jst_gemm_desc for the meaning).
struct GemmArgs {
    int transA, transB;
    int M, N, K, batch;
    const float* A; int64_t lda, strideA;
    const float* B; int64_t ldb, strideB;
    float* C; int64_t ldc, strideC;
    const float* bias;
    int bias_row;  // bias indexed by row (JST_EPI_BIAS_ROW*) instead of column
    int relu;
    const float* aux;  // JST_EPI_MASK: C *= (aux > 0)
    int64_t ld_aux, stride_aux;
};

// Check a public descriptor and normalise it into `a` (no device work).
int validate_gemm_desc(const jst_gemm_desc* d, GemmArgs* a);

// Whether launches on `s` may be programmatic dependents: not while `s` is
// being captured into a CUDA graph (a captured MLP step measured no faster
// with programmatic edges than with plain ones).
inline bool dependent_launch_ok(cudaStream_t s) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(s, &st) == cudaSuccess && st == cudaStreamCaptureStatusNone;
}

// Launch `kernel` as a programmatic dependent of the previous kernel on `s`:
// its blocks may be scheduled while that kernel drains, and the kernel must
// execute griddepcontrol.wait before touching global memory.  A plain launch
// under stream capture.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                    Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent_launch_ok(s) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Stream-ordered scratch from the library's per-device pool (checks the device first).
int workspace_alloc(size_t bytes, cudaStream_t s, void** out);
int workspace_free(void* p, cudaStream_t s);

// Record `status` with `msg` as the calling thread's last status; returns status.
int set_status(int status, const char* msg);

// Per-device error word written by kernels whose bounded waits gave up.
uint32_t* device_error_word();
// The separate timeout word of jst_gemm_tc_noalloc (a file-scope device
// variable, so that entry point allocates nothing): read-and-clear on device
// `dev` (0 when that entry point never ran there), and a host-side setter.
int noalloc_take_error(int dev, uint32_t* out);
int noalloc_set_error(int dev, uint32_t value);

// 3 x TF32 tcgen05 path
size_t tc_workspace_bytes(const GemmArgs& a);
int tc_gemm_run(const GemmArgs& a, void* workspace, cudaStream_t s);
// Split pass alone: `rows` x K operand rows (K-major source when kmajor, else
// stored [K, rows]) into hi / lo planes [batch][rows][Kp], Kp = K rounded up to 4.
int tc_split(const float* src, int kmajor, int64_t ld, int64_t sstride, int rows, int K, int batch, float* hi,
             float* lo, cudaStream_t s);
// Tensor-core kernel alone on existing planes (A planes M rows, B planes N rows).
// mc_store: C is the multicast view of a multicast-backed buffer; every tile
// is stored once through it and reaches every GPU of the team.
// a_bcast / b_bcast: that operand's planes hold one batch entry shared by all.
// split_a: a_hi is the raw K-major fp32 A (row stride lda_raw, batch stride
// strideA_raw, 16-byte aligned) and a_lo is unused; the kernel splits A tiles
// in shared memory (narrow tiles only).
// kslices > 1: split K into that many slices; C then receives the raw partial
// products part[slice][batch][M][N] (ldc = N, strideC = M * N, no epilogue) for
// splitk_reduce_run to combine.
// pdl: launch as a programmatic dependent of the previous kernel on `s` (the
// kernel's set-up overlaps that kernel's tail; it waits for its completion
// before touching global memory).
int tc_gemm_planes(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo, int M, int N, int K,
                   int batch, float* C, int64_t ldc, int64_t strideC, const float* bias, int relu, uint32_t* err,
                   cudaStream_t s, int mc_store = 0, const float* aux = nullptr, int64_t ld_aux = 0,
                   int64_t stride_aux = 0, int bias_row = 0, int a_bcast = 0, int b_bcast = 0, int kslices = 1,
                   int split_a = 0, int64_t lda_raw = 0, int64_t strideA_raw = 0, int pdl = 0);
// Tile width (64, 128 or 256 columns of C per CTA) the tensor-core kernel uses for a shape.
int tc_pick_bn(int M, int N, int K);
// split-K slices the tensor-core path uses for `a` (1: none)
int tc_split_k(const GemmArgs& a);

// FFMA SIMT path
int ffma_gemm_run(const GemmArgs& a, cudaStream_t s);
// split-K plan of the FFMA kernel (slices = 1: none) and its workspace size
struct SplitK {
    int slices, chunk;
};
SplitK ffma_split_k(const GemmArgs& a);
size_t ffma_workspace_bytes(const GemmArgs& a);

// K == 0: C = epilogue(0)
int fill_epilogue_run(const GemmArgs& a, cudaStream_t s);

// Free the pinned staging of jst_copy_h2d / jst_copy_d2h (hostio.cu).
int hostio_release();

// Reduce of a split-K GEMM (splitk.cu): C = epilogue(sum over slices of part).
struct SplitKReduce {
    const float* part;  // [slices][batch][M][N] packed
    int slices, batch, M, N;
    float* C;
    int64_t ldc, strideC;
    const float* bias;
    int bias_row, relu;
    const float* aux;
    int64_t ld_aux, stride_aux;
    int vecC;
};
SplitKReduce splitk_reduce_args(const GemmArgs& a, const float* part, int slices);
int splitk_reduce_run(const SplitKReduce& r, cudaStream_t s);

// ---- launch accounting / optional event timing (profile.cu)
enum KernelId {
    KID_TC_GEMM = 0,
    KID_SPLIT_ROWS,
    KID_SPLIT_TRANSPOSE,
    KID_FFMA_GEMM,
    KID_FILL,
    KID_CONV,  // im2col / col2im / permute of the convolution launchers
    KID_SPLITK_REDUCE,
    KID_RNN,  // GRU gate kernel
    KERNEL_ID_COUNT
};

// Construct immediately before a kernel launch and let it go out of scope
// right after: counts the launch and, when profiling is on, brackets it with
// CUDA events on stream `s`.
class ProfScope {
  public:
    ProfScope(cudaStream_t s, int kernel);
    ~ProfScope();
    ProfScope(const ProfScope&) = delete;
    ProfScope& operator=(const ProfScope&) = delete;

  private:
    cudaStream_t s_;
    int kernel_;
    void* ev0_ = nullptr;
    void* ev1_ = nullptr;
};

}  // namespace jst
