/*
 * jstorch_gemm.h -- C ABI of the B200 (sm_100a) fp32 GEMM library that
 * replaces JsTorch's cuBLAS matmul path.
 *
 * Library: jstorch_b200/libjstorch_gemm.so.  Plain C linkage, plain pointers
 * and sizes.  All matrices are fp32 and row-major, as in JsTorch.
 *
 * Reference interfaces replaced (paths relative to the JsTorch project root):
 *   launch_matmul  native/ops/matmul.cu:28   (declared native/core/tensor.cpp:69)
 *   launch_bmm     native/ops/matmul.cu:40   (declared native/core/tensor.cpp:71)
 *   launch_linear  native/ops/matmul.cu:54   (declared native/core/tensor.cpp:70)
 * They keep the reference signatures and `void` return, so tensor.cpp links
 * against this library unchanged; their status is readable afterwards through
 * jst_get_last_status().  Everything else here is new surface that the
 * reference does not have (it has no status codes, no NT/TN forms, no
 * epilogue options and no multi-GPU path).
 */
#ifndef JSTORCH_GEMM_H
#define JSTORCH_GEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers (same type). */
typedef struct CUstream_st* jst_stream_t;

/* ---------------------------------------------------------------- status */
typedef enum jst_status {
    JST_OK = 0,
    JST_ERR_ARG = 1,          /* bad shape, stride, pointer or enum value        */
    JST_ERR_ALIGN = 2,        /* a forced kernel cannot take this alignment      */
    JST_ERR_CUDA = 3,         /* a CUDA runtime call or launch failed            */
    JST_ERR_NCCL = 4,         /* an NCCL call failed                             */
    JST_ERR_TIMEOUT = 5,      /* a bounded device or host wait gave up           */
    JST_ERR_UNSUPPORTED = 6,  /* no kernel of this build can run the request     */
    JST_ERR_NOMEM = 7,        /* device or pinned host allocation failed         */
    JST_ERR_NO_DEVICE = 8     /* no CUDA device of compute capability 10.x       */
} jst_status;

/* Human-readable text of the last non-OK status raised on the calling thread. */
const char* jst_last_error(void);
/* Status of the last call made on the calling thread (for the void launchers). */
int jst_get_last_status(void);

/* ---------------------------------------------------------------- GEMM */
typedef enum jst_epilogue {
    JST_EPI_NONE = 0,
    JST_EPI_BIAS = 1,       /* C[i,j] = acc + bias[j]            */
    JST_EPI_RELU = 2,       /* C[i,j] = max(acc, 0)              */
    JST_EPI_BIAS_RELU = 3,  /* C[i,j] = max(acc + bias[j], 0)    */
    JST_EPI_MASK = 4,       /* C[i,j] = acc * (aux[i,j] > 0 ? 1 : 0): the ReLU
                               backward of the layer whose output is aux, fused
                               into the GEMM that produces its upstream gradient */
    JST_EPI_BIAS_ROW = 8,   /* C[i,j] = acc + bias[i]  (bias [M]: one value per
                               output channel of a convolution)              */
    JST_EPI_BIAS_ROW_RELU = 10  /* C[i,j] = max(acc + bias[i], 0)            */
} jst_epilogue;

typedef enum jst_kernel {
    JST_KERNEL_AUTO = 0,      /* shape heuristic                                  */
    JST_KERNEL_TC3XTF32 = 1,  /* tcgen05/TMEM split-precision (3 x TF32) kernel   */
    JST_KERNEL_FFMA = 2       /* fp32 FFMA SIMT kernel                            */
} jst_kernel;

/*
 * C[b] = epilogue( op(A[b]) * op(B[b]) ),  b = 0 .. batch-1
 *   op(A) is [M, K]: transA = 0 -> A stored [M, K] (lda >= K),
 *                    transA = 1 -> A stored [K, M] (lda >= M).
 *   op(B) is [K, N]: transB = 0 -> B stored [K, N] (ldb >= N),
 *                    transB = 1 -> B stored [N, K] (ldb >= K).
 *   C is [M, N] with ldc >= N.  Strides are in elements; batch strides may be 0
 *   (broadcast operand).  All pointers are device pointers of the current device.
 *   The call is asynchronous on `stream` (NULL = legacy default stream, as the
 *   reference uses).  M, N or K of 0 is legal: K == 0 writes epilogue(0).
 */
typedef struct jst_gemm_desc {
    int transA, transB;
    int M, N, K;
    const float* A; int64_t lda; int64_t strideA;
    const float* B; int64_t ldb; int64_t strideB;
    float* C;       int64_t ldc; int64_t strideC;
    int batch;                 /* >= 1                                            */
    const float* bias;         /* [N] (or [M] for *_BIAS_ROW*), required for the bias epilogues */
    int epilogue;              /* jst_epilogue                                    */
    int kernel;                /* jst_kernel                                      */
    jst_stream_t stream;
    const float* aux;          /* JST_EPI_MASK: [batch][M][N] with ld_aux, stride_aux */
    int64_t ld_aux; int64_t stride_aux;
} jst_gemm_desc;

/* Fill a descriptor for a packed row-major C = A*B (NN, batch 1, no epilogue). */
void jst_gemm_desc_init(jst_gemm_desc* d, int M, int N, int K,
                        const float* A, const float* B, float* C);

int jst_gemm_ex(const jst_gemm_desc* d);

/* Which kernel JST_KERNEL_AUTO would run for `d` (JST_KERNEL_TC3XTF32 or _FFMA). */
int jst_gemm_select_kernel(const jst_gemm_desc* d);

/*
 * jst_gemm_tc_noalloc -- the tensor-core (3 x TF32) GEMM of jst_gemm_ex
 * without any device allocation.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: hosts whose device memory belongs
 * to another allocator that forbids side allocations, embedders that budget
 * all device memory up front, and latency-critical code that cannot afford
 * cudaMalloc / cudaFree (they may synchronise the whole device).
 * jst_gemm_ex takes its scratch (the hi/lo split planes) from a pool it
 * allocates; this entry point uses a fixed 64 MiB file-scope device array
 * instead, and calls no cudaMalloc, cudaFree or other allocating routine.
 *   - Same descriptor and result as jst_gemm_ex with kernel = TC3XTF32
 *     (`kernel` must be AUTO or TC3XTF32).  The caller passes A, B, C, bias.
 *   - Limit: the tensor-core path's scratch must fit 64 MiB: hi/lo planes of
 *     2 * Kp * (M * Ba + N * Bb) * 4 bytes (Kp = K rounded up to a multiple
 *     of 4; Ba, Bb = batch, or 1 for an operand with batch stride 0; Ba = 0
 *     when the kernel splits a K-major A itself, as it does for outputs at
 *     most 128 columns wide or K <= 256), plus S * batch * M * N * 4 bytes of
 *     split-K partials when the output tiles fill less than half the SMs
 *     (e.g. 2048^3 fits exactly); larger requests return JST_ERR_ARG without
 *     launching.
 *   - The array exists once per device, for the life of the process, and is
 *     shared by all calls: calls whose work overlaps on the GPU (different
 *     streams or threads) race and must be serialised by the caller.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *     cudaDeviceReset() is not supported after that (the address is cached).
 *   - A pipeline wait that timed out is reported by jst_device_error(), as on
 *     the allocating path.
 */
int jst_gemm_tc_noalloc(const jst_gemm_desc* d);

/* ------------------------------------------- reference-compatible launchers */
/* native/ops/matmul.cu:28 -- row-major [M,K] x [K,N] -> [M,N] */
void launch_matmul(const float* a, const float* b, float* c, int M, int K, int N, jst_stream_t s);
/* native/ops/matmul.cu:40 -- [B,M,K] x [B,K,N] -> [B,M,N], packed strides */
void launch_bmm(const float* a, const float* b, float* c, int B, int M, int K, int N, jst_stream_t s);
/* native/ops/matmul.cu:54 -- out[B,out_f] = x[B,in_f] * w[out_f,in_f]^T + bias (nullable) */
void launch_linear(const float* x, const float* w, const float* bias, float* out,
                   int B, int in_f, int out_f, jst_stream_t s);

/* --------------------------------------------- torch.matmul(a, b, M, K, N) */
/*
 * README.md:37-84 of the reference documents torch.matmul(a, b, M, K, N) on
 * row-major Float32Array returning a Float32Array; the code base never
 * implemented it.  This is the native entry point an N-API shim binds: HOST
 * pointers in and out (pageable or pinned), device buffers cached per device,
 * computed on the current device, synchronous on return.  Large products are
 * moved in row chunks so that the host->device copies, the GEMM and the
 * device->host copy overlap.  c must hold M*N floats.
 */
int jst_matmul_host(const float* a, const float* b, float* c, int M, int K, int N);

/*
 * Stream-ordered form of jst_matmul_host (no counterpart in the reference):
 * enqueues the host->device copies, the GEMM and the device->host copy on
 * `stream` (NULL = the legacy default stream) and returns.  With pinned (page-locked) host buffers the call is
 * asynchronous and `c` is valid once the stream reaches that point; with
 * pageable buffers the copies synchronise as cudaMemcpyAsync does.  The
 * device staging buffers are per device: a call on one stream waits on the
 * GPU (not on the host) until the previous call, on any stream, has finished
 * with them, so calls on different streams of a device take turns rather
 * than overlap.
 */
int jst_matmul_host_async(const float* a, const float* b, float* c, int M, int K, int N, jst_stream_t stream);

/* ------------------------------------------ host <-> device transfers */
/*
 * The copies either side of the path: what Tensor::from_array / from_buffer
 * (native/core/tensor.cpp:740-750, a synchronous pageable cudaMemcpy) and
 * Tensor::to_array (tensor.cpp:775-800, cudaDeviceSynchronize + copy) do, for
 * an N-API shim that passes the Float32Array's storage directly.
 * Pageable host memory is staged through two pinned 8 MiB chunks per device
 * (host copy of one chunk overlapping the DMA of the other); page-locked host
 * memory is copied by one direct DMA.
 *   jst_copy_h2d: returns once `src_host` has been read (the caller may reuse
 *     it); the device data is ready in `stream` order.
 *   jst_copy_d2h: ordered after earlier work on `stream`; waits for that
 *     stream only, and returns when `dst_host` holds the data.
 * Calls on one device share its staging chunks and are serialised.
 */
int jst_copy_h2d(void* dst_device, const void* src_host, size_t bytes, jst_stream_t stream);
int jst_copy_d2h(void* dst_host, const void* src_device, size_t bytes, jst_stream_t stream);

/* ---------------------------------------------------- device-side status */
/*
 * Kernels never trap: a pipeline wait that exceeds its bound sets a device
 * error word and the kernel exits.  jst_device_error() synchronises the
 * current device and returns (and clears) that word: 0 = none, 1 = timeout.
 * It covers every entry point of this library, jst_gemm_tc_noalloc included.
 */
int jst_device_error(void);

/*
 * Testing aid (no counterpart in the reference): set an error word of the
 * current device from the host, exactly as a kernel whose bounded wait gave
 * up would, so that a caller's handling of jst_device_error() can be tested
 * without stalling or faulting a GPU.  word 0: the word of the allocating
 * entry points; word 1: the word of jst_gemm_tc_noalloc.  JST_ERR_ARG for
 * any other value.
 */
int jst_test_set_device_error(int word);

/* Release cached device workspace and pinned staging buffers of this process
 * (including the jst_copy_h2d / jst_copy_d2h staging chunks). */
void jst_release_caches(void);

/* ------------------------------------------------------------ profiling */
/* (no counterpart in the reference, which has no tracing) */
typedef struct jst_kernel_stat {
    char name[32];       /* kernel family: tc_gemm, split_rows, ffma_gemm, ...  */
    int64_t launches;
    double total_ms;     /* summed device time between the bracketing events   */
} jst_kernel_stat;

/* Number of kernels this library has launched in the process so far. */
int64_t jst_launch_count(void);
/* on != 0: bracket every launch with CUDA events on its stream.  Resets stats. */
int jst_profile_enable(int on);
/* Wait for the recorded events and fill up to max_entries stats; returns the
 * number of kernel families seen (or -status on a CUDA error). */
int jst_profile_read(jst_kernel_stat* out, int max_entries);

#ifdef __cplusplus
}
#endif
#endif /* JSTORCH_GEMM_H */
