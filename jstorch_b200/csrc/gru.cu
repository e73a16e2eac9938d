// gru.cu -- jst_gru_layer_forward: one layer and direction of the reference's
// GRU (src/nn.js:451-536) on this library's GEMMs.
//
// The reference runs, per time step, _cell (nn.js:477-485):
//   gi = x_t . W_ih^T + b_ih            gh = h . W_hh^T + b_hh
//   r = sigmoid(gi_r + gh_r)             z = sigmoid(gi_z + gh_z)
//   n = tanh(gi_n + r * gh_n)            h' = (1 - z) * n + z * h
// with every op a separate kernel (two GEMMs, three slices, adds, muls,
// sigmoid, tanh).  Here:
//   * the input projections of all steps are ONE GEMM (they do not depend on
//     h): GI[seq*batch, 3H] = X . W_ih^T + b_ih, bias in the epilogue;
//   * per step, one NT GEMM gh = h . W_hh^T + b_hh (bias in the epilogue) and
//     one fused gate kernel that reads gi, gh and h and writes h' straight
//     into the output sequence, which is also the next step's h;
//   * at the first step with no initial state, gh = b_hh and the GEMM is
//     skipped.
// The gate arithmetic follows the reference op by op in fp32: sigmoid as
// 1 / (1 + __expf(-x)) and tanhf (native/ops/kernels.cuh:48-49), (1 - z) as
// (-z) + 1, and h' = ((1 - z) * n) + (z * h) with each product rounded.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/jstorch_rnn.h"
#include "gemm_internal.h"

namespace jst {
namespace {

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + __expf(-x)); }

// h_out[b][j] from gi[b][{j, H+j, 2H+j}], gh[b][...] (or b_hh when gh is
// null) and h_prev[b][j] (or 0 when null).
__global__ void gru_gate_kernel(const float* __restrict__ gi, const float* __restrict__ gh,
                                const float* __restrict__ b_hh, const float* __restrict__ h_prev, int64_t ld_prev,
                                float* __restrict__ h_out, int64_t ld_out, int batch, int H) {
    const int64_t total = (int64_t)batch * H;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(i / H), j = (int)(i - (int64_t)b * H);
        const float* gib = gi + (int64_t)b * 3 * H;
        float ghr, ghz, ghn;
        if (gh) {
            const float* ghb = gh + (int64_t)b * 3 * H;
            ghr = ghb[j];
            ghz = ghb[H + j];
            ghn = ghb[2 * H + j];
        } else {
            ghr = b_hh ? b_hh[j] : 0.0f;
            ghz = b_hh ? b_hh[H + j] : 0.0f;
            ghn = b_hh ? b_hh[2 * H + j] : 0.0f;
        }
        const float r = sigmoid_ref(__fadd_rn(gib[j], ghr));
        const float z = sigmoid_ref(__fadd_rn(gib[H + j], ghz));
        const float n = tanhf(__fadd_rn(gib[2 * H + j], __fmul_rn(r, ghn)));
        const float h = h_prev ? h_prev[(int64_t)b * ld_prev + j] : 0.0f;
        const float one_minus_z = __fadd_rn(-z, 1.0f);
        h_out[(int64_t)b * ld_out + j] = __fadd_rn(__fmul_rn(one_minus_z, n), __fmul_rn(z, h));
    }
}

int gate(const float* gi, const float* gh, const float* b_hh, const float* h_prev, int64_t ld_prev, float* h_out,
         int64_t ld_out, int batch, int H, cudaStream_t s) {
    const int64_t total = (int64_t)batch * H;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    {
        ProfScope prof(s, KID_RNN);
        gru_gate_kernel<<<blocks, 256, 0, s>>>(gi, gh, b_hh, h_prev, ld_prev, h_out, ld_out, batch, H);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, "gru gate launch failed");
}

// C[M, 3H] = A[M, K] . W^T (+ bias), W stored [3H, K]
int nt_gemm(const float* A, int64_t lda, const float* W, const float* bias, float* C, int M, int N, int K,
            cudaStream_t s) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, A, W, C);
    d.lda = lda;
    d.transB = 1;
    d.ldb = K;
    d.bias = bias;
    d.epilogue = bias ? JST_EPI_BIAS : JST_EPI_NONE;
    d.stream = reinterpret_cast<jst_stream_t>(s);
    return jst_gemm_ex(&d);
}

}  // namespace
}  // namespace jst

extern "C" int jst_gru_layer_forward(const float* x, int seq, int batch, int input_size, int hidden,
                                     const float* w_ih, const float* w_hh, const float* b_ih, const float* b_hh,
                                     const float* h0, int reverse, float* out, int64_t ld_out, float* h_n,
                                     jst_stream_t stream) {
    using namespace jst;
    if (seq < 0 || batch < 0 || input_size < 0 || hidden < 0)
        return set_status(JST_ERR_ARG, "gru: negative size");
    if (ld_out < hidden) return set_status(JST_ERR_ARG, "gru: ld_out < hidden");
    const int64_t rows = (int64_t)seq * batch, G = 3LL * hidden;
    if (rows > 0x7fffffffLL || G > 0x7fffffffLL) return set_status(JST_ERR_ARG, "gru: size exceeds int");
    if (seq == 0 || batch == 0 || hidden == 0) {
        if (h_n && batch && hidden && seq == 0 && h0)
            return set_status(cudaMemcpyAsync(h_n, h0, (size_t)batch * hidden * 4, cudaMemcpyDeviceToDevice,
                                              reinterpret_cast<cudaStream_t>(stream)) == cudaSuccess
                                  ? JST_OK
                                  : JST_ERR_CUDA,
                              "gru: h_n copy");
        return set_status(JST_OK, nullptr);
    }
    if (!x || !w_ih || !w_hh || !out) return set_status(JST_ERR_ARG, "gru: null pointer");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    void* ws = nullptr;
    int rc = workspace_alloc((size_t)(rows + batch) * G * sizeof(float), s, &ws);
    if (rc) return rc;
    float* gi = static_cast<float*>(ws);  // [seq][batch][3H]
    float* gh = gi + rows * G;            // [batch][3H]
    // all input projections at once (nn.js:480 for every step)
    rc = nt_gemm(x, input_size, w_ih, b_ih, gi, (int)rows, (int)G, input_size, s);
    const float* h_prev = h0;  // row stride `hidden` for h0, ld_out for rows of `out`
    int64_t ld_prev = hidden;
    for (int step = 0; step < seq && !rc; ++step) {
        const int t = reverse ? seq - 1 - step : step;
        const float* ghp = nullptr;
        if (h_prev) {  // nn.js:481
            rc = nt_gemm(h_prev, ld_prev, w_hh, b_hh, gh, batch, (int)G, hidden, s);
            if (rc) break;
            ghp = gh;
        }
        float* h_out = out + (int64_t)t * batch * ld_out;
        rc = gate(gi + (int64_t)t * batch * G, ghp, b_hh, h_prev, ld_prev, h_out, ld_out, batch, hidden, s);
        h_prev = h_out;
        ld_prev = ld_out;
    }
    if (!rc && h_n)
        rc = cudaMemcpy2DAsync(h_n, (size_t)hidden * 4, h_prev, (size_t)ld_prev * 4, (size_t)hidden * 4, batch,
                               cudaMemcpyDeviceToDevice, s) == cudaSuccess
                 ? JST_OK
                 : set_status(JST_ERR_CUDA, "gru: h_n copy");
    const int frc = workspace_free(ws, s);
    if (rc) return rc;
    return frc ? frc : set_status(JST_OK, nullptr);
}
