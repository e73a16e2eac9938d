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
//     skipped;
//   * for realistic sizes the recurrent product runs on the tensor cores as
//     ghT = W_hh . h^T: W_hh is split into tf32 planes once per call, the
//     GEMM is cut into K-slices so its few output tiles fill the SMs, and one
//     kernel sums the slices in order, adds b_hh, applies the gates and
//     writes h' both into the output sequence and as the tf32 hi / lo planes
//     the next step's GEMM reads (two launches per step).
// The gate arithmetic follows the reference op by op in fp32: sigmoid as
// 1 / (1 + __expf(-x)) and tanhf (native/ops/kernels.cuh:48-49), (1 - z) as
// (-z) + 1, and h' = ((1 - z) * n) + (z * h) with each product rounded.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/jstorch_rnn.h"
#include "gemm_internal.h"
#include "ptx.cuh"

namespace jst {
namespace {

__device__ __forceinline__ float sigmoid_ref(float x) { return 1.0f / (1.0f + __expf(-x)); }

constexpr int kMaxSlices = 16;  // K-slices of the recurrent GEMM (recurrent_slices caps at 16)

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

// Tensor-core step: ghT partials part[s][3H][batch] (K-slices of W_hh . h^T).
// A block of 256 threads takes 8 hidden units x 32 batch rows: it sums the
// slices in order and adds b_hh with 32 threads along the batch per hidden
// unit (128-byte reads of the [row][batch] partials), transposes through
// shared memory, then applies the gates with 8 threads along the hidden units
// per batch row (whole 32-byte sectors of gi, h and h').  Same arithmetic as
// gru_gate_kernel.  With nh_hi set it also writes the 3xTF32 split of h'
// into the [batch][Kp] planes of the next step's GEMM (the values the split
// pass would write; this step's GEMM has finished reading them).
__global__ void __launch_bounds__(256) gru_gate_t_kernel(const float* __restrict__ gi, const float* __restrict__ part,
                                                         int slices, const float* __restrict__ b_hh,
                                                         const float* __restrict__ h_prev, int64_t ld_prev,
                                                         float* __restrict__ h_out, int64_t ld_out, int batch, int H,
                                                         float* __restrict__ nh_hi, float* __restrict__ nh_lo, int Kp) {
    __shared__ float g[3][8][33];  // [gate][hidden unit][batch row]
    ptx::griddep_wait();  // launched as a programmatic dependent of the step's GEMM
    const int j0 = blockIdx.x * 8, b0 = blockIdx.y * 32;
    const int64_t plane = 3LL * H * batch;
    const int t = threadIdx.x;
    {
        const int bl = t & 31, jl = t >> 5;  // sum phase: batch fastest
        const int j = j0 + jl, b = b0 + bl;
        float acc[3] = {0.0f, 0.0f, 0.0f};
        if (j < H && b < batch) {
            // all slice loads first (independent), then the sums in slice order
            float v[3][kMaxSlices];
#pragma unroll
            for (int sl = 0; sl < kMaxSlices; ++sl)
#pragma unroll
                for (int gate = 0; gate < 3; ++gate)
                    v[gate][sl] = sl < slices ? part[sl * plane + (int64_t)(gate * H + j) * batch + b] : 0.0f;
#pragma unroll
            for (int sl = 0; sl < kMaxSlices; ++sl)
#pragma unroll
                for (int gate = 0; gate < 3; ++gate)
                    if (sl < slices) acc[gate] += v[gate][sl];
            if (b_hh)
#pragma unroll
                for (int gate = 0; gate < 3; ++gate) acc[gate] = __fadd_rn(acc[gate], b_hh[gate * H + j]);
        }
#pragma unroll
        for (int gate = 0; gate < 3; ++gate) g[gate][jl][bl] = acc[gate];
    }
    __syncthreads();
    const int jl = t & 7, bl = t >> 3;  // gate phase: hidden unit fastest
    const int j = j0 + jl, b = b0 + bl;
    if (b >= batch || j >= H) return;
    const float* gib = gi + (int64_t)b * 3 * H;
    const float r = sigmoid_ref(__fadd_rn(gib[j], g[0][jl][bl]));
    const float z = sigmoid_ref(__fadd_rn(gib[H + j], g[1][jl][bl]));
    const float n = tanhf(__fadd_rn(gib[2 * H + j], __fmul_rn(r, g[2][jl][bl])));
    const float h = h_prev[(int64_t)b * ld_prev + j];
    const float one_minus_z = __fadd_rn(-z, 1.0f);
    const float hv = __fadd_rn(__fmul_rn(one_minus_z, n), __fmul_rn(z, h));
    h_out[(int64_t)b * ld_out + j] = hv;
    if (nh_hi) {
        const float hi = ptx::to_tf32(hv);
        nh_hi[(int64_t)b * Kp + j] = hi;
        nh_lo[(int64_t)b * Kp + j] = ptx::to_tf32(hv - hi);
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

// Recurrent GEMM on the tensor cores: worth it once the step's product is
// large enough to cover the split of h and the reduce.
bool use_tc_recurrent(int batch, int H) {
    return H >= 128 && batch >= 8 && (double)3 * H * H * batch >= (double)(1 << 24);
}

// K-slices for ghT = W_hh . h^T (M = 3H, N = batch): fill the SMs with
// (tile, slice) CTAs, slices of at least 4 BK steps; normalised so that no
// slice is empty.
int recurrent_slices(int batch, int H) {
    const int bn = tc_pick_bn(3 * H, batch, H);
    const int tiles = ((3 * H + 127) / 128) * ((batch + bn - 1) / bn);
    const int num_kb = (H + 15) / 16;
    int S = std::min(std::min(148 / std::max(tiles, 1), num_kb / 4), 16);
    if (S <= 1) return 1;
    const int per = (num_kb + S - 1) / S;
    return (num_kb + per - 1) / per;
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
    const bool tc = use_tc_recurrent(batch, hidden);
    const int Kp = (hidden + 3) & ~3;
    const int S = tc ? recurrent_slices(batch, hidden) : 1;
    // workspace: gi [seq][batch][3H]; gh [batch][3H]; tensor-core path: W_hh
    // planes [3H][Kp] x2, h planes [batch][Kp] x2, partials [S][3H][batch]
    // every region starts on a 256-byte boundary (the planes are TMA sources)
    auto up = [](size_t n) { return (n + 63) & ~size_t(63); };
    const size_t n_gi = up((size_t)rows * G), n_gh = up((size_t)batch * G);
    const size_t n_w = tc ? up((size_t)G * Kp) : 0, n_h = tc ? up((size_t)batch * Kp) : 0;
    const size_t n_part = tc ? up((size_t)S * G * batch) : 0;
    void* ws = nullptr;
    int rc = workspace_alloc((n_gi + n_gh + 2 * n_w + 2 * n_h + n_part) * sizeof(float), s, &ws);
    if (rc) return rc;
    float* gi = static_cast<float*>(ws);  // [seq][batch][3H]
    float* gh = gi + n_gi;                // [batch][3H]
    float* w_hi = gh + n_gh;
    float* w_lo = w_hi + n_w;
    float* h_hi = w_lo + n_w;
    float* h_lo = h_hi + n_h;
    float* part = h_lo + n_h;
    // all input projections at once (nn.js:480 for every step)
    rc = nt_gemm(x, input_size, w_ih, b_ih, gi, (int)rows, (int)G, input_size, s);
    // W_hh is the same at every step: split it once
    if (!rc && tc) rc = tc_split(w_hh, 1, hidden, 0, (int)G, hidden, 1, w_hi, w_lo, s);
    const float* h_prev = h0;  // row stride `hidden` for h0, ld_out for rows of `out`
    int64_t ld_prev = hidden;
    bool h_split = false;  // h_hi / h_lo hold the split of h_prev
    for (int step = 0; step < seq && !rc; ++step) {
        const int t = reverse ? seq - 1 - step : step;
        float* h_out = out + (int64_t)t * batch * ld_out;
        const float* git = gi + (int64_t)t * batch * G;
        if (h_prev && tc) {
            // nn.js:481 as ghT[3H][batch] = W_hh . h^T on the tensor cores, split over K,
            // the slices summed with b_hh and the gates in one kernel
            if (!h_split) rc = tc_split(h_prev, 1, ld_prev, 0, batch, hidden, 1, h_hi, h_lo, s);
            if (!rc)
                rc = tc_gemm_planes(w_hi, w_lo, h_hi, h_lo, (int)G, batch, hidden, 1, part, batch, G * batch, nullptr,
                                    0, device_error_word(), s, 0, nullptr, 0, 0, 0, 0, 0, S, 0, 0, 0, /*pdl=*/1);
            if (!rc) {
                {
                    ProfScope prof(s, KID_RNN);
                    const bool more = step + 1 < seq;
                    // a programmatic dependent of the GEMM: its blocks are
                    // scheduled while the GEMM drains and wait for it in-kernel
                    if (launch_dependent(gru_gate_t_kernel, dim3((hidden + 7) / 8, (batch + 31) / 32), dim3(256), 0, s,
                                         git, (const float*)part, S, b_hh, h_prev, ld_prev, h_out, ld_out, batch,
                                         hidden, more ? h_hi : nullptr, more ? h_lo : nullptr, Kp) != cudaSuccess)
                        rc = set_status(JST_ERR_CUDA, "gru gate launch failed");
                    h_split = more;
                }
                if (!rc && cudaPeekAtLastError() != cudaSuccess) rc = set_status(JST_ERR_CUDA, "gru gate launch failed");
            }
        } else {
            h_split = false;
            const float* ghp = nullptr;
            if (h_prev) {  // nn.js:481
                rc = nt_gemm(h_prev, ld_prev, w_hh, b_hh, gh, batch, (int)G, hidden, s);
                if (rc) break;
                ghp = gh;
            }
            rc = gate(git, ghp, b_hh, h_prev, ld_prev, h_out, ld_out, batch, hidden, s);
        }
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
