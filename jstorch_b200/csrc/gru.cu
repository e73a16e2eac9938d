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
// saved (training forward, else null): [batch][4H] rows of r, z, n and the
// n-gate's recurrent term gh_n, which the backward pass reads.
__global__ void gru_gate_kernel(const float* __restrict__ gi, const float* __restrict__ gh,
                                const float* __restrict__ b_hh, const float* __restrict__ h_prev, int64_t ld_prev,
                                float* __restrict__ h_out, int64_t ld_out, int batch, int H,
                                float* __restrict__ saved) {
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
        if (saved) {
            float* sv = saved + (int64_t)b * 4 * H;
            sv[j] = r;
            sv[H + j] = z;
            sv[2 * H + j] = n;
            sv[3 * H + j] = ghn;
        }
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
                                                         float* __restrict__ nh_hi, float* __restrict__ nh_lo, int Kp,
                                                         float* __restrict__ saved) {
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
    if (saved) {
        float* sv = saved + (int64_t)b * 4 * H;
        sv[j] = r;
        sv[H + j] = z;
        sv[2 * H + j] = n;
        sv[3 * H + j] = g[2][jl][bl];
    }
    if (nh_hi) {
        const float hi = ptx::to_tf32(hv);
        nh_hi[(int64_t)b * Kp + j] = hi;
        nh_lo[(int64_t)b * Kp + j] = ptx::to_tf32(hv - hi);
    }
}

// ------------------------------------------------------------------ backward
// One step of back-propagation through time for the cell of nn.js:477-485,
// the gradients GradTensor's closures produce for its ops (sigmoid, tanh,
// mul, add, slice; native/core/autograd.hpp) composed for one (b, j):
//   g   = dL/dh'  = dout_t + (z' g')_next + (dgh_next . W_hh)
//   dn  = g (1 - z)        dz = g (h - n)        dh_direct = g z
//   da_n = dn (1 - n^2)    da_r = (da_n gh_n) r (1 - r)    da_z = dz z (1 - z)
//   dgi = (da_r, da_z, da_n)        dgh = (da_r, da_z, da_n r)
// `part` holds S slices of P = dgh_next . W_hh with element (b, j) of slice
// sl at part[sl * plane + j * sj + b * sb] (the tensor-core path's [H][batch]
// partials, or one [batch][H] product), or is null at the first backward
// step.  A block takes 8 hidden units x 32 batch rows: it sums the slices in
// order with batch fastest (128-byte reads of the [H][batch] partials),
// transposes through shared memory, then works with 8 threads along the
// hidden units per batch row (whole 32-byte sectors of the [batch][..] rows).
// With p_hi set it also writes the tf32 hi / lo split of dgh into the
// [batch][Kp3] planes the next step's GEMM reads.
__global__ void __launch_bounds__(256) gru_gate_bwd_kernel(
    const float* __restrict__ part, int slices, int64_t plane, int64_t sj, int64_t sb,
    const float* __restrict__ carry_in, const float* __restrict__ dout, int64_t ld_dout,
    const float* __restrict__ saved, const float* __restrict__ h_prev, int64_t ld_prev, float* __restrict__ dgi,
    float* __restrict__ dgh, float* __restrict__ carry_out, float* __restrict__ p_hi, float* __restrict__ p_lo,
    int Kp3, int batch, int H) {
    __shared__ float ps[8][33];  // [hidden unit][batch row]
    ptx::griddep_wait();  // a programmatic dependent of the step's GEMM
    const int j0 = blockIdx.x * 8, b0 = blockIdx.y * 32;
    const int t = threadIdx.x;
    {
        const int bl = t & 31, jl = t >> 5;  // sum phase: batch fastest
        const int j = j0 + jl, b = b0 + bl;
        float acc = 0.0f;
        if (part && j < H && b < batch) {
            float v[kMaxSlices];
#pragma unroll
            for (int sl = 0; sl < kMaxSlices; ++sl) v[sl] = sl < slices ? part[sl * plane + j * sj + b * sb] : 0.0f;
#pragma unroll
            for (int sl = 0; sl < kMaxSlices; ++sl)
                if (sl < slices) acc += v[sl];
        }
        ps[jl][bl] = acc;
    }
    __syncthreads();
    const int jl = t & 7, bl = t >> 3;  // gate phase: hidden unit fastest
    const int j = j0 + jl, b = b0 + bl;
    if (b >= batch || j >= H) return;
    float g = ps[jl][bl];
    if (carry_in) g = __fadd_rn(g, carry_in[(int64_t)b * H + j]);
    if (dout) g = __fadd_rn(g, dout[(int64_t)b * ld_dout + j]);
    const float* sv = saved + (int64_t)b * 4 * H;
    const float r = sv[j], z = sv[H + j], n = sv[2 * H + j], ghn = sv[3 * H + j];
    const float hp = h_prev ? h_prev[(int64_t)b * ld_prev + j] : 0.0f;
    const float dn = __fmul_rn(g, __fadd_rn(1.0f, -z));
    const float dz = __fmul_rn(g, __fadd_rn(hp, -n));
    const float dan = __fmul_rn(dn, __fadd_rn(1.0f, -__fmul_rn(n, n)));
    const float dar = __fmul_rn(__fmul_rn(dan, ghn), __fmul_rn(r, __fadd_rn(1.0f, -r)));
    const float daz = __fmul_rn(dz, __fmul_rn(z, __fadd_rn(1.0f, -z)));
    const float dghn = __fmul_rn(dan, r);
    float* gi_row = dgi + (int64_t)b * 3 * H;
    float* gh_row = dgh + (int64_t)b * 3 * H;
    gi_row[j] = dar;
    gi_row[H + j] = daz;
    gi_row[2 * H + j] = dan;
    gh_row[j] = dar;
    gh_row[H + j] = daz;
    gh_row[2 * H + j] = dghn;
    carry_out[(int64_t)b * H + j] = __fmul_rn(g, z);
    if (p_hi) {
        float* hi = p_hi + (int64_t)b * Kp3;
        float* lo = p_lo + (int64_t)b * Kp3;
        const float v3[3] = {dar, daz, dghn};
#pragma unroll
        for (int gate = 0; gate < 3; ++gate) {
            const float h = ptx::to_tf32(v3[gate]);
            hi[gate * H + j] = h;
            lo[gate * H + j] = ptx::to_tf32(v3[gate] - h);
        }
    }
}

// dh0 = carry (z_0 g_0) + P (the S slices of dgh_0 . W_hh, layout as above);
// accumulate adds it to dh0's contents.
__global__ void gru_dh0_kernel(const float* __restrict__ part, int slices, int64_t plane, int64_t sj, int64_t sb,
                               const float* __restrict__ carry, float* __restrict__ dh0, int accumulate, int batch,
                               int H) {
    ptx::griddep_wait();
    const int64_t total = (int64_t)batch * H;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(i / H), j = (int)(i - (int64_t)b * H);
        float acc = 0.0f;
        for (int sl = 0; sl < slices; ++sl) acc += part[sl * plane + j * sj + b * sb];
        float v = __fadd_rn(acc, carry[i]);
        if (accumulate) v = __fadd_rn(dh0[i], v);
        dh0[i] = v;
    }
}

// Column sums of a [rows][cols] matrix in a fixed order (bit-identical
// reruns): pass 1 sums row chunks into partial[chunk][cols], pass 2 adds the
// chunks in order (and to out's contents when accumulating).
constexpr int kColsumRows = 256;
__global__ void colsum_partial_kernel(const float* __restrict__ a, int64_t rows, int cols,
                                      float* __restrict__ partial) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= cols) return;
    const int64_t r0 = (int64_t)blockIdx.y * kColsumRows;
    const int64_t r1 = std::min<int64_t>(r0 + kColsumRows, rows);
    float acc = 0.0f;
    for (int64_t r = r0; r < r1; ++r) acc += a[r * cols + j];
    partial[(int64_t)blockIdx.y * cols + j] = acc;
}

__global__ void colsum_final_kernel(const float* __restrict__ partial, int nchunks, int cols, float* __restrict__ out,
                                    int accumulate) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= cols) return;
    float acc = 0.0f;
    for (int c = 0; c < nchunks; ++c) acc += partial[(int64_t)c * cols + j];
    out[j] = accumulate ? __fadd_rn(out[j], acc) : acc;
}

// dst += src (n floats)
__global__ void accumulate_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __fadd_rn(dst[i], src[i]);
}

int gate(const float* gi, const float* gh, const float* b_hh, const float* h_prev, int64_t ld_prev, float* h_out,
         int64_t ld_out, int batch, int H, float* saved, cudaStream_t s) {
    const int64_t total = (int64_t)batch * H;
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
    {
        ProfScope prof(s, KID_RNN);
        gru_gate_kernel<<<blocks, 256, 0, s>>>(gi, gh, b_hh, h_prev, ld_prev, h_out, ld_out, batch, H, saved);
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

// K-slices of a recurrent product with few output tiles (M x N, reduction K):
// fill the SMs with (tile, slice) CTAs, slices of at least 4 BK steps;
// normalised so that no slice is empty.  Forward: ghT = W_hh . h^T (M = 3H,
// N = batch, K = H); backward: P^T = W_hh^T . dgh^T (M = H, N = batch, K = 3H).
int product_slices(int M, int N, int K) {
    const int bn = tc_pick_bn(M, N, K);
    const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
    const int num_kb = (K + 15) / 16;
    int S = std::min(std::min(148 / std::max(tiles, 1), num_kb / 4), kMaxSlices);
    if (S <= 1) return 1;
    const int per = (num_kb + S - 1) / S;
    return (num_kb + per - 1) / per;
}

int recurrent_slices(int batch, int H) { return product_slices(3 * H, batch, H); }

}  // namespace
}  // namespace jst

namespace jst {
namespace {
// One layer and direction forward; `saved` (null for inference) receives
// [seq][batch][4H] rows of r, z, n, gh_n for the backward pass.
int gru_forward_impl(const float* x, int seq, int batch, int input_size, int hidden, const float* w_ih,
                     const float* w_hh, const float* b_ih, const float* b_hh, const float* h0, int reverse, float* out,
                     int64_t ld_out, float* h_n, float* saved, jst_stream_t stream) {
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
                                         hidden, more ? h_hi : nullptr, more ? h_lo : nullptr, Kp,
                                         saved ? saved + (int64_t)t * batch * 4 * hidden : nullptr) != cudaSuccess)
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
            rc = gate(git, ghp, b_hh, h_prev, ld_prev, h_out, ld_out, batch, hidden,
                      saved ? saved + (int64_t)t * batch * 4 * hidden : nullptr, s);
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
}  // namespace
}  // namespace jst

extern "C" int jst_gru_layer_forward(const float* x, int seq, int batch, int input_size, int hidden,
                                     const float* w_ih, const float* w_hh, const float* b_ih, const float* b_hh,
                                     const float* h0, int reverse, float* out, int64_t ld_out, float* h_n,
                                     jst_stream_t stream) {
    return jst::gru_forward_impl(x, seq, batch, input_size, hidden, w_ih, w_hh, b_ih, b_hh, h0, reverse, out, ld_out,
                                 h_n, nullptr, stream);
}

extern "C" int jst_gru_layer_forward_train(const float* x, int seq, int batch, int input_size, int hidden,
                                           const float* w_ih, const float* w_hh, const float* b_ih, const float* b_hh,
                                           const float* h0, int reverse, float* out, int64_t ld_out, float* h_n,
                                           float* saved, jst_stream_t stream) {
    if (!saved && seq > 0 && batch > 0 && hidden > 0) return jst::set_status(JST_ERR_ARG, "gru: null saved buffer");
    return jst::gru_forward_impl(x, seq, batch, input_size, hidden, w_ih, w_hh, b_ih, b_hh, h0, reverse, out, ld_out,
                                 h_n, saved, stream);
}

namespace jst {
namespace {

int launch_ok(const char* what) {
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, what);
}

// Column sums of a [rows][cols] row-major matrix into out (added when accumulating).
int colsum(const float* a, int64_t rows, int cols, float* partial, float* out, int accumulate, cudaStream_t s) {
    const int nchunks = (int)((rows + kColsumRows - 1) / kColsumRows);
    {
        ProfScope prof(s, KID_RNN);
        colsum_partial_kernel<<<dim3((cols + 255) / 256, nchunks), 256, 0, s>>>(a, rows, cols, partial);
    }
    {
        ProfScope prof(s, KID_RNN);
        colsum_final_kernel<<<(cols + 255) / 256, 256, 0, s>>>(partial, nchunks, cols, out, accumulate);
    }
    return launch_ok("gru: column-sum launch failed");
}

// Run the GEMM `d` into dst (n floats, packed); when accumulating, into tmp
// first and then added to dst's contents.
int gemm_into(jst_gemm_desc d, float* dst, int64_t n, int accumulate, float* tmp, cudaStream_t s) {
    d.C = accumulate ? tmp : dst;
    int rc = jst_gemm_ex(&d);
    if (rc || !accumulate) return rc;
    {
        ProfScope prof(s, KID_RNN);
        const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
        accumulate_kernel<<<blocks, 256, 0, s>>>(dst, tmp, n);
    }
    return launch_ok("gru: accumulate launch failed");
}

int gru_backward_impl(const float* x, int seq, int batch, int input_size, int hidden, const float* w_ih,
                      const float* w_hh, const float* h0, int reverse, const float* out, int64_t ld_out,
                      const float* saved, const float* dout, int64_t ld_dout, const float* dh_n, float* dx,
                      float* dw_ih, float* dw_hh, float* db_ih, float* db_hh, float* dh0, int accumulate,
                      cudaStream_t s) {
    const int H = hidden;
    const int64_t rows = (int64_t)seq * batch, G = 3LL * H;
    const bool tc = use_tc_recurrent(batch, H);
    const int Kp3 = (int)((G + 3) & ~3LL);
    const int S = tc ? product_slices(H, batch, (int)G) : 1;
    auto up = [](size_t n) { return (n + 63) & ~size_t(63); };
    const size_t n_g = up((size_t)rows * G), n_hp = up((size_t)rows * H), n_c = up((size_t)batch * H);
    const size_t n_p = up(tc ? (size_t)S * H * batch : (size_t)batch * H);
    const size_t n_wt = tc ? up((size_t)H * Kp3) : 0, n_pl = tc ? up((size_t)batch * Kp3) : 0;
    const size_t n_cs = up((size_t)((rows + kColsumRows - 1) / kColsumRows) * G);
    const int acc_dx = (accumulate & JST_GRU_ACC_DX) != 0, acc_p = (accumulate & JST_GRU_ACC_PARAMS) != 0,
              acc_h = (accumulate & JST_GRU_ACC_DH0) != 0;
    const size_t n_tmp =
        (acc_dx || acc_p) ? up(std::max<size_t>((size_t)rows * input_size, (size_t)G * std::max(input_size, H))) : 0;
    void* ws = nullptr;
    int rc = workspace_alloc((2 * n_g + n_hp + 2 * n_c + n_p + 2 * n_wt + 2 * n_pl + n_cs + n_tmp) * sizeof(float), s,
                             &ws);
    if (rc) return rc;
    float* dgi = static_cast<float*>(ws);  // [seq][batch][3H]
    float* dgh = dgi + n_g;                // [seq][batch][3H]
    float* hp = dgh + n_g;                 // [seq][batch][H]: the state each step started from
    float* carry[2] = {hp + n_hp, hp + n_hp + n_c};
    float* P = carry[1] + n_c;
    float* wt_hi = P + n_p;
    float* wt_lo = wt_hi + n_wt;
    float* p_hi = wt_lo + n_wt;
    float* p_lo = p_hi + n_pl;
    float* cs_part = p_lo + n_pl;
    float* tmp = cs_part + n_cs;
    auto cuda_ok = [&](cudaError_t e, const char* what) -> int {
        if (e == cudaSuccess) return JST_OK;
        cudaGetLastError();
        return set_status(JST_ERR_CUDA, what);
    };
    // hp: step t started from out[t -/+ 1] (forward / reverse), the first
    // step processed from h0 (zeros when null)
    const int64_t blk = (int64_t)batch * H;
    const int t_first = reverse ? seq - 1 : 0;
    if (seq > 1)
        rc = cuda_ok(cudaMemcpy2DAsync(hp + (reverse ? 0 : blk), (size_t)H * 4, out + (reverse ? batch * ld_out : 0),
                                       (size_t)ld_out * 4, (size_t)H * 4, (size_t)(seq - 1) * batch,
                                       cudaMemcpyDeviceToDevice, s),
                     "gru: state copy");
    if (!rc)
        rc = h0 ? cuda_ok(cudaMemcpyAsync(hp + t_first * blk, h0, (size_t)blk * 4, cudaMemcpyDeviceToDevice, s),
                          "gru: h0 copy")
                : cuda_ok(cudaMemsetAsync(hp + t_first * blk, 0, (size_t)blk * 4, s), "gru: zero state");
    // W_hh^T as the A operand of P^T = W_hh^T . dgh^T, split once
    if (!rc && tc) rc = tc_split(w_hh, 0, H, 0, H, (int)G, 1, wt_hi, wt_lo, s);
    // the partials' layout: [S][H][batch] (tensor cores) or [batch][H] (one product)
    const int64_t plane = tc ? (int64_t)H * batch : blk, sj = tc ? batch : 1, sb = tc ? 1 : H;
    for (int step = seq - 1; step >= 0 && !rc; --step) {  // processing order, last step first
        const int t = reverse ? seq - 1 - step : step;
        const bool first = step == seq - 1;
        const bool need_product = step > 0 || dh0 != nullptr;
        float* dgh_t = dgh + (int64_t)t * batch * G;
        {
            ProfScope prof(s, KID_RNN);
            if (launch_dependent(gru_gate_bwd_kernel, dim3((H + 7) / 8, (batch + 31) / 32), dim3(256), 0, s,
                                 first ? (const float*)nullptr : (const float*)P, first ? 0 : S, plane, sj, sb,
                                 first ? dh_n : (const float*)carry[(step + 1) & 1],
                                 dout ? dout + (int64_t)t * batch * ld_dout : nullptr, ld_dout,
                                 saved + (int64_t)t * batch * 4 * H, (const float*)(hp + t * blk), (int64_t)H,
                                 dgi + (int64_t)t * batch * G, dgh_t, carry[step & 1],
                                 tc && need_product ? p_hi : nullptr, p_lo, Kp3, batch, H) != cudaSuccess)
                rc = set_status(JST_ERR_CUDA, "gru: backward gate launch failed");
        }
        if (!rc) rc = launch_ok("gru: backward gate launch failed");
        if (rc || !need_product) break;
        // P = dgh_t . W_hh (nn.js:481's matmul, backward: g . b^T with b = W_hh^T)
        if (tc) {
            rc = tc_gemm_planes(wt_hi, wt_lo, p_hi, p_lo, H, batch, (int)G, 1, P, batch, (int64_t)H * batch, nullptr,
                                0, device_error_word(), s, 0, nullptr, 0, 0, 0, 0, 0, S, 0, 0, 0, /*pdl=*/1);
        } else {
            jst_gemm_desc d;
            jst_gemm_desc_init(&d, batch, H, (int)G, dgh_t, w_hh, P);
            d.stream = reinterpret_cast<jst_stream_t>(s);
            rc = jst_gemm_ex(&d);
        }
    }
    if (!rc && dh0) {
        ProfScope prof(s, KID_RNN);
        const int blocks = (int)std::min<int64_t>((blk + 255) / 256, 148 * 8);
        if (launch_dependent(gru_dh0_kernel, dim3(blocks), dim3(256), 0, s, (const float*)P, S, plane, sj, sb,
                             (const float*)carry[0], dh0, acc_h, batch, H) != cudaSuccess)
            rc = set_status(JST_ERR_CUDA, "gru: dh0 launch failed");
    }
    if (!rc) rc = launch_ok("gru: dh0 launch failed");
    auto desc = [&](int M, int N, int K) {
        jst_gemm_desc d;
        jst_gemm_desc_init(&d, M, N, K, nullptr, nullptr, nullptr);
        d.stream = reinterpret_cast<jst_stream_t>(s);
        return d;
    };
    // dW_ih = dGI^T . X (all steps at once: one TN GEMM with K = seq * batch)
    if (!rc && dw_ih) {
        jst_gemm_desc d = desc((int)G, input_size, (int)rows);
        d.transA = 1; d.A = dgi; d.lda = G;
        d.B = x; d.ldb = input_size;
        rc = gemm_into(d, dw_ih, G * input_size, acc_p, tmp, s);
    }
    // dW_hh = dGH^T . Hprev
    if (!rc && dw_hh) {
        jst_gemm_desc d = desc((int)G, H, (int)rows);
        d.transA = 1; d.A = dgh; d.lda = G;
        d.B = hp; d.ldb = H;
        rc = gemm_into(d, dw_hh, G * H, acc_p, tmp, s);
    }
    if (!rc && db_ih) rc = colsum(dgi, rows, (int)G, cs_part, db_ih, acc_p, s);
    if (!rc && db_hh) rc = colsum(dgh, rows, (int)G, cs_part, db_hh, acc_p, s);
    // dX = dGI . W_ih
    if (!rc && dx) {
        jst_gemm_desc d = desc((int)rows, input_size, (int)G);
        d.A = dgi; d.lda = G;
        d.B = w_ih; d.ldb = input_size;
        rc = gemm_into(d, dx, rows * input_size, acc_dx, tmp, s);
    }
    const int frc = workspace_free(ws, s);
    if (rc) return rc;
    return frc ? frc : set_status(JST_OK, nullptr);
}

}  // namespace
}  // namespace jst

extern "C" int jst_gru_layer_backward(const float* x, int seq, int batch, int input_size, int hidden,
                                      const float* w_ih, const float* w_hh, const float* h0, int reverse,
                                      const float* out, int64_t ld_out, const float* saved, const float* dout,
                                      int64_t ld_dout, const float* dh_n, float* dx, float* dw_ih, float* dw_hh,
                                      float* db_ih, float* db_hh, float* dh0, int accumulate, jst_stream_t stream) {
    using namespace jst;
    if (seq < 0 || batch < 0 || input_size < 0 || hidden < 0)
        return set_status(JST_ERR_ARG, "gru backward: negative size");
    if (accumulate & ~(JST_GRU_ACC_DX | JST_GRU_ACC_PARAMS | JST_GRU_ACC_DH0))
        return set_status(JST_ERR_ARG, "gru backward: unknown accumulate flag");
    const int64_t rows = (int64_t)seq * batch, G = 3LL * hidden;
    if (rows > 0x7fffffffLL || G > 0x7fffffffLL) return set_status(JST_ERR_ARG, "gru backward: size exceeds int");
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (hidden == 0) return set_status(JST_OK, nullptr);
    if (seq == 0 || batch == 0) {  // no step: parameter gradients are zero, dh0 = dh_n
        if (!(accumulate & JST_GRU_ACC_PARAMS)) {
            const struct { float* p; size_t n; } z[] = {{dw_ih, (size_t)G * input_size}, {dw_hh, (size_t)G * hidden},
                                                        {db_ih, (size_t)G}, {db_hh, (size_t)G}};
            for (const auto& e : z)
                if (e.p && cudaMemsetAsync(e.p, 0, e.n * 4, s) != cudaSuccess) {
                    cudaGetLastError();
                    return set_status(JST_ERR_CUDA, "gru backward: zero fill");
                }
        }
        if (dh0 && batch) {
            const size_t n = (size_t)batch * hidden * 4;
            cudaError_t e = cudaSuccess;
            if (!(accumulate & JST_GRU_ACC_DH0)) e = dh_n ? cudaMemcpyAsync(dh0, dh_n, n, cudaMemcpyDeviceToDevice, s)
                                      : cudaMemsetAsync(dh0, 0, n, s);
            else if (dh_n) {
                ProfScope prof(s, KID_RNN);
                accumulate_kernel<<<148, 256, 0, s>>>(dh0, dh_n, (int64_t)batch * hidden);
                e = cudaPeekAtLastError();
            }
            if (e != cudaSuccess) {
                cudaGetLastError();
                return set_status(JST_ERR_CUDA, "gru backward: dh0");
            }
        }
        return set_status(JST_OK, nullptr);
    }
    if (ld_out < hidden || (dout && ld_dout < hidden)) return set_status(JST_ERR_ARG, "gru backward: leading dimension < hidden");
    if (!w_hh || !out || !saved) return set_status(JST_ERR_ARG, "gru backward: null w_hh, out or saved");
    if ((dx && !w_ih) || (dw_ih && !x)) return set_status(JST_ERR_ARG, "gru backward: null w_ih or x");
    return gru_backward_impl(x, seq, batch, input_size, hidden, w_ih, w_hh, h0, reverse, out, ld_out, saved, dout,
                             ld_dout, dh_n, dx, dw_ih, dw_hh, db_ih, db_hh, dh0, accumulate, s);
}
