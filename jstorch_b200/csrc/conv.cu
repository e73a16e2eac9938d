// conv.cu -- the eight im2col-GEMM convolution launchers of the reference
// (native/ops/conv.cu:324-627) on this library's GEMM kernels.
//
// Same extern "C" signatures and the same caller-provided col_buf of
// B * C * kH * kW * (output spatial) floats.  What changes:
//   * the per-(batch, group) cublasSgemm loops (conv.cu:345-352, 380-389,
//     421-430, 450-459) become ONE strided-batched GEMM per group (the
//     weights are a stride-0 operand), and the bias add (add_bias_*_kernel)
//     moves into the GEMM epilogue as a per-row bias, or into col2im for the
//     transposed convolutions;
//   * the backward-weight launchers (conv.cu:495-627) zero grad_weight and
//     accumulate B GEMMs with beta = 1.  Here im2col writes the columns
//     batch-inner, col[c*kk + tap][b*N + n], and the other operand is permuted
//     to the same [rows][b*N + n] order, so the sum over the batch is the K
//     loop of one NT GEMM (K = B * N), batched over the groups;
//   * a 1 x 1, stride-1, unpadded conv2d uses the input as its column matrix
//     (no im2col pass);
//   * indices are 64-bit; 1-D launchers are the 2-D ones with H = 1.
// All GEMMs run in fp32 with the library's kernel choice (3xTF32 tensor-core
// or FFMA), so the results meet the path's error bound, unlike the TF32
// math mode the reference sets (conv.cu:190-196).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/jstorch_conv.h"
#include "gemm_internal.h"

namespace jst {
namespace conv {

struct Geo {
    int B, C, H, W;      // image batch, channels, spatial size read by im2col
    int kH, kW, sH, sW, pH, pW, dH, dW;
    int Ho, Wo;          // spatial size of the column matrix
};

// col (batch-outer) [b][c*kH*kW + kh*kW + kw][ho*Wo + wo]  -- conv.cu:202-220
// col (batch-inner) [c*kH*kW + kh*kW + kw][b][ho*Wo + wo]
// One block per row of the column matrix (fixed b, c, kh, kw): the row's
// coordinates are decoded once, the threads walk its Ho*Wo entries, so the
// stores are coalesced and (stride 1) so are the loads.
template <bool INNER>
__global__ void im2col_kernel(const float* __restrict__ in, float* __restrict__ col, const Geo g) {
    const int N = g.Ho * g.Wo;
    const int kk = g.kH * g.kW;
    const int64_t row = blockIdx.x + (int64_t)blockIdx.y * gridDim.x;  // destination row
    int b, r;
    if (INNER) {
        b = (int)(row % g.B);
        r = (int)(row / g.B);
    } else {
        r = (int)(row % ((int64_t)g.C * kk));
        b = (int)(row / ((int64_t)g.C * kk));
    }
    if (b >= g.B) return;
    const int c = r / kk, tap = r % kk;
    const int oh = (tap / g.kW) * g.dH - g.pH, ow = (tap % g.kW) * g.dW - g.pW;
    const float* src = in + ((int64_t)b * g.C + c) * g.H * g.W;
    float* dst = col + row * N;
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
        const int ho = n / g.Wo, wo = n - ho * g.Wo;
        const int hi = ho * g.sH + oh, wi = wo * g.sW + ow;
        float v = 0.0f;
        if ((unsigned)hi < (unsigned)g.H && (unsigned)wi < (unsigned)g.W) v = __ldg(src + hi * g.W + wi);
        dst[n] = v;
    }
}

// output[b][c][h][w] = sum over taps of col[b][c*kk + tap][hi*Wi + wi] (+ bias[c])
// -- conv.cu:223-247, the bias (conv.cu:250-257) added after the tap sum.
// Here g.H x g.W is the output image and g.Ho x g.Wo the column spatial size.
// One block per output plane (b, c).
__global__ void col2im_kernel(const float* __restrict__ col, float* __restrict__ out, const float* __restrict__ bias,
                              const Geo g) {
    const int64_t bc = blockIdx.x + (int64_t)blockIdx.y * gridDim.x;
    if (bc >= (int64_t)g.B * g.C) return;
    const int c = (int)(bc % g.C);
    const int HW = g.H * g.W;
    const int Ni = g.Ho * g.Wo;
    const int kk = g.kH * g.kW;
    const float* cb = col + bc * kk * Ni;
    const float bv = bias ? __ldg(bias + c) : 0.0f;
    float* o = out + bc * HW;
    for (int i = threadIdx.x; i < HW; i += blockDim.x) {
        const int h = i / g.W, w = i - h * g.W;
        float sum = 0.0f;
        for (int kh = 0; kh < g.kH; ++kh) {
            const int nh = h + g.pH - kh * g.dH;
            if (nh < 0 || nh % g.sH) continue;
            const int hi = nh / g.sH;
            if (hi >= g.Ho) continue;
            for (int kw = 0; kw < g.kW; ++kw) {
                const int nw = w + g.pW - kw * g.dW;
                if (nw < 0 || nw % g.sW) continue;
                const int wi = nw / g.sW;
                if (wi >= g.Wo) continue;
                sum += __ldg(cb + (int64_t)(kh * g.kW + kw) * Ni + hi * g.Wo + wi);
            }
        }
        if (bias) sum += bv;
        o[i] = sum;
    }
}

// dst[c][b][n] = src[b][c][n], one block per (c, b) row
__global__ void permute_bcn_kernel(const float* __restrict__ src, float* __restrict__ dst, int B, int C, int N) {
    const int64_t row = blockIdx.x + (int64_t)blockIdx.y * gridDim.x;  // c * B + b
    if (row >= (int64_t)B * C) return;
    const int b = (int)(row % B), c = (int)(row / B);
    const float* s = src + ((int64_t)b * C + c) * N;
    float* d = dst + row * N;
    for (int n = threadIdx.x; n < N; n += blockDim.x) d[n] = __ldg(s + n);
}

// Grid of `rows` blocks as (x, y) with x <= 65535 * 1024.
dim3 row_grid(int64_t rows) {
    const int64_t x = std::min<int64_t>(rows, 1 << 20);
    return dim3((unsigned)x, (unsigned)((rows + x - 1) / x));
}

int im2col(const float* in, float* col, const Geo& g, bool inner, cudaStream_t s) {
    const int64_t rows = (int64_t)g.B * g.C * g.kH * g.kW;
    if (rows == 0 || (int64_t)g.Ho * g.Wo == 0) return JST_OK;
    {
        ProfScope prof(s, KID_CONV);
        if (inner) im2col_kernel<true><<<row_grid(rows), 256, 0, s>>>(in, col, g);
        else im2col_kernel<false><<<row_grid(rows), 256, 0, s>>>(in, col, g);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, "im2col launch failed");
}

int col2im(const float* col, float* out, const float* bias, const Geo& g, cudaStream_t s) {
    const int64_t planes = (int64_t)g.B * g.C;
    if (planes == 0 || (int64_t)g.H * g.W == 0) return JST_OK;
    {
        ProfScope prof(s, KID_CONV);
        col2im_kernel<<<row_grid(planes), 256, 0, s>>>(col, out, bias, g);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, "col2im launch failed");
}

int permute_bcn(const float* src, float* dst, int B, int C, int64_t N, cudaStream_t s) {
    const int64_t rows = (int64_t)B * C;
    if (rows == 0 || N == 0) return JST_OK;
    {
        ProfScope prof(s, KID_CONV);
        permute_bcn_kernel<<<row_grid(rows), 256, 0, s>>>(src, dst, B, C, (int)N);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, "permute launch failed");
}

bool fits_int(int64_t v) { return v >= 0 && v <= 0x7fffffffLL; }

int check_geo(int B, int Ci, int H, int W, int Co, int kH, int kW, int sH, int sW, int pH, int pW, int dH, int dW,
              int groups, int Ho, int Wo) {
    if (B < 0 || Ci < 0 || H < 0 || W < 0 || Co < 0 || Ho < 0 || Wo < 0)
        return set_status(JST_ERR_ARG, "conv: negative size");
    if (kH < 1 || kW < 1 || sH < 1 || sW < 1 || dH < 1 || dW < 1 || pH < 0 || pW < 0)
        return set_status(JST_ERR_ARG, "conv: kernel, stride and dilation must be >= 1, padding >= 0");
    if (groups < 1 || Ci % groups || Co % groups) return set_status(JST_ERR_ARG, "conv: groups must divide channels");
    return JST_OK;
}

// One GEMM descriptor, everything else defaulted.
jst_gemm_desc desc(int M, int N, int K, const float* A, int64_t lda, int64_t sA, int transA, const float* Bm,
                   int64_t ldb, int64_t sB, int transB, float* C, int64_t ldc, int64_t sC, int batch, cudaStream_t s) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, A, Bm, C);
    d.transA = transA;
    d.lda = lda;
    d.strideA = sA;
    d.transB = transB;
    d.ldb = ldb;
    d.strideB = sB;
    d.ldc = ldc;
    d.strideC = sC;
    d.batch = batch;
    d.stream = reinterpret_cast<jst_stream_t>(s);
    return d;
}

// Conv2d forward (conv.cu:402-434): out[b, g] = W_g . col[b, g] (+ bias), batched over b.
int conv2d(const float* input, const float* weight, const float* bias, float* output, float* col_buf, int B, int Ci,
           int H, int W, int Co, int kH, int kW, int sH, int sW, int pH, int pW, int dH, int dW, int groups, int Ho,
           int Wo, cudaStream_t s) {
    int rc = check_geo(B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, groups, Ho, Wo);
    if (rc) return rc;
    const int Ci_g = Ci / groups, Co_g = Co / groups;
    const int64_t N = (int64_t)Ho * Wo, kk = (int64_t)kH * kW, Kg = Ci_g * kk;
    if (!fits_int(N) || !fits_int(Kg)) return set_status(JST_ERR_ARG, "conv: GEMM dimension exceeds int");
    const bool direct = kH == 1 && kW == 1 && sH == 1 && sW == 1 && pH == 0 && pW == 0 && Ho == H && Wo == W;
    const float* col = input;
    if (!direct) {
        if (!col_buf) return set_status(JST_ERR_ARG, "conv: null col_buf");
        rc = im2col(input, col_buf, Geo{B, Ci, H, W, kH, kW, sH, sW, pH, pW, dH, dW, Ho, Wo}, false, s);
        if (rc) return rc;
        col = col_buf;
    }
    for (int g = 0; g < groups; ++g) {
        jst_gemm_desc d = desc(Co_g, (int)N, (int)Kg, weight + (int64_t)g * Co_g * Kg, Kg, 0, 0,
                               col + (int64_t)g * Kg * N, N, (int64_t)Ci * kk * N, 0, output + (int64_t)g * Co_g * N, N,
                               (int64_t)Co * N, B, s);
        if (bias) {
            d.bias = bias + (int64_t)g * Co_g;
            d.epilogue = JST_EPI_BIAS_ROW;
        }
        if (B > 0 && (rc = jst_gemm_ex(&d))) return rc;
    }
    return set_status(JST_OK, nullptr);
}

// ConvTranspose2d forward (conv.cu:436-466): col[b, g] = W_g^T . x[b, g], then col2im (+ bias).
int conv_transpose2d(const float* input, const float* weight, const float* bias, float* output, float* col_buf, int B,
                     int Ci, int Hi, int Wi, int Co, int kH, int kW, int sH, int sW, int pH, int pW, int dH, int dW,
                     int groups, int Ho, int Wo, cudaStream_t s) {
    int rc = check_geo(B, Ci, Hi, Wi, Co, kH, kW, sH, sW, pH, pW, dH, dW, groups, Ho, Wo);
    if (rc) return rc;
    if (!col_buf) return set_status(JST_ERR_ARG, "conv: null col_buf");
    const int Ci_g = Ci / groups, Co_g = Co / groups;
    const int64_t Nin = (int64_t)Hi * Wi, kk = (int64_t)kH * kW, Mg = Co_g * kk;
    if (!fits_int(Nin) || !fits_int(Mg)) return set_status(JST_ERR_ARG, "conv: GEMM dimension exceeds int");
    for (int g = 0; g < groups && B > 0; ++g) {
        // weight group g is stored [Ci_g, Co_g*kk]: op(A) = its transpose (TN)
        jst_gemm_desc d = desc((int)Mg, (int)Nin, Ci_g, weight + (int64_t)g * Ci_g * Mg, Mg, 0, 1,
                               input + (int64_t)g * Ci_g * Nin, Nin, (int64_t)Ci * Nin, 0,
                               col_buf + (int64_t)g * Mg * Nin, Nin, (int64_t)Co * kk * Nin, B, s);
        if ((rc = jst_gemm_ex(&d))) return rc;
    }
    // output image Ho x Wo, columns over the input grid Hi x Wi
    rc = col2im(col_buf, output, bias, Geo{B, Co, Ho, Wo, kH, kW, sH, sW, pH, pW, dH, dW, Hi, Wi}, s);
    return rc ? rc : set_status(JST_OK, nullptr);
}

// grad_weight[g] = P[g] . Q[g]^T over K = B*N, where P = rows_src permuted to
// [rows][B*N] and Q = im2col(col_src) batch-inner (conv.cu:495-627).
//   P: [Prows][B*N]  (group g: rows g*Pg ..)
//   Q: [Qrows][B*N]  (group g: rows g*Qg ..)
//   grad_weight group g: [Pg, Qg] at g*Pg*Qg
int backward_weight(const float* rows_src, int Prows, const float* col_src, const Geo& cg, float* grad_weight,
                    float* col_buf, int groups, cudaStream_t s) {
    const int B = cg.B;
    const int64_t N = (int64_t)cg.Ho * cg.Wo, kk = (int64_t)cg.kH * cg.kW;
    const int64_t BN = (int64_t)B * N;
    const int Pg = Prows / groups;
    const int64_t Qg = (int64_t)(cg.C / groups) * kk;
    if (!fits_int(BN) || !fits_int(Qg)) return set_status(JST_ERR_ARG, "conv: GEMM dimension exceeds int");
    if (!col_buf) return set_status(JST_ERR_ARG, "conv: null col_buf");
    int rc = im2col(col_src, col_buf, cg, true, s);
    if (rc) return rc;
    const float* P = rows_src;
    void* ws = nullptr;
    if (B > 1) {
        rc = workspace_alloc((size_t)Prows * BN * sizeof(float), s, &ws);
        if (rc) return rc;
        rc = permute_bcn(rows_src, static_cast<float*>(ws), B, Prows, N, s);
        P = static_cast<const float*>(ws);
    }
    if (!rc) {
        jst_gemm_desc d = desc(Pg, (int)Qg, (int)BN, P, BN, (int64_t)Pg * BN, 0, col_buf, BN, Qg * BN, 1,
                               grad_weight, Qg, (int64_t)Pg * Qg, groups, s);
        rc = jst_gemm_ex(&d);
    }
    if (ws) {
        const int frc = workspace_free(ws, s);
        if (!rc) rc = frc;
    }
    return rc ? rc : set_status(JST_OK, nullptr);
}

}  // namespace conv
}  // namespace jst

using jst::conv::Geo;

extern "C" {

// conv.cu:324-361 -- Conv1d = Conv2d over a 1 x L_in image with a 1 x K kernel
void launch_conv1d(const float* input, const float* weight, const float* bias, float* output, float* col_buf, int B,
                   int C_in, int L_in, int C_out, int K, int stride, int padding, int dilation, int groups, int L_out,
                   jst_stream_t s) {
    jst::conv::conv2d(input, weight, bias, output, col_buf, B, C_in, 1, L_in, C_out, 1, K, 1, stride, 0, padding, 1,
                      dilation, groups, 1, L_out, reinterpret_cast<cudaStream_t>(s));
}

// conv.cu:363-400
void launch_conv_transpose1d(const float* input, const float* weight, const float* bias, float* output,
                             float* col_buf, int B, int C_in, int L_in, int C_out, int K, int stride, int padding,
                             int dilation, int groups, int L_out, jst_stream_t s) {
    jst::conv::conv_transpose2d(input, weight, bias, output, col_buf, B, C_in, 1, L_in, C_out, 1, K, 1, stride, 0,
                                padding, 1, dilation, groups, 1, L_out, reinterpret_cast<cudaStream_t>(s));
}

// conv.cu:402-434
void launch_conv2d(const float* input, const float* weight, const float* bias, float* output, float* col_buf, int B,
                   int Ci, int H, int W, int Co, int kH, int kW, int sH, int sW, int pH, int pW, int dH, int dW,
                   int groups, int Ho, int Wo, jst_stream_t s) {
    jst::conv::conv2d(input, weight, bias, output, col_buf, B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, groups,
                      Ho, Wo, reinterpret_cast<cudaStream_t>(s));
}

// conv.cu:436-466
void launch_conv_transpose2d(const float* input, const float* weight, const float* bias, float* output,
                             float* col_buf, int B, int Ci, int Hi, int Wi, int Co, int kH, int kW, int sH, int sW,
                             int pH, int pW, int dH, int dW, int groups, int Ho, int Wo, jst_stream_t s) {
    jst::conv::conv_transpose2d(input, weight, bias, output, col_buf, B, Ci, Hi, Wi, Co, kH, kW, sH, sW, pH, pW, dH,
                                dW, groups, Ho, Wo, reinterpret_cast<cudaStream_t>(s));
}

// conv.cu:495-528 -- grad_weight [C_out, C_in/g, K] = sum_b go[b] . im2col(x[b])^T
void launch_conv1d_backward_weight(const float* input, const float* grad_output, float* grad_weight, float* col_buf,
                                   int B, int C_in, int L_in, int C_out, int K, int stride, int padding, int dilation,
                                   int groups, int L_out, jst_stream_t s) {
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (jst::conv::check_geo(B, C_in, 1, L_in, C_out, 1, K, 1, stride, 0, padding, 1, dilation, groups, 1, L_out))
        return;
    jst::conv::backward_weight(grad_output, C_out, input, Geo{B, C_in, 1, L_in, 1, K, 1, stride, 0, padding, 1,
                                                              dilation, 1, L_out},
                               grad_weight, col_buf, groups, st);
}

// conv.cu:530-563
void launch_conv2d_backward_weight(const float* input, const float* grad_output, float* grad_weight, float* col_buf,
                                   int B, int Ci, int H, int W, int Co, int kH, int kW, int sH, int sW, int pH, int pW,
                                   int dH, int dW, int groups, int Ho, int Wo, jst_stream_t s) {
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (jst::conv::check_geo(B, Ci, H, W, Co, kH, kW, sH, sW, pH, pW, dH, dW, groups, Ho, Wo)) return;
    jst::conv::backward_weight(grad_output, Co, input, Geo{B, Ci, H, W, kH, kW, sH, sW, pH, pW, dH, dW, Ho, Wo},
                               grad_weight, col_buf, groups, st);
}

// conv.cu:565-598 -- grad_weight [C_in, C_out/g, K] = sum_b x[b] . im2col(go[b])^T
void launch_conv_transpose1d_backward_weight(const float* input, const float* grad_output, float* grad_weight,
                                             float* col_buf, int B, int C_in, int L_in, int C_out, int K, int stride,
                                             int padding, int dilation, int groups, int L_out, jst_stream_t s) {
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (jst::conv::check_geo(B, C_in, 1, L_in, C_out, 1, K, 1, stride, 0, padding, 1, dilation, groups, 1, L_out))
        return;
    jst::conv::backward_weight(input, C_in, grad_output, Geo{B, C_out, 1, L_out, 1, K, 1, stride, 0, padding, 1,
                                                             dilation, 1, L_in},
                               grad_weight, col_buf, groups, st);
}

// conv.cu:600-627
void launch_conv_transpose2d_backward_weight(const float* input, const float* grad_output, float* grad_weight,
                                             float* col_buf, int B, int Ci, int Hi, int Wi, int Co, int kH, int kW,
                                             int sH, int sW, int pH, int pW, int dH, int dW, int groups, int Ho,
                                             int Wo, jst_stream_t s) {
    const cudaStream_t st = reinterpret_cast<cudaStream_t>(s);
    if (jst::conv::check_geo(B, Ci, Hi, Wi, Co, kH, kW, sH, sW, pH, pW, dH, dW, groups, Ho, Wo)) return;
    jst::conv::backward_weight(input, Ci, grad_output, Geo{B, Co, Ho, Wo, kH, kW, sH, sW, pH, pW, dH, dW, Hi, Wi},
                               grad_weight, col_buf, groups, st);
}

}  // extern "C"
