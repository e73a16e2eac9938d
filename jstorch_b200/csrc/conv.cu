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
//   * when the GEMM runs on the tensor-core kernel, im2col is fused into its
//     split pass: the hi / lo tf32 planes the kernel streams are written
//     straight from the image, and the column matrix never exists in memory
//     (col_buf is left untouched);
//   * indices are 64-bit; 1-D launchers are the 2-D ones with H = 1.
// All GEMMs run in fp32 with the library's kernel choice (3xTF32 tensor-core
// or FFMA), so the results meet the path's error bound, unlike the TF32
// math mode the reference sets (conv.cu:190-196).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/jstorch_conv.h"
#include "gemm_internal.h"
#include "ptx.cuh"

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

// The same sum with the taps tabulated once per block.  A tap (kh, kw) that
// lands on output (h, w) reads col at (kh*kW + kw)*Ni + hi*Wo + wi, which
// splits into a row part kh*kW*Ni + hi*Wo (valid kh, hi depend on h only) and
// a column part kw*Ni + wi (kw, wi depend on w only).  The block builds, in
// shared memory, the valid row parts of every output row and the valid column
// parts of every output column (the only divides), then each output element
// adds col[row part + column part] over its pairs in the order of
// col2im_kernel (kh outer, kw inner), so the results are identical.
// Shared memory: H*(1+kH) + W*(1+kW) ints; the host checks the size and that
// the offsets fit an int.
__global__ void col2im_tab_kernel(const float* __restrict__ col, float* __restrict__ out,
                                  const float* __restrict__ bias, const Geo g) {
    extern __shared__ int tab[];
    int* rcnt = tab;                 // [H]
    int* roff = rcnt + g.H;          // [H][kH]
    int* ccnt = roff + g.H * g.kH;   // [W]
    int* coff = ccnt + g.W;          // [W][kW]
    const int Ni = g.Ho * g.Wo;
    for (int h = threadIdx.x; h < g.H; h += blockDim.x) {
        int n = 0;
        for (int kh = 0; kh < g.kH; ++kh) {
            const int nh = h + g.pH - kh * g.dH;
            if (nh < 0 || nh % g.sH) continue;
            const int hi = nh / g.sH;
            if (hi >= g.Ho) continue;
            roff[h * g.kH + n++] = kh * g.kW * Ni + hi * g.Wo;
        }
        rcnt[h] = n;
    }
    for (int w = threadIdx.x; w < g.W; w += blockDim.x) {
        int n = 0;
        for (int kw = 0; kw < g.kW; ++kw) {
            const int nw = w + g.pW - kw * g.dW;
            if (nw < 0 || nw % g.sW) continue;
            const int wi = nw / g.sW;
            if (wi >= g.Wo) continue;
            coff[w * g.kW + n++] = kw * Ni + wi;
        }
        ccnt[w] = n;
    }
    __syncthreads();
    const int64_t nplanes = (int64_t)g.B * g.C;
    const int HW = g.H * g.W;
    const int kk = g.kH * g.kW;
    const int dh = blockDim.x / g.W, dw = blockDim.x % g.W;
    for (int64_t bc = blockIdx.x + (int64_t)blockIdx.y * gridDim.x; bc < nplanes;
         bc += (int64_t)gridDim.x * gridDim.y) {
        const int c = (int)(bc % g.C);
        const float* cb = col + bc * kk * Ni;
        const float bv = bias ? __ldg(bias + c) : 0.0f;
        float* o = out + bc * HW;
        int h = threadIdx.x / g.W, w = threadIdx.x % g.W;
        for (int i = threadIdx.x; i < HW; i += blockDim.x) {
            float sum = 0.0f;
            const int nr = rcnt[h], nc = ccnt[w];
            for (int a = 0; a < nr; ++a) {
                const float* rp = cb + roff[h * g.kH + a];
                for (int q = 0; q < nc; ++q) sum += __ldg(rp + coff[w * g.kW + q]);
            }
            if (bias) sum += bv;
            o[i] = sum;
            h += dh;
            w += dw;
            if (w >= g.W) {
                w -= g.W;
                ++h;
            }
        }
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

// ---- im2col fused with the 3xTF32 split (hi = rn_tf32(v), lo = rn_tf32(v - hi))

// Forward operand: planes [b][n][Kp] of the column matrix of one group,
// element (k = c*kk + tap, n) read from image channel c0 + c.  A block covers
// 32 pixels x 128 k values (KT_PER_BLOCK x 32): its image reads go along n
// (one pixel per lane) into a [pixel][k] shared-memory tile with a row pitch
// of 129 floats, and its plane writes go along k as float4 stores.  A warp's
// store covers 4 pixels x 32 k (four 128-byte runs), which makes the tile
// reads conflict-free: bank (n + k) mod 32 = p + 4 c8 + const over lane
// (p, c8).  The block's k values are decoded once into a 16-byte record each
// (image offset of the channel and tap, tap row and column offsets), so the
// element loop has no division; a padding column k >= Kg and a pixel n >= N
// carry a large negative row offset, so the one unsigned row check rejects
// them.  Image offsets are 32-bit (the host routes larger images elsewhere).
constexpr int KT_PER_BLOCK = 4;
constexpr int IM2COL_BK = 32 * KT_PER_BLOCK;
constexpr int OFF_ROW = -(1 << 29);  // row offset that fails every row check
struct __align__(16) KTap {
    int off;     // c * H * W + dh * W + dw
    int dh, dw;  // kh * dH - pH, kw * dW - pW
    int pad_;
};
__global__ void __launch_bounds__(256) im2col_split_t_kernel(const float* __restrict__ x, const Geo g, int c0, int Kg,
                                                             int Kp, float* __restrict__ hi, float* __restrict__ lo) {
    __shared__ float tile[32][IM2COL_BK + 1];  // [pixel][k]
    __shared__ KTap taps[IM2COL_BK];
    const int b = blockIdx.z;
    const int n0 = blockIdx.x * 32, kb0 = blockIdx.y * IM2COL_BK;
    const int N = g.Ho * g.Wo, kk = g.kH * g.kW, HW = g.H * g.W;
    const int tid = threadIdx.y * 32 + threadIdx.x;
    if (tid < IM2COL_BK) {
        const int k = kb0 + tid;
        const int c = k / kk, tap = k - c * kk;
        const int kh = tap / g.kW, kw = tap - kh * g.kW;
        const int dh = kh * g.dH - g.pH, dw = kw * g.dW - g.pW;
        taps[tid] = k < Kg ? KTap{(int)((unsigned)c * HW + (unsigned)(dh * g.W + dw)), dh, dw, 0}
                           : KTap{0, OFF_ROW, 0, 0};
    }
    const float* xb = x + ((int64_t)b * g.C + c0) * HW;
    const int n = n0 + threadIdx.x;
    const int nc = n < N ? n : 0;
    const int ho = nc / g.Wo, wo = nc - ho * g.Wo;
    const int hs = n < N ? ho * g.sH : OFF_ROW, ws = wo * g.sW;
    const unsigned p0 = (unsigned)(ho * g.sH) * g.W + ws;
    __syncthreads();
    // every image load of the block's 32 x 128 elements is issued before the
    // tile barrier: 16 loads in flight per thread
    float v[IM2COL_BK / 8];
#pragma unroll
    for (int i = 0; i < IM2COL_BK / 8; ++i) {
        const KTap t = taps[threadIdx.y + 8 * i];
        const bool ok = (unsigned)(hs + t.dh) < (unsigned)g.H && (unsigned)(ws + t.dw) < (unsigned)g.W;
        v[i] = ok ? __ldg(xb + (p0 + (unsigned)t.off)) : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < IM2COL_BK / 8; ++i) tile[threadIdx.x][threadIdx.y + 8 * i] = v[i];
    __syncthreads();
    // store phase: warp w writes pixels 4w .. 4w+3, lane (p, c8) = pixel 4w + p,
    // k = 32 q + 4 c8 .. +3 in pass q
    const int nl = threadIdx.y * 4 + (threadIdx.x >> 3), c8 = threadIdx.x & 7;
    const int nn = n0 + nl;
    if (nn >= N) return;
    float* hrow = hi + ((int64_t)b * N + nn) * Kp;
    float* lrow = lo + ((int64_t)b * N + nn) * Kp;
#pragma unroll
    for (int q = 0; q < KT_PER_BLOCK; ++q) {
        const int kl = 32 * q + 4 * c8;
        const int k = kb0 + kl;
        if (k >= Kp) break;
        float h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float val = tile[nl][kl + j];
            h[j] = ptx::to_tf32(val);
            l[j] = ptx::to_tf32(val - h[j]);
        }
        // Kp % 4 == 0, k % 4 == 0: 16-byte aligned
        *reinterpret_cast<float4*>(hrow + k) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(lrow + k) = make_float4(l[0], l[1], l[2], l[3]);
    }
}

// Weight-gradient operand: planes [r][Kp] with r = c*kk + tap (image channel
// c0 + c) and K index k = b*N + n over batch x column pixels -- the batch-inner
// column matrix, split as it is formed.  With a 1 x 1 geometry this is the
// [B][C][N] -> [C][B*N] permute of the other operand.  One block row per r,
// four consecutive k per thread (float4 stores).
__global__ void __launch_bounds__(256) im2col_split_rows_kernel(const float* __restrict__ x, const Geo g, int c0,
                                                                int rows, int64_t BN, int64_t Kp,
                                                                float* __restrict__ hi, float* __restrict__ lo) {
    const int r = blockIdx.y;
    if (r >= rows) return;
    const int N = g.Ho * g.Wo, kk = g.kH * g.kW, HW = g.H * g.W;
    const int c = r / kk, tap = r - c * kk;
    const int oh = (tap / g.kW) * g.dH - g.pH, ow = (tap % g.kW) * g.dW - g.pW;
    const float* xc = x + (int64_t)(c0 + c) * HW;
    const int64_t img = (int64_t)g.C * HW;
    float* ho_ = hi + (int64_t)r * Kp;
    float* lo_ = lo + (int64_t)r * Kp;
    int64_t k4 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
    if (k4 >= Kp) return;
    // (b, h, w) of the thread's first k, then advanced by the loop stride as
    // mixed-radix digits (stride = sb images + sh rows + sw columns, with
    // sh < Ho and sw < Wo, so each digit carries at most once)
    const int64_t step = (int64_t)gridDim.x * blockDim.x * 4;
    int b = (int)(k4 / N);
    int h = (int)(k4 - (int64_t)b * N);
    int w = h % g.Wo;
    h /= g.Wo;
    const int sb = (int)(step / N), srem = (int)(step - (int64_t)sb * N);
    const int sh = srem / g.Wo, sw = srem - sh * g.Wo;
    for (; k4 < Kp; k4 += step) {
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (w + 3 < g.Wo && k4 + 4 <= BN) {
            // the four k lie on one output row: one row check, one base address
            const int ih = h * g.sH + oh;
            if ((unsigned)ih < (unsigned)g.H) {
                const float* xr = xc + b * img + ih * g.W;
                const int iw0 = w * g.sW + ow;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int iw = iw0 + j * g.sW;
                    if ((unsigned)iw < (unsigned)g.W) v[j] = __ldg(xr + iw);
                }
            }
        } else {
            int bb = b, hh = h, ww = w;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int ih = hh * g.sH + oh, iw = ww * g.sW + ow;
                if (k4 + j < BN && (unsigned)ih < (unsigned)g.H && (unsigned)iw < (unsigned)g.W)
                    v[j] = __ldg(xc + bb * img + ih * g.W + iw);
                if (++ww == g.Wo) {
                    ww = 0;
                    if (++hh == g.Ho) {
                        hh = 0;
                        ++bb;
                    }
                }
            }
        }
        float hv[4], lv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            hv[j] = ptx::to_tf32(v[j]);
            lv[j] = ptx::to_tf32(v[j] - hv[j]);
        }
        *reinterpret_cast<float4*>(ho_ + k4) = make_float4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<float4*>(lo_ + k4) = make_float4(lv[0], lv[1], lv[2], lv[3]);
        w += sw;
        if (w >= g.Wo) {
            w -= g.Wo;
            ++h;
        }
        h += sh;
        if (h >= g.Ho) {
            h -= g.Ho;
            ++b;
        }
        b += sb;
    }
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
    const size_t tab_bytes = ((size_t)g.H * (1 + g.kH) + (size_t)g.W * (1 + g.kW)) * sizeof(int);
    const int64_t span = (int64_t)g.kH * g.kW * g.Ho * g.Wo;  // largest table offset
    if (tab_bytes <= 32 * 1024 && span < 0x7fffffffLL) {
        // one block per output plane up to 16 waves of 8 resident blocks,
        // each block then walks planes (the tables are built once per block)
        const int64_t blocks = std::min<int64_t>(planes, 148LL * 8 * 16);
        ProfScope prof(s, KID_CONV);
        col2im_tab_kernel<<<row_grid(blocks), 256, tab_bytes, s>>>(col, out, bias, g);
    } else {
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

// Whether the library's automatic choice puts this GEMM on the tensor-core kernel.
bool on_tensor_cores(int M, int N, int K, int batch) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, reinterpret_cast<const float*>(16), reinterpret_cast<const float*>(16),
                       reinterpret_cast<float*>(16));
    d.batch = batch;
    d.strideA = (int64_t)M * K;
    d.strideB = (int64_t)K * N;
    d.strideC = (int64_t)M * N;
    return jst_gemm_select_kernel(&d) == JST_KERNEL_TC3XTF32;
}

GemmArgs shape_args(int M, int N, int K, int batch) {
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.batch = batch;
    return a;
}

int launch_im2col_split_rows(const float* x, const Geo& g, int c0, int rows, int64_t BN, int64_t Kp, float* hi,
                             float* lo, cudaStream_t s) {
    if (rows == 0 || Kp == 0) return JST_OK;
    if (rows > 65535) return set_status(JST_ERR_UNSUPPORTED, "conv: more than 65535 column rows per group");
    const int64_t want = (Kp / 4 + 255) / 256;
    const int bx = (int)std::min<int64_t>(want, std::max<int64_t>(1, 148LL * 8 / rows + 1));
    {
        ProfScope prof(s, KID_CONV);
        im2col_split_rows_kernel<<<dim3(bx, rows), 256, 0, s>>>(x, g, c0, rows, BN, Kp, hi, lo);
    }
    return cudaPeekAtLastError() == cudaSuccess ? JST_OK : set_status(JST_ERR_CUDA, "im2col split launch failed");
}

// Forward on the tensor-core kernel with im2col fused into the split of the
// column operand; the weights are split once per group and broadcast over b.
int conv2d_tc(const float* input, const float* weight, const float* bias, float* output, const Geo& g, int Co,
              int groups, cudaStream_t s) {
    const int Ci_g = g.C / groups, Co_g = Co / groups;
    const int N = g.Ho * g.Wo, Kg = Ci_g * g.kH * g.kW, Kp = (Kg + 3) & ~3;
    const size_t a_plane = (size_t)Co_g * Kp, b_plane = (size_t)g.B * N * Kp;
    void* ws = nullptr;
    int rc = workspace_alloc(2 * (a_plane + b_plane) * sizeof(float), s, &ws);
    if (rc) return rc;
    float* a_hi = static_cast<float*>(ws);
    float* a_lo = a_hi + a_plane;
    float* b_hi = a_lo + a_plane;
    float* b_lo = b_hi + b_plane;
    for (int grp = 0; grp < groups && !rc; ++grp) {
        rc = tc_split(weight + (int64_t)grp * Co_g * Kg, 1, Kg, 0, Co_g, Kg, 1, a_hi, a_lo, s);
        if (rc) break;
        {
            ProfScope prof(s, KID_CONV);
            im2col_split_t_kernel<<<dim3((N + 31) / 32, (Kp + IM2COL_BK - 1) / IM2COL_BK, g.B),
                                    dim3(32, 8), 0, s>>>(input, g, grp * Ci_g, Kg, Kp, b_hi, b_lo);
        }
        if (cudaPeekAtLastError() != cudaSuccess) {
            rc = set_status(JST_ERR_CUDA, "im2col split launch failed");
            break;
        }
        rc = tc_gemm_planes(a_hi, a_lo, b_hi, b_lo, Co_g, N, Kg, g.B, output + (int64_t)grp * Co_g * N, N,
                            (int64_t)Co * N, bias ? bias + (int64_t)grp * Co_g : nullptr, 0, device_error_word(), s,
                            0, nullptr, 0, 0, /*bias_row=*/bias ? 1 : 0, /*a_bcast=*/1, /*b_bcast=*/0, /*kslices=*/1);
    }
    const int frc = workspace_free(ws, s);
    return rc ? rc : frc;
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
    // the fused im2col split addresses one group's image with 32-bit offsets
    if (!direct && B > 0 && B <= 65535 && Co_g > 0 && Kg > 0 && fits_int((int64_t)Ci_g * H * W) &&
        on_tensor_cores(Co_g, (int)N, (int)Kg, B) &&
        tc_split_k(shape_args(Co_g, (int)N, (int)Kg, B)) == 1) {
        rc = conv2d_tc(input, weight, bias, output, Geo{B, Ci, H, W, kH, kW, sH, sW, pH, pW, dH, dW, Ho, Wo}, Co,
                       groups, s);
        return rc ? rc : set_status(JST_OK, nullptr);
    }
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

// Weight gradient on the tensor-core kernel: both operands are K-major rows
// over K = B*N and are split as they are gathered (the permute of rows_src and
// the batch-inner im2col of col_src), so neither the permuted copy nor the
// column matrix is written.  K is usually long and the output small, so the
// product is split over K when the tiles cannot fill the SMs.
int backward_weight_tc(const float* rows_src, int Prows, const float* col_src, const Geo& cg, float* grad_weight,
                       int groups, cudaStream_t s) {
    const int B = cg.B, N = cg.Ho * cg.Wo;
    const int64_t BN = (int64_t)B * N, Kp = (BN + 3) & ~int64_t(3);
    const int Pg = Prows / groups, Cg = cg.C / groups, Qg = Cg * cg.kH * cg.kW;
    const int S = tc_split_k(shape_args(Pg, Qg, (int)BN, 1));
    const size_t p_plane = (size_t)Pg * Kp, q_plane = (size_t)Qg * Kp, part = S > 1 ? (size_t)S * Pg * Qg : 0;
    void* ws = nullptr;
    int rc = workspace_alloc((2 * (p_plane + q_plane) + part) * sizeof(float), s, &ws);
    if (rc) return rc;
    float* p_hi = static_cast<float*>(ws);
    float* p_lo = p_hi + p_plane;
    float* q_hi = p_lo + p_plane;
    float* q_lo = q_hi + q_plane;
    float* pt = q_lo + q_plane;
    // rows_src [B][Prows][N] as a 1 x 1 "image" of N pixels: its im2col rows are the permute
    const Geo pg{B, Prows, 1, N, 1, 1, 1, 1, 0, 0, 1, 1, 1, N};
    for (int grp = 0; grp < groups && !rc; ++grp) {
        rc = launch_im2col_split_rows(rows_src, pg, grp * Pg, Pg, BN, Kp, p_hi, p_lo, s);
        if (!rc) rc = launch_im2col_split_rows(col_src, cg, grp * Cg, Qg, BN, Kp, q_hi, q_lo, s);
        if (rc) break;
        float* gw = grad_weight + (int64_t)grp * Pg * Qg;
        if (S <= 1) {
            rc = tc_gemm_planes(p_hi, p_lo, q_hi, q_lo, Pg, Qg, (int)BN, 1, gw, Qg, (int64_t)Pg * Qg, nullptr, 0,
                                device_error_word(), s);
        } else {
            rc = tc_gemm_planes(p_hi, p_lo, q_hi, q_lo, Pg, Qg, (int)BN, 1, pt, Qg, (int64_t)Pg * Qg, nullptr, 0,
                                device_error_word(), s, 0, nullptr, 0, 0, 0, 0, 0, S);
            if (!rc) {
                SplitKReduce r{};
                r.part = pt;
                r.slices = S;
                r.batch = 1;
                r.M = Pg;
                r.N = Qg;
                r.C = gw;
                r.ldc = Qg;
                r.strideC = (int64_t)Pg * Qg;
                r.vecC = (reinterpret_cast<uintptr_t>(gw) & 15) == 0 && (Qg % 4) == 0;
                rc = splitk_reduce_run(r, s);
            }
        }
    }
    const int frc = workspace_free(ws, s);
    return rc ? rc : frc;
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
    if (Pg > 0 && Qg > 0 && BN > 0 && Pg <= 65535 && Qg <= 65535 && on_tensor_cores(Pg, (int)Qg, (int)BN, groups)) {
        const int rc = backward_weight_tc(rows_src, Prows, col_src, cg, grad_weight, groups, s);
        return rc ? rc : set_status(JST_OK, nullptr);
    }
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
