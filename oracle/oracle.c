/*
 * oracle.c -- CPU oracle for JsTorch's fp32 GEMM path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the jstorch_b200 package,
 * its CUDA kernels or its C-ABI library) links, loads or calls this file.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
 * and only as the checker (or, for jo_sgemm_f32_cpu, as the timed CPU baseline).
 *
 * What it restates (reference paths are relative to the JsTorch project root):
 *
 *   jo_gemm_rows_f64   C = op(A)·op(B) [+ bias] [relu], fp64-accumulated, for
 *                      every layout the path uses.
 *                        NN, beta = 0 ........ native/ops/matmul.cu:28-37
 *                        batch strides ....... native/ops/matmul.cu:40-50
 *                                              (strideA = M*K, strideB = K*N,
 *                                               strideC = M*N when packed)
 *                        Y = X·W^T + bias ..... native/ops/matmul.cu:54-67
 *                                              (W stored [out_f, in_f]; bias
 *                                               added after the product,
 *                                               add_bias_kernel :18-23)
 *                        relu ................ native/ops/kernels.cuh:50
 *                                              (max(x, 0)), applied after bias
 *                                              as nn.js:105-110 + nn.js:547
 *                                              compose them.
 *                      The reference computes the product in cuBLAS with TF32
 *                      tensor-op math (matmul.cu:12); the oracle is the exact
 *                      product the fp32 interface promises, accumulated in fp64.
 *
 *   jo_max_rel_err     the tolerance metric of the path:
 *                      max_ij |C - C_ref| / (||op(A)_i,:||_2 * ||op(B)_:,j||_2 + |bias_j|)
 *
 *   jo_sgemm_f32_cpu   the reference has no CPU fallback; its row-major fp32
 *                      triple loop (i-k-j order, fp32 accumulation into the C
 *                      row, OpenMP over rows of C) is the CPU baseline.
 *
 * Parity pins: the known-answer vector of README.md:41-55 and fixtures made by
 * running the reference's own matmul.cu (compiled from its source by
 * oracle/Makefile into oracle/_ref/) on integer-valued inputs, for which TF32
 * math is exact; see tests/test_oracle.py.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* element (r, k) of op(X) where op(X) is [rows, K]; trans = stored as [K, rows] */
static inline double op_at(const float* X, int trans, long ld, long r, long k) {
    return trans ? (double)X[k * ld + r] : (double)X[r * ld + k];
}

/*
 * C_out[b][t][j] = relu?( sum_k op(A)[rows[t], k] * op(B)[k, j] + bias[j] )
 * op(A) is [M, K]; op(B) is [K, N].  transA: A stored [K, M] (lda >= M);
 * transB: B stored [N, K] (ldb >= K).  rows == NULL means all M rows
 * (nrows must then equal M).  C_out is dense [batch][nrows][N] fp64.
 * Returns 0, or -1 on a bad argument.
 */
int jo_gemm_rows_f64(int transA, int transB, int M, int N, int K,
                     const float* A, long lda, long long strideA,
                     const float* B, long ldb, long long strideB,
                     int batch, const float* bias, int relu,
                     const int* rows, int nrows, double* C_out) {
    if (M < 0 || N < 0 || K < 0 || batch < 1 || nrows < 0) return -1;
    if (!rows && nrows != M) return -1;
    for (int b = 0; b < batch; b++) {
        const float* Ab = A + (long long)b * strideA;
        const float* Bb = B + (long long)b * strideB;
        double* Cb = C_out + (long long)b * nrows * N;
#pragma omp parallel
        {
            double* arow = (double*)malloc(sizeof(double) * (size_t)(K > 0 ? K : 1));
            double* acc = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
#pragma omp for schedule(dynamic, 1)
            for (int t = 0; t < nrows; t++) {
                long i = rows ? rows[t] : t;
                for (long k = 0; k < K; k++) arow[k] = op_at(Ab, transA, lda, i, k);
                if (!transB) {
                    for (long j = 0; j < N; j++) acc[j] = 0.0;
                    for (long k = 0; k < K; k++) {
                        const double a = arow[k];
                        const float* brow = Bb + k * ldb;
                        for (long j = 0; j < N; j++) acc[j] += a * (double)brow[j];
                    }
                } else {
                    for (long j = 0; j < N; j++) {
                        const float* bcol = Bb + j * ldb;
                        double s = 0.0;
                        for (long k = 0; k < K; k++) s += arow[k] * (double)bcol[k];
                        acc[j] = s;
                    }
                }
                double* crow = Cb + (long long)t * N;
                for (long j = 0; j < N; j++) {
                    double v = acc[j] + (bias ? (double)bias[j] : 0.0);
                    if (relu && !(v > 0.0)) v = 0.0;
                    crow[j] = v;
                }
            }
            free(arow);
            free(acc);
        }
    }
    return 0;
}

/*
 * Tolerance metric over the sampled rows:
 *   err_ij = |C_test[rows[t], j] - C_ref[t, j]| / (||op(A)_i,:|| * ||op(B)_:,j|| + |bias_j|)
 * C_test is [batch] x [M, N] with leading dimension ldc and batch stride strideC;
 * C_ref is the dense output of jo_gemm_rows_f64 for the same rows.
 * A NaN/Inf in C_test, or a nonzero difference over a zero denominator, gives +inf.
 * worst (nullable, 3 ints): batch, row, column of the maximum.
 */
double jo_max_rel_err(int transA, int transB, int M, int N, int K,
                      const float* A, long lda, long long strideA,
                      const float* B, long ldb, long long strideB,
                      int batch, const float* bias,
                      const float* C_test, long ldc, long long strideC,
                      const double* C_ref, const int* rows, int nrows, int* worst) {
    (void)M;
    double maxerr = 0.0;
    int wb = -1, wi = -1, wj = -1;
    double* bn = (double*)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
    for (int b = 0; b < batch; b++) {
        const float* Ab = A + (long long)b * strideA;
        const float* Bb = B + (long long)b * strideB;
        const float* Cb = C_test + (long long)b * strideC;
        const double* Rb = C_ref + (long long)b * nrows * N;
        for (long j = 0; j < N; j++) {
            double s = 0.0;
            for (long k = 0; k < K; k++) {
                double v = transB ? (double)Bb[j * ldb + k] : (double)Bb[k * ldb + j];
                s += v * v;
            }
            bn[j] = sqrt(s);
        }
        for (int t = 0; t < nrows; t++) {
            long i = rows ? rows[t] : t;
            double s = 0.0;
            for (long k = 0; k < K; k++) {
                double v = op_at(Ab, transA, lda, i, k);
                s += v * v;
            }
            const double an = sqrt(s);
            for (long j = 0; j < N; j++) {
                const double c = (double)Cb[i * ldc + j];
                const double r = Rb[(long long)t * N + j];
                const double den = an * bn[j] + (bias ? fabs((double)bias[j]) : 0.0);
                double e;
                if (!isfinite(c)) e = INFINITY;
                else if (den == 0.0) e = (c == r) ? 0.0 : INFINITY;
                else e = fabs(c - r) / den;
                if (e > maxerr || wb < 0) {
                    if (e > maxerr) maxerr = e;
                    wb = b; wi = (int)i; wj = (int)j;
                }
            }
        }
    }
    free(bn);
    if (worst) { worst[0] = wb; worst[1] = wi; worst[2] = wj; }
    return maxerr;
}

/*
 * CPU baseline: C[r, :] = A[r, :]·B for r in [row0, row0 + nrows), row-major NN
 * fp32 with fp32 accumulation, i-k-j order (the loop order that streams rows
 * of B, as a row-major implementation does), OpenMP over rows with `threads`
 * threads (<= 0: the OpenMP default).  Returns the thread count used.
 */
int jo_sgemm_f32_cpu(int M, int N, int K, const float* A, const float* B, float* C,
                     int row0, int nrows, int threads) {
    (void)M;
    int used = 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
    {
#pragma omp single
        used = omp_get_num_threads();
    }
#else
    (void)threads;
#endif
#pragma omp parallel for schedule(static)
    for (int r = row0; r < row0 + nrows; r++) {
        float* crow = C + (long long)r * N;
        for (long j = 0; j < N; j++) crow[j] = 0.0f;
        const float* arow = A + (long long)r * K;
        for (long k = 0; k < K; k++) {
            const float a = arow[k];
            const float* brow = B + k * (long long)N;
            for (long j = 0; j < N; j++) crow[j] += a * brow[j];
        }
    }
    return used;
}

int jo_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
