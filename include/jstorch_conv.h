/*
 * jstorch_conv.h -- the im2col-GEMM convolution launchers of JsTorch,
 * exported by jstorch_b200/libjstorch_gemm.so with the reference signatures
 * (paths relative to the JsTorch project root; all in native/ops/conv.cu):
 *
 *   launch_conv1d                            conv.cu:324
 *   launch_conv_transpose1d                  conv.cu:363
 *   launch_conv2d                            conv.cu:402
 *   launch_conv_transpose2d                  conv.cu:436
 *   launch_conv1d_backward_weight            conv.cu:495
 *   launch_conv2d_backward_weight            conv.cu:530
 *   launch_conv_transpose1d_backward_weight  conv.cu:565
 *   launch_conv_transpose2d_backward_weight  conv.cu:600
 *
 * Layouts as the reference: input [B, C, H, W] (1-D: [B, C, L]), conv weight
 * [C_out, C_in/groups, kH, kW], transposed-conv weight [C_in, C_out/groups,
 * kH, kW], bias [C_out] or NULL.  col_buf is caller-provided device scratch of
 * B * C * kH * kW * (spatial size of the columns) floats, exactly what the
 * reference asks for; a 1 x 1, stride-1, unpadded conv2d does not touch it.
 * The backward-weight launchers overwrite grad_weight (the reference zeroes it
 * and accumulates, with the same result).  All pointers are device pointers;
 * calls are asynchronous on `s` and return void like the reference; their
 * status is readable through jst_get_last_status() (jstorch_gemm.h).
 * Arithmetic is fp32 through the library's GEMM kernels, within the path's
 * 2e-6 bound (the reference runs TF32 math, conv.cu:190-196).
 */
#ifndef JSTORCH_CONV_H
#define JSTORCH_CONV_H

#include "jstorch_gemm.h"

#ifdef __cplusplus
extern "C" {
#endif

void launch_conv1d(const float* input, const float* weight, const float* bias, float* output, float* col_buf,
                   int B, int C_in, int L_in, int C_out, int K, int stride, int padding, int dilation, int groups,
                   int L_out, jst_stream_t s);
void launch_conv_transpose1d(const float* input, const float* weight, const float* bias, float* output,
                             float* col_buf, int B, int C_in, int L_in, int C_out, int K, int stride, int padding,
                             int dilation, int groups, int L_out, jst_stream_t s);
void launch_conv2d(const float* input, const float* weight, const float* bias, float* output, float* col_buf,
                   int B, int Ci, int H, int W, int Co, int kH, int kW, int sH, int sW, int pH, int pW, int dH,
                   int dW, int groups, int Ho, int Wo, jst_stream_t s);
void launch_conv_transpose2d(const float* input, const float* weight, const float* bias, float* output,
                             float* col_buf, int B, int Ci, int Hi, int Wi, int Co, int kH, int kW, int sH, int sW,
                             int pH, int pW, int dH, int dW, int groups, int Ho, int Wo, jst_stream_t s);
void launch_conv1d_backward_weight(const float* input, const float* grad_output, float* grad_weight,
                                   float* col_buf, int B, int C_in, int L_in, int C_out, int K, int stride,
                                   int padding, int dilation, int groups, int L_out, jst_stream_t s);
void launch_conv2d_backward_weight(const float* input, const float* grad_output, float* grad_weight,
                                   float* col_buf, int B, int Ci, int H, int W, int Co, int kH, int kW, int sH,
                                   int sW, int pH, int pW, int dH, int dW, int groups, int Ho, int Wo,
                                   jst_stream_t s);
void launch_conv_transpose1d_backward_weight(const float* input, const float* grad_output, float* grad_weight,
                                             float* col_buf, int B, int C_in, int L_in, int C_out, int K,
                                             int stride, int padding, int dilation, int groups, int L_out,
                                             jst_stream_t s);
void launch_conv_transpose2d_backward_weight(const float* input, const float* grad_output, float* grad_weight,
                                             float* col_buf, int B, int Ci, int Hi, int Wi, int Co, int kH, int kW,
                                             int sH, int sW, int pH, int pW, int dH, int dW, int groups, int Ho,
                                             int Wo, jst_stream_t s);

#ifdef __cplusplus
}
#endif
#endif /* JSTORCH_CONV_H */
