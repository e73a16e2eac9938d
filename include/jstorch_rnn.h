/*
 * jstorch_rnn.h -- the GRU of JsTorch (src/nn.js:451-536, class GRU) on the
 * fp32 GEMM path, exported by jstorch_b200/libjstorch_gemm.so.  The reference
 * runs the GRU in JS, one time step at a time (_cell, nn.js:477-485: two
 * Tensor.matmul calls + elementwise ops); there is no native counterpart, so
 * this is new surface a JS shim would call from GRU._run_direction
 * (nn.js:487-511).
 */
#ifndef JSTORCH_RNN_H
#define JSTORCH_RNN_H

#include "jstorch_gemm.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * One layer and direction over a sequence, PyTorch gate order (r, z, n):
 *   x     [seq][batch][input_size] row-major (a layer's input, contiguous)
 *   w_ih  [3*hidden][input_size], w_hh [3*hidden][hidden], b_ih / b_hh [3*hidden] or NULL
 *   h0    [batch][hidden] or NULL (zeros, as nn.js:494)
 *   out   [seq][batch][ld_out]: step t's state is written to row block t even
 *         when reverse != 0 (nn.js:504, outputs.unshift), so a bidirectional
 *         layer writes the two directions into column halves of one buffer
 *         (ld_out = 2*hidden, out + hidden for the reverse direction)
 *   h_n   [batch][hidden] or NULL: the state after the last step processed
 * Asynchronous on `stream`; returns a jst_status.  Arithmetic is fp32 and
 * follows the reference op by op; the GEMMs meet the path's error bound.
 */
int jst_gru_layer_forward(const float* x, int seq, int batch, int input_size, int hidden,
                          const float* w_ih, const float* w_hh, const float* b_ih, const float* b_hh,
                          const float* h0, int reverse, float* out, int64_t ld_out, float* h_n,
                          jst_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* JSTORCH_RNN_H */
