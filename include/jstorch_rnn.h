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

/*
 * Training forward: jst_gru_layer_forward that also keeps what the backward
 * pass needs.  saved [seq][batch][4*hidden] receives, per step and batch row,
 * r, z, n and the n-gate's recurrent term gh_n = (h W_hn^T + b_hn), the
 * intermediate values GradTensor keeps alive for its closures when the
 * reference GRU runs with parameters that require grad (nn.js:442-444,
 * 477-485).  Same outputs as jst_gru_layer_forward.
 */
int jst_gru_layer_forward_train(const float* x, int seq, int batch, int input_size, int hidden,
                                const float* w_ih, const float* w_hh, const float* b_ih, const float* b_hh,
                                const float* h0, int reverse, float* out, int64_t ld_out, float* h_n,
                                float* saved, jst_stream_t stream);

/*
 * Backward of one layer and direction after jst_gru_layer_forward_train
 * (what GradTensor's backward sweep, native/core/autograd.hpp:40-65, computes
 * through the cell's two matmuls, autograd.hpp:433-441, and its gate ops):
 *   x, w_ih, w_hh, h0, reverse, out / ld_out, saved: as given to / written by
 *         the training forward (h0 NULL = zeros)
 *   dout  [seq][batch][ld_dout]: dL/d(out) for this direction's columns, or
 *         NULL (zero)
 *   dh_n  [batch][hidden]: dL/d(h_n), or NULL (zero)
 * Outputs (each may be NULL to skip it):
 *   dx    [seq][batch][input_size]    dw_ih [3*hidden][input_size]
 *   dw_hh [3*hidden][hidden]          db_ih, db_hh [3*hidden]
 *   dh0   [batch][hidden]
 * accumulate: a mask of JST_GRU_ACC_* bits; an output whose bit is set is
 * added to its contents, the others are overwritten (the two directions of a
 * bidirectional layer sum into one dx; repeated backward calls accumulate
 * parameter gradients as GradTensor's .grad does).
 * Per step one fused gate-backward kernel and one product dgh . W_hh (on the
 * tensor cores at realistic sizes); the weight gradients of all steps are one
 * GEMM each afterwards.  Asynchronous on `stream`; returns a jst_status.
 */
enum { JST_GRU_ACC_DX = 1, JST_GRU_ACC_PARAMS = 2, JST_GRU_ACC_DH0 = 4 };
int jst_gru_layer_backward(const float* x, int seq, int batch, int input_size, int hidden,
                           const float* w_ih, const float* w_hh, const float* h0, int reverse,
                           const float* out, int64_t ld_out, const float* saved,
                           const float* dout, int64_t ld_dout, const float* dh_n,
                           float* dx, float* dw_ih, float* dw_hh, float* db_ih, float* db_hh, float* dh0,
                           int accumulate, jst_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* JSTORCH_RNN_H */
