"""GRU through jst_gru_layer_forward (include/jstorch_rnn.h) on torch CUDA tensors.

Mirrors the reference's nn.GRU (src/nn.js:451-536): PyTorch parameter names
(weight_ih_l{l}[_reverse] [3H, in], weight_hh_l{l} [3H, H], bias_ih_l{l},
bias_hh_l{l} [3H]), gate order (r, z, n), num_layers, bidirectional and
batch_first, forward(x, h0=None) -> (output, h_n).

Training: the reference trains the GRU through GradTensor when its
parameters require grad (nn.js:442-444, 477-485; backward through
autograd.hpp:433-441 for the cell's matmuls and the gate ops' closures).
Here forward_train() runs jst_gru_layer_forward_train and keeps the gate
values, and backward(ctx, dout, dh_n) runs jst_gru_layer_backward per layer
and direction, last layer first: parameter gradients accumulate into
self.grads (as .grad does; zero_grad() clears them) and the gradients of x
and h0 are returned.
"""
from __future__ import annotations

import ctypes

from . import _lib


ACC_DX, ACC_PARAMS, ACC_DH0 = 1, 2, 4  # JST_GRU_ACC_* (include/jstorch_rnn.h)


class _TrainContext:
    """What backward() needs from one forward_train() call."""

    def __init__(self, seq, batch, inps, outs, saved, h0):
        self.seq, self.batch = seq, batch
        self.inps, self.outs, self.saved, self.h0 = inps, outs, saved, h0


class GRU:
    def __init__(self, input_size: int, hidden_size: int, num_layers: int = 1, bidirectional: bool = False,
                 batch_first: bool = False, device="cuda", generator=None):
        import torch
        self.input_size, self.hidden_size = input_size, hidden_size
        self.num_layers, self.bidirectional, self.batch_first = num_layers, bidirectional, batch_first
        dirs = 2 if bidirectional else 1
        self.params = {}
        k = hidden_size ** -0.5
        for l in range(num_layers):
            in_sz = input_size if l == 0 else hidden_size * dirs
            for sfx in ([""] + (["_reverse"] if bidirectional else [])):
                shapes = {f"weight_ih_l{l}{sfx}": (3 * hidden_size, in_sz),
                          f"weight_hh_l{l}{sfx}": (3 * hidden_size, hidden_size),
                          f"bias_ih_l{l}{sfx}": (3 * hidden_size,), f"bias_hh_l{l}{sfx}": (3 * hidden_size,)}
                for name, shp in shapes.items():
                    t = torch.empty(shp, dtype=torch.float32, device=device)
                    t.uniform_(-k, k, generator=generator)
                    self.params[name] = t

    def load_state_dict(self, state: dict) -> None:
        """Copy matching parameters (nn.js:58-80, Module.load_state_dict)."""
        for k, v in state.items():
            if k in self.params:
                if tuple(v.shape) != tuple(self.params[k].shape):
                    raise ValueError(f"{k}: shape {tuple(v.shape)} != {tuple(self.params[k].shape)}")
                self.params[k].copy_(v)

    def __call__(self, x, h0=None):
        return self.forward(x, h0)

    def forward(self, x, h0=None):
        import torch
        if self.batch_first:
            x = x.transpose(0, 1)
        x = x.contiguous()
        if x.dtype != torch.float32 or not x.is_cuda or x.dim() != 3:
            raise ValueError("x must be a 3-D float32 CUDA tensor")
        seq, batch = x.shape[0], x.shape[1]
        H, dirs = self.hidden_size, 2 if self.bidirectional else 1
        if h0 is not None:
            h0 = h0.contiguous()
            if tuple(h0.shape) != (self.num_layers * dirs, batch, H):
                raise ValueError("h0 must be [num_layers * num_directions, batch, hidden]")
        lib = _lib.load()
        stream = torch.cuda.current_stream().cuda_stream
        h_n = torch.empty((self.num_layers * dirs, batch, H), dtype=torch.float32, device=x.device)
        inp = x
        for l in range(self.num_layers):
            out = torch.empty((seq, batch, H * dirs), dtype=torch.float32, device=x.device)
            for d in range(dirs):
                sfx = "_reverse" if d else ""
                p = self.params
                h0p = h0[l * dirs + d].data_ptr() if h0 is not None else None
                _lib.check(lib.jst_gru_layer_forward(
                    inp.data_ptr(), seq, batch, inp.shape[2], H, p[f"weight_ih_l{l}{sfx}"].data_ptr(),
                    p[f"weight_hh_l{l}{sfx}"].data_ptr(), p[f"bias_ih_l{l}{sfx}"].data_ptr(),
                    p[f"bias_hh_l{l}{sfx}"].data_ptr(), h0p, d, out.data_ptr() + 4 * d * H, H * dirs,
                    h_n[l * dirs + d].data_ptr(), stream))
            inp = out
        if self.batch_first:
            inp = inp.transpose(0, 1)
        return inp, h_n

    # ------------------------------------------------------------ training
    def zero_grad(self) -> None:
        """Clear the accumulated parameter gradients (self.grads)."""
        for g in getattr(self, "grads", {}).values():
            g.zero_()

    def _check_x(self, x, h0):
        import torch
        if self.batch_first:
            x = x.transpose(0, 1)
        x = x.contiguous()
        if x.dtype != torch.float32 or not x.is_cuda or x.dim() != 3:
            raise ValueError("x must be a 3-D float32 CUDA tensor")
        dirs = 2 if self.bidirectional else 1
        if h0 is not None:
            h0 = h0.contiguous()
            if tuple(h0.shape) != (self.num_layers * dirs, x.shape[1], self.hidden_size):
                raise ValueError("h0 must be [num_layers * num_directions, batch, hidden]")
        return x, h0

    def forward_train(self, x, h0=None):
        """forward() that also keeps the gate values of every step for
        backward(); returns (output, h_n, ctx)."""
        import torch
        x, h0 = self._check_x(x, h0)
        seq, batch = x.shape[0], x.shape[1]
        H, dirs = self.hidden_size, 2 if self.bidirectional else 1
        lib = _lib.load()
        stream = torch.cuda.current_stream().cuda_stream
        h_n = torch.empty((self.num_layers * dirs, batch, H), dtype=torch.float32, device=x.device)
        inps, outs, saved = [], [], []
        inp = x
        for l in range(self.num_layers):
            out = torch.empty((seq, batch, H * dirs), dtype=torch.float32, device=x.device)
            sv = [torch.empty((seq, batch, 4 * H), dtype=torch.float32, device=x.device) for _ in range(dirs)]
            for d in range(dirs):
                sfx = "_reverse" if d else ""
                p = self.params
                h0p = h0[l * dirs + d].data_ptr() if h0 is not None else None
                _lib.check(lib.jst_gru_layer_forward_train(
                    inp.data_ptr(), seq, batch, inp.shape[2], H, p[f"weight_ih_l{l}{sfx}"].data_ptr(),
                    p[f"weight_hh_l{l}{sfx}"].data_ptr(), p[f"bias_ih_l{l}{sfx}"].data_ptr(),
                    p[f"bias_hh_l{l}{sfx}"].data_ptr(), h0p, d, out.data_ptr() + 4 * d * H, H * dirs,
                    h_n[l * dirs + d].data_ptr(), sv[d].data_ptr(), stream))
            inps.append(inp)
            outs.append(out)
            saved.append(sv)
            inp = out
        ctx = _TrainContext(seq, batch, inps, outs, saved, h0)
        output = inp.transpose(0, 1) if self.batch_first else inp
        return output, h_n, ctx

    def backward(self, ctx, dout, dh_n=None):
        """Back-propagate dL/d(output) (and dL/d(h_n)) through the pass of
        forward_train that produced ctx.  Adds every parameter's gradient to
        self.grads[name]; returns (dx, dh0) (dh0 None when no h0 was given)."""
        import torch
        if not hasattr(self, "grads"):
            self.grads = {k: torch.zeros_like(v) for k, v in self.params.items()}
        if self.batch_first:
            dout = dout.transpose(0, 1)
        g = dout.contiguous()
        seq, batch = ctx.seq, ctx.batch
        H, dirs = self.hidden_size, 2 if self.bidirectional else 1
        if tuple(g.shape) != (seq, batch, H * dirs):
            raise ValueError("dout must have the output's shape")
        if dh_n is not None:
            dh_n = dh_n.contiguous()
        lib = _lib.load()
        stream = torch.cuda.current_stream().cuda_stream
        dh0 = torch.empty_like(ctx.h0) if ctx.h0 is not None else None
        for l in range(self.num_layers - 1, -1, -1):
            inp, out = ctx.inps[l], ctx.outs[l]
            dinp = torch.empty_like(inp)
            for d in range(dirs):
                sfx = "_reverse" if d else ""
                p, gr = self.params, self.grads
                k = l * dirs + d
                acc = ACC_PARAMS | (ACC_DX if d else 0)
                _lib.check(lib.jst_gru_layer_backward(
                    inp.data_ptr(), seq, batch, inp.shape[2], H, p[f"weight_ih_l{l}{sfx}"].data_ptr(),
                    p[f"weight_hh_l{l}{sfx}"].data_ptr(), ctx.h0[k].data_ptr() if ctx.h0 is not None else None, d,
                    out.data_ptr() + 4 * d * H, H * dirs, ctx.saved[l][d].data_ptr(), g.data_ptr() + 4 * d * H,
                    H * dirs, dh_n[k].data_ptr() if dh_n is not None else None, dinp.data_ptr(),
                    gr[f"weight_ih_l{l}{sfx}"].data_ptr(), gr[f"weight_hh_l{l}{sfx}"].data_ptr(),
                    gr[f"bias_ih_l{l}{sfx}"].data_ptr(), gr[f"bias_hh_l{l}{sfx}"].data_ptr(),
                    dh0[k].data_ptr() if dh0 is not None else None, acc, stream))
            g = dinp
        dx = g.transpose(0, 1) if self.batch_first else g
        return dx, dh0
