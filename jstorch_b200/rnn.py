"""GRU through jst_gru_layer_forward (include/jstorch_rnn.h) on torch CUDA tensors.

Mirrors the reference's nn.GRU (src/nn.js:451-536): PyTorch parameter names
(weight_ih_l{l}[_reverse] [3H, in], weight_hh_l{l} [3H, H], bias_ih_l{l},
bias_hh_l{l} [3H]), gate order (r, z, n), num_layers, bidirectional and
batch_first, forward(x, h0=None) -> (output, h_n).  Inference forward only.
"""
from __future__ import annotations

import ctypes

from . import _lib


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
