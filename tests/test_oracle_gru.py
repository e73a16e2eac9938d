"""Pins the GRU restatement of the oracle (oracle.gru_forward_f64, restating
src/nn.js:451-536) against an independent implementation: torch.nn.GRU in
fp64 on the CPU.  CPU only."""
import numpy as np
import pytest
import torch

from oracle import oracle


@pytest.mark.parametrize("layers,bidir,with_h0", [(1, False, False), (2, True, True), (2, False, True)])
def test_gru_oracle_against_torch(layers, bidir, with_h0):
    """oracle.gru_forward_f64 (restating src/nn.js:451-536) against torch.nn.GRU
    in fp64, which uses the same gate equations and parameter names."""
    rng = np.random.default_rng(layers * 10 + bidir)
    seq, batch, inp, H = 7, 3, 5, 4
    gru = torch.nn.GRU(inp, H, num_layers=layers, bidirectional=bidir).double()
    params = {k: v.detach().numpy() for k, v in gru.named_parameters()}
    x = rng.standard_normal((seq, batch, inp))
    dirs = 2 if bidir else 1
    h0 = rng.standard_normal((layers * dirs, batch, H)) if with_h0 else None
    out_t, hn_t = gru(torch.from_numpy(x), torch.from_numpy(h0) if with_h0 else None)
    out, hn = oracle.gru_forward_f64(x, params, H, layers, bidir, h0)
    np.testing.assert_allclose(out, out_t.detach().numpy(), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(hn, hn_t.detach().numpy(), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("layers,bidir,with_h0", [(1, False, False), (2, True, True), (3, False, True)])
def test_gru_backward_oracle_against_torch_autograd(layers, bidir, with_h0):
    """oracle.gru_backward_f64 against torch autograd through torch.nn.GRU in
    fp64: every parameter gradient, dx and dh0 for L = sum(dout * output) +
    sum(dh_n * h_n)."""
    rng = np.random.default_rng(100 + layers * 10 + bidir)
    seq, batch, inp, H = 6, 3, 5, 4
    gru = torch.nn.GRU(inp, H, num_layers=layers, bidirectional=bidir).double()
    params = {k: v.detach().numpy() for k, v in gru.named_parameters()}
    dirs = 2 if bidir else 1
    x = torch.from_numpy(rng.standard_normal((seq, batch, inp))).requires_grad_(True)
    h0 = torch.from_numpy(rng.standard_normal((layers * dirs, batch, H))).requires_grad_(True) if with_h0 else None
    dout = rng.standard_normal((seq, batch, H * dirs))
    dhn = rng.standard_normal((layers * dirs, batch, H))
    out, hn = gru(x, h0)
    ((out * torch.from_numpy(dout)).sum() + (hn * torch.from_numpy(dhn)).sum()).backward()
    grads, dx, dh0 = oracle.gru_backward_f64(x.detach().numpy(), params, H, layers, bidir,
                                             h0.detach().numpy() if with_h0 else None, dout, dhn)
    for k, v in gru.named_parameters():
        np.testing.assert_allclose(grads[k], v.grad.numpy(), rtol=1e-10, atol=1e-12, err_msg=k)
    np.testing.assert_allclose(dx, x.grad.numpy(), rtol=1e-10, atol=1e-12)
    if with_h0:
        np.testing.assert_allclose(dh0, h0.grad.numpy(), rtol=1e-10, atol=1e-12)
    else:
        assert dh0 is None
