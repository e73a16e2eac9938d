"""GRU training through jst_gru_layer_forward_train / jst_gru_layer_backward
(include/jstorch_rnn.h) via jstorch_b200.rnn.GRU, against the fp64 oracle
(oracle.gru_backward_f64, pinned against torch autograd).

The reference trains its GRU through GradTensor (src/nn.js:442-444, 477-485;
native/core/autograd.hpp:433-441 for the cell's matmuls).  Checked: every
parameter gradient, dx and dh0, for L = sum(dout * output) + sum(dh_n * h_n).

Bound: for each gradient tensor, max |G - G_ref| <= RTOL * max |G_ref|.  The
GEMMs meet the path's 2e-6 bound; the gate arithmetic is fp32 and its
rounding errors compound through the steps of the recurrence.  Measured on a
B200: 1e-7 .. 9e-7 for the cases below, 3.9e-6 for 8 steps and 1.4e-5 for 64
steps at hidden 1024 (the weight gradients of the recurrent product), so
RTOL = 1e-4 leaves about 7x margin at the longest sequence measured."""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu
RTOL = 1e-4


def _setup(seq, batch, inp, H, layers, bidir, with_h0, batch_first=False, seed=0):
    import torch
    from jstorch_b200.rnn import GRU
    g = torch.Generator(device="cuda").manual_seed(seed)
    gru = GRU(inp, H, layers, bidir, batch_first, generator=g)
    rng = np.random.default_rng(seed)
    dirs = 2 if bidir else 1
    x = rng.standard_normal((seq, batch, inp)).astype(np.float32)
    h0 = (rng.standard_normal((layers * dirs, batch, H)) * 0.5).astype(np.float32) if with_h0 else None
    dout = rng.standard_normal((seq, batch, H * dirs)).astype(np.float32)
    dhn = rng.standard_normal((layers * dirs, batch, H)).astype(np.float32)
    return gru, x, h0, dout, dhn


def _to_dev(a, batch_first=False):
    import torch
    if a is None:
        return None
    t = torch.from_numpy(a).cuda()
    return t.transpose(0, 1).contiguous() if batch_first else t


def _rel(got, ref):
    scale = float(np.max(np.abs(ref)))
    return float(np.max(np.abs(got - ref))) / (scale if scale > 0 else 1.0)


def _check(seq, batch, inp, H, layers, bidir, with_h0, batch_first=False, seed=0):
    import torch
    gru, x, h0, dout, dhn = _setup(seq, batch, inp, H, layers, bidir, with_h0, batch_first, seed)
    out, hn, ctx = gru.forward_train(_to_dev(x, batch_first), _to_dev(h0))
    dx, dh0 = gru.backward(ctx, _to_dev(dout, batch_first), _to_dev(dhn))
    torch.cuda.synchronize()
    params = {k: v.cpu().numpy() for k, v in gru.params.items()}
    ref_out, ref_hn = oracle.gru_forward_f64(x, params, H, layers, bidir, h0)
    o = out.cpu().numpy()
    if batch_first:
        o = o.transpose(1, 0, 2)
    assert np.max(np.abs(o - ref_out)) <= 2e-5  # the training forward is the inference forward
    assert np.max(np.abs(hn.cpu().numpy() - ref_hn)) <= 2e-5
    grads, ref_dx, ref_dh0 = oracle.gru_backward_f64(x, params, H, layers, bidir, h0, dout, dhn)
    errs = {k: _rel(gru.grads[k].cpu().numpy(), v) for k, v in grads.items()}
    d = dx.cpu().numpy()
    if batch_first:
        d = d.transpose(1, 0, 2)
    errs["dx"] = _rel(d, ref_dx)
    if with_h0:
        errs["dh0"] = _rel(dh0.cpu().numpy(), ref_dh0)
    else:
        assert dh0 is None
    worst = max(errs, key=errs.get)
    assert errs[worst] <= RTOL, (worst, errs[worst], errs)
    return gru, errs


@pytest.mark.parametrize("seq,batch,inp,H,layers,bidir,with_h0", [
    (5, 3, 7, 9, 1, False, False),       # odd sizes, FFMA recurrent products
    (12, 16, 64, 128, 2, True, True),    # stacked, bidirectional, given h0
    (10, 24, 96, 512, 2, True, True),    # tensor-core recurrent products, bidirectional, 2 layers
    (7, 24, 40, 510, 1, False, True),    # tensor-core step, 3H not a multiple of 4 (plane padding)
    (1, 5, 6, 8, 1, True, True),         # one step: the only product is dh0's
    (3, 1, 1, 1, 1, True, False),        # the degenerate one-unit case
])
def test_gru_gradients_against_oracle(seq, batch, inp, H, layers, bidir, with_h0):
    _check(seq, batch, inp, H, layers, bidir, with_h0, seed=seq * 7 + H)


def test_gru_gradients_batch_first():
    _check(6, 4, 8, 16, 2, True, True, batch_first=True, seed=5)


def test_gru_realistic_two_layer_bidirectional():
    """The bench's shape family at reduced length: 2 layers, bidirectional,
    hidden 1024, every product on the tensor cores."""
    _check(8, 64, 512, 1024, 2, True, False, seed=11)


def test_gru_gradients_accumulate_over_backward_calls():
    import torch
    gru, x, h0, dout, dhn = _setup(6, 32, 48, 256, 1, True, True, seed=21)
    out, hn, ctx = gru.forward_train(_to_dev(x), _to_dev(h0))
    gru.backward(ctx, _to_dev(dout), _to_dev(dhn))
    once = {k: v.clone() for k, v in gru.grads.items()}
    gru.backward(ctx, _to_dev(dout), _to_dev(dhn))
    torch.cuda.synchronize()
    for k, v in gru.grads.items():
        assert torch.equal(v, 2 * once[k]), k  # x + x is exact
    gru.zero_grad()
    assert all(float(v.abs().max()) == 0.0 for v in gru.grads.values())
