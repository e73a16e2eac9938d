"""jst_gru_layer_forward (include/jstorch_rnn.h) through jstorch_b200.rnn.GRU,
the reference's GRU (src/nn.js:451-536), against the fp64 oracle.

Bound: |h - h_ref| <= 2e-5 absolute on every output and final state (states
lie in (-1, 1); the fp32 GEMMs meet the path's 2e-6 bound and the gate math
is fp32 like the reference's)."""
import numpy as np
import pytest

from oracle import oracle

pytestmark = pytest.mark.gpu
ATOL = 2e-5


def _run(seq, batch, inp, H, layers, bidir, with_h0, batch_first=False, seed=0):
    import torch
    from jstorch_b200.rnn import GRU
    g = torch.Generator(device="cuda").manual_seed(seed)
    gru = GRU(inp, H, layers, bidir, batch_first, generator=g)
    rng = np.random.default_rng(seed)
    dirs = 2 if bidir else 1
    x = rng.standard_normal((seq, batch, inp)).astype(np.float32)
    h0 = rng.standard_normal((layers * dirs, batch, H)).astype(np.float32) * 0.5 if with_h0 else None
    xt = torch.from_numpy(x).cuda()
    if batch_first:
        xt = xt.transpose(0, 1).contiguous()
    out, hn = gru(xt, torch.from_numpy(h0).cuda() if with_h0 else None)
    torch.cuda.synchronize()
    out = out.cpu().numpy()
    if batch_first:
        out = out.transpose(1, 0, 2)
    params = {k: v.cpu().numpy() for k, v in gru.params.items()}
    ref_out, ref_hn = oracle.gru_forward_f64(x, params, H, layers, bidir, h0)
    assert out.shape == ref_out.shape and hn.shape == ref_hn.shape
    assert np.max(np.abs(out - ref_out)) <= ATOL, np.max(np.abs(out - ref_out))
    assert np.max(np.abs(hn.cpu().numpy() - ref_hn)) <= ATOL


@pytest.mark.parametrize("seq,batch,inp,H,layers,bidir,with_h0", [
    (5, 3, 7, 9, 1, False, False),       # odd sizes, zero initial state
    (12, 16, 64, 128, 2, True, True),    # stacked, bidirectional, given h0
    (40, 64, 256, 512, 1, False, True),  # recurrent GEMMs of a realistic size (tensor-core step)
    (10, 24, 96, 512, 2, True, True),    # tensor-core step, bidirectional, batch not a multiple of 4
    (7, 24, 40, 510, 1, False, True),    # tensor-core step, H not a multiple of 4 (zero plane padding)
    (3, 1, 1, 1, 1, True, False),        # the degenerate one-unit case
])
def test_gru_against_oracle(seq, batch, inp, H, layers, bidir, with_h0):
    _run(seq, batch, inp, H, layers, bidir, with_h0, seed=seq + H)


def test_gru_batch_first():
    _run(6, 4, 8, 16, 2, False, True, batch_first=True, seed=3)


def test_gru_large_projection_on_tensor_cores():
    """seq*batch x 3H x in large enough that the all-steps input projection
    runs on the tensor-core kernel."""
    from jstorch_b200 import select_kernel
    assert select_kernel(64 * 128, 3 * 1024, 1024) == "tc3xtf32"
    _run(64, 128, 1024, 1024, 1, False, False, seed=9)
