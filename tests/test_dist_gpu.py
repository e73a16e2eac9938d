"""Multi-GPU (one process per GPU) tests of libjstorch_dist.so; skipped with
fewer than two GPUs.  NVLS stays off (NCCL_NVLS_ENABLE=0) in these tests so
a rank that leaves holds no NVLS binding."""
import os

import pytest

from tests.test_dist_cpu import _run
from tests import _dist_workers as W

pytestmark = pytest.mark.gpu


def _ngpus():
    import torch
    return torch.cuda.device_count()


@pytest.fixture(autouse=True)
def _nvls_off(monkeypatch):
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")


@pytest.mark.skipif("_ngpus() < 2")
def test_two_gpus_rowsharded_and_batchsharded():
    out = _run(W.gpu_sharded, world=2, timeout=300)
    for r in (0, 1):
        assert out[r].startswith("ok "), out


@pytest.mark.skipif("_ngpus() < 2")
def test_peer_that_never_joins_times_out_on_the_host():
    out = _run(W.gpu_peer_never_joins, world=2, timeout=120)
    assert out[1] == "left"
    assert out[0].startswith("status 5 after"), out[0]  # JST_ERR_TIMEOUT
    assert float(out[0].split()[3].rstrip("s")) < 30.0
