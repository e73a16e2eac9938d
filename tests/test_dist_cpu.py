"""Multi-rank host logic on CPU (gloo, world size 2): the block-cyclic row
plan of jst_gemm_rowsharded, its all-gather layout, and failure detection
when a rank leaves."""
import multiprocessing as mp
import socket

import pytest

from jstorch_b200 import dist as jdist
from tests import _dist_workers as W


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, msg = q.get(timeout=timeout)
        out[r] = msg
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("nranks,m_local,chunk", [(1, 64, 64), (2, 96, 32), (8, 8192, 2048), (3, 30, 10)])
def test_row_plan_covers_every_row_once(nranks, m_local, chunk):
    seen = []
    for r in range(nranks):
        plan = jdist.row_plan(nranks, r, m_local, chunk)
        assert [b.local_row0 for b in plan] == list(range(0, m_local, chunk))
        for b in plan:
            seen.extend(range(b.global_row0, b.global_row0 + b.rows))
    assert sorted(seen) == list(range(nranks * m_local))
    # each all-gather round is one contiguous slab of C_full ordered by rank
    for i in range(m_local // chunk):
        starts = [jdist.row_plan(nranks, r, m_local, chunk)[i].global_row0 for r in range(nranks)]
        assert starts == [i * nranks * chunk + r * chunk for r in range(nranks)]


def test_row_plan_plain_blocks_when_one_chunk():
    assert jdist.row_plan(4, 2, 100, 100) == [jdist.RowBlock(0, 200, 100)]
    with pytest.raises(ValueError):
        jdist.row_plan(2, 0, 100, 30)


def test_gloo_two_ranks_rowsharded_layout():
    out = _run(W.gloo_rowsharded_layout)
    assert out == {0: "ok", 1: "ok"}, out


def test_gloo_two_ranks_batchsharded_layout():
    out = _run(W.gloo_batchsharded_layout)
    assert out == {0: "ok", 1: "ok"}, out


def test_gloo_rank_leaves_survivor_errors():
    out = _run(W.gloo_rank_dies)
    assert out[1] == "left"
    assert out[0].startswith("error after"), out[0]
