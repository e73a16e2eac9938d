"""Rank bodies for the multi-process tests (imported by spawned processes)."""
from __future__ import annotations

import os
import time
import traceback

import numpy as np


def _init_pg(rank: int, world: int, port: int, backend: str = "gloo", timeout_s: float = 20.0):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def gloo_rowsharded_layout(rank: int, world: int, port: int, out_q) -> None:
    """Host logic of the row-sharded GEMM on CPU ranks: each rank takes the
    rows row_plan gives it, multiplies them with the fp64 oracle and places
    them in C_full exactly where jst_gemm_rowsharded's in-place all-gather
    rounds put them (gloo all_gather per round)."""
    try:
        import torch

        from jstorch_b200 import dist as jdist
        from jstorch_b200 import synth
        from oracle import oracle

        d = _init_pg(rank, world, port)
        m_local, k, n, chunk = 96, 40, 56, 32
        plan = jdist.row_plan(world, rank, m_local, chunk)
        a_local = np.concatenate([synth.matrix(9, synth.A, blk.rows, k, "uniform", row0=blk.global_row0)
                                  for blk in plan])
        b = synth.matrix(9, synth.B, k, n, "uniform") if rank == 0 else np.zeros((k, n), np.float32)
        bt = torch.from_numpy(b)
        d.broadcast(bt, src=0)  # the B broadcast
        b = bt.numpy()
        c_local = oracle.gemm_f64(a_local, b).astype(np.float32)
        c_full = np.zeros((m_local * world, n), np.float32)
        for i, blk in enumerate(plan):  # one all-gather round per block index
            parts = [torch.zeros((chunk, n)) for _ in range(world)]
            d.all_gather(parts, torch.from_numpy(c_local[blk.local_row0:blk.local_row0 + chunk]))
            c_full[i * world * chunk:(i + 1) * world * chunk] = torch.cat(parts).numpy()
        a_full = synth.matrix(9, synth.A, m_local * world, k, "uniform")
        ref = oracle.gemm_f64(a_full, b).astype(np.float32)
        out_q.put((rank, "ok" if np.array_equal(c_full, ref) else "mismatch"))
        d.destroy_process_group()
    except Exception:
        out_q.put((rank, traceback.format_exc()))


def gloo_batchsharded_layout(rank: int, world: int, port: int, out_q) -> None:
    """Host logic of jst_bmm_batchsharded on CPU ranks: rank r owns batches
    [r*bl, (r+1)*bl) of A and B, multiplies them with the fp64 oracle into
    its slice of C_full, and one all-gather (gloo, the same layout as the
    in-place ncclAllGather) fills every rank's C_full.  Checked for both
    config-4 shapes at reduced size."""
    try:
        import torch

        from jstorch_b200 import synth
        from oracle import oracle

        d = _init_pg(rank, world, port)
        ok = True
        for (M, K, N) in ((32, 8, 32), (32, 32, 8)):
            bl = 3
            A = synth.matrix(3, synth.A, bl * world * M, K, "normal", 0.35).reshape(bl * world, M, K)
            B = synth.matrix(3, synth.B, bl * world * K, N, "normal", 0.35).reshape(bl * world, K, N)
            mine = slice(rank * bl, (rank + 1) * bl)
            c_local = oracle.gemm_f64(A[mine], B[mine]).astype(np.float32)
            parts = [torch.zeros((bl, M, N)) for _ in range(world)]
            d.all_gather(parts, torch.from_numpy(c_local))
            c_full = torch.cat(parts).numpy()
            ref = oracle.gemm_f64(A, B).astype(np.float32)
            ok = ok and np.array_equal(c_full, ref)
        out_q.put((rank, "ok" if ok else "mismatch"))
        d.destroy_process_group()
    except Exception:
        out_q.put((rank, traceback.format_exc()))


def gloo_rank_dies(rank: int, world: int, port: int, out_q) -> None:
    """Failure path on the host: rank 1 leaves before the collective; rank 0's
    next collective must end with an error within the group timeout."""
    try:
        import torch

        d = _init_pg(rank, world, port, timeout_s=5.0)
        if rank == 1:
            out_q.put((rank, "left"))
            out_q.close()
            out_q.join_thread()  # flush the message before dying
            os._exit(0)  # dies between steps, with nothing in flight
        t0 = time.time()
        try:
            d.all_gather([torch.zeros(4) for _ in range(world)], torch.ones(4))
            out_q.put((rank, "no error"))
        except Exception as e:  # the expected outcome
            out_q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    except Exception:
        out_q.put((rank, traceback.format_exc()))


def gpu_sharded(rank: int, world: int, port: int, out_q) -> None:
    """Row-sharded GEMM and batch-sharded bmm on `world` GPUs vs the oracle."""
    try:
        import torch

        from jstorch_b200 import dist as jdist
        from jstorch_b200 import synth
        from oracle import oracle

        torch.cuda.set_device(rank)
        d = _init_pg(rank, world, port)
        comm = jdist.Comm.from_process_group(timeout_s=30.0)
        m_local, k, n, chunk = 768, 320, 1024, 256
        plan = jdist.row_plan(world, rank, m_local, chunk)
        a_local = np.concatenate([synth.matrix(4, synth.A, blk.rows, k, "uniform", row0=blk.global_row0)
                                  for blk in plan])
        b_host = synth.matrix(4, synth.B, k, n, "uniform")
        a = torch.from_numpy(a_local).cuda()
        b = torch.from_numpy(b_host if rank == 0 else np.zeros_like(b_host)).cuda()  # only the root holds B
        c = torch.full((m_local * world, n), float("nan"), device="cuda")
        st = torch.cuda.current_stream()
        comm.gemm_rowsharded(a, b, c, chunk, root=0, stream=st)
        comm.sync(st)
        a_full = synth.matrix(4, synth.A, m_local * world, k, "uniform")
        ref = oracle.gemm_f64(a_full, b_host)
        err, where = oracle.max_rel_err(a_full, b_host, c.cpu().numpy(), ref)
        msgs = [f"rowsharded err {err:.2e}"]
        ok = err <= 2e-6 and np.array_equal(b.cpu().numpy(), b_host)
        # batch-sharded bmm: rank r owns batches [r*bl, (r+1)*bl)
        bl, M, K, N = 3, 70, 48, 90
        A = synth.matrix(5, synth.A, bl * world * M, K, "normal").reshape(bl * world, M, K)
        B = synth.matrix(5, synth.B, bl * world * K, N, "normal").reshape(bl * world, K, N)
        cf = torch.full((bl * world, M, N), float("nan"), device="cuda")
        comm.bmm_batchsharded(torch.from_numpy(A[rank * bl:(rank + 1) * bl].copy()).cuda(),
                              torch.from_numpy(B[rank * bl:(rank + 1) * bl].copy()).cuda(), cf, stream=st)
        comm.sync(st)
        err2, _ = oracle.max_rel_err(A, B, cf.cpu().numpy(), oracle.gemm_f64(A, B))
        msgs.append(f"batchsharded err {err2:.2e}")
        ok = ok and err2 <= 2e-6
        # copy-engine path: C registered with every rank
        cr = torch.full((m_local * world, n), float("nan"), device="cuda")
        reg = comm.register(cr)
        try:
            b.zero_() if rank != 0 else None
            comm.gemm_rowsharded(a, b, cr, chunk, root=0, stream=st)
            comm.sync(st)
            err4, _ = oracle.max_rel_err(a_full, b_host, cr.cpu().numpy(), ref)
            msgs.append(f"copy-engine err {err4:.2e}")
            ok = ok and err4 <= 2e-6
        finally:
            reg.deregister()
        # fused path: C in a multicast-backed buffer, no all-gather collective
        buf = comm.symm_alloc(m_local * world * n * 4)
        try:
            cs = buf.tensor((m_local * world, n))
            cs.fill_(float("nan"))
            b.zero_() if rank != 0 else None
            comm.gemm_rowsharded(a, b, cs, chunk, root=0, stream=st)
            comm.sync(st)
            err3, _ = oracle.max_rel_err(a_full, b_host, cs.cpu().numpy(), ref)
            msgs.append(f"fused multicast err {err3:.2e}")
            ok = ok and err3 <= 2e-6 and np.array_equal(b.cpu().numpy(), b_host)  # B arrived in place too
        finally:
            buf.free()
        # fused path, ragged: K not a multiple of 4, last panel of B 232 columns wide
        k2, n2 = 317, 1000
        a2_local = np.concatenate([synth.matrix(6, synth.A, blk.rows, k2, "normal", row0=blk.global_row0)
                                   for blk in plan])
        b2_host = synth.matrix(6, synth.B, k2, n2, "normal")
        b2 = torch.from_numpy(b2_host if rank == 0 else np.zeros_like(b2_host)).cuda()
        buf2 = comm.symm_alloc(m_local * world * n2 * 4)
        try:
            cs2 = buf2.tensor((m_local * world, n2))
            cs2.fill_(float("nan"))
            a2 = torch.from_numpy(a2_local).cuda()  # alive until the sync: read on the library's own streams too
            comm.gemm_rowsharded(a2, b2, cs2, chunk, root=0, stream=st)
            comm.sync(st)
            a2_full = synth.matrix(6, synth.A, m_local * world, k2, "normal")
            err5, _ = oracle.max_rel_err(a2_full, b2_host, cs2.cpu().numpy(), oracle.gemm_f64(a2_full, b2_host))
            msgs.append(f"fused multicast ragged err {err5:.2e}")
            ok = ok and err5 <= 2e-6 and np.array_equal(b2.cpu().numpy(), b2_host)
        finally:
            buf2.free()
        comm.destroy()
        d.destroy_process_group()
        out_q.put((rank, ("ok " if ok else "FAIL ") + "; ".join(msgs)))
    except Exception:
        out_q.put((rank, traceback.format_exc()))


def gpu_peer_never_joins(rank: int, world: int, port: int, out_q) -> None:
    """jst_comm_init on rank 0 while rank 1 never creates its communicator:
    the host deadline must end the call with JST_ERR_TIMEOUT."""
    try:
        import torch

        from jstorch_b200 import _lib
        from jstorch_b200 import dist as jdist

        torch.cuda.set_device(rank)
        d = _init_pg(rank, world, port)
        obj = [jdist.Comm.unique_id() if rank == 0 else None]
        d.broadcast_object_list(obj, src=0)
        if rank == 1:
            out_q.put((rank, "left"))
            out_q.close()
            out_q.join_thread()
            os._exit(0)  # never joins the NCCL communicator
        t0 = time.time()
        try:
            jdist.Comm(world, rank, obj[0], timeout_s=5.0)
            out_q.put((rank, "no error"))
        except _lib.JstError as e:
            out_q.put((rank, f"status {e.status} after {time.time() - t0:.1f}s"))
        out_q.close()
        out_q.join_thread()
        os._exit(0)
    except Exception:
        out_q.put((rank, traceback.format_exc()))
