"""Multi-GPU face of the path: one process per GPU, libjstorch_dist.so
(include/jstorch_dist.h) for the NCCL row-sharded GEMM and batch-sharded bmm.

torch.distributed (any backend; gloo is enough) is used only to hand the
communicator id from rank 0 to the others; all data moves through the
library's own NCCL communicator.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

from . import _lib

LIB_PATH = Path(__file__).resolve().parent / "libjstorch_dist.so"
ID_BYTES = 128
_dlib = None


def load() -> ctypes.CDLL:
    global _dlib
    if _dlib is None:
        _lib.load()  # libjstorch_gemm.so first (status messages live there)
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m jstorch_b200.build`")
        d = ctypes.CDLL(str(LIB_PATH))
        vp, ci, cd = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
        d.jst_comm_get_unique_id.restype = ci
        d.jst_comm_get_unique_id.argtypes = [ctypes.c_char_p]
        d.jst_comm_init.restype = ci
        d.jst_comm_init.argtypes = [ctypes.POINTER(vp), ci, ci, ctypes.c_char_p, cd]
        d.jst_comm_sync.restype = ci
        d.jst_comm_sync.argtypes = [vp, vp]
        d.jst_comm_destroy.restype = ci
        d.jst_comm_destroy.argtypes = [vp]
        d.jst_comm_rank.restype = ci
        d.jst_comm_rank.argtypes = [vp]
        d.jst_comm_size.restype = ci
        d.jst_comm_size.argtypes = [vp]
        d.jst_gemm_rowsharded.restype = ci
        d.jst_gemm_rowsharded.argtypes = [vp, vp, ci, ci, vp, ci, ci, vp, ci, vp]
        d.jst_bmm_batchsharded.restype = ci
        d.jst_bmm_batchsharded.argtypes = [vp, vp, vp, ci, ci, ci, ci, vp, vp]
        d.jst_comm_trace.restype = ci
        d.jst_comm_trace.argtypes = [vp, ci]
        d.jst_comm_trace_read.restype = ci
        d.jst_comm_trace_read.argtypes = [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ci]
        d.jst_comm_register.restype = ci
        d.jst_comm_register.argtypes = [vp, vp, ctypes.c_size_t, ctypes.POINTER(vp)]
        d.jst_comm_deregister.restype = ci
        d.jst_comm_deregister.argtypes = [vp]
        d.jst_symm_alloc.restype = ci
        d.jst_symm_alloc.argtypes = [vp, ctypes.c_size_t, ctypes.POINTER(vp), ctypes.POINTER(vp)]
        d.jst_symm_free.restype = ci
        d.jst_symm_free.argtypes = [vp]
        _dlib = d
    return _dlib


@dataclass(frozen=True)
class RowBlock:
    local_row0: int   # first row of the block in this rank's A_local / C rows
    global_row0: int  # first row of the block in the global A / C_full
    rows: int


def row_plan(nranks: int, rank: int, m_local: int, chunk_rows: int) -> list[RowBlock]:
    """Row blocks owned by `rank` in jst_gemm_rowsharded's block-cyclic layout:
    block i of rank r holds global rows (i * nranks + r) * chunk_rows + [0, chunk_rows)."""
    if chunk_rows < 1 or m_local % chunk_rows:
        raise ValueError("m_local must be a positive multiple of chunk_rows")
    return [RowBlock(i * chunk_rows, (i * nranks + rank) * chunk_rows, chunk_rows)
            for i in range(m_local // chunk_rows)]


class _DeviceArray:
    """Minimal __cuda_array_interface__ so torch can view library-owned memory."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


class SymmBuffer:
    """A multicast-backed buffer on every rank (jst_symm_alloc): a row-sharded
    GEMM whose C lives here fuses its all-gather into the kernel epilogue."""

    def __init__(self, comm: "Comm", nbytes: int):
        h, p = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(load().jst_symm_alloc(comm.handle, nbytes, ctypes.byref(h), ctypes.byref(p)))
        self.handle, self.ptr, self.nbytes = h, p.value, nbytes

    def tensor(self, shape, dtype=None):
        """A torch CUDA tensor viewing this rank's copy (no copy, fp32)."""
        import torch

        n = 1
        for d in shape:
            n *= d
        if n * 4 > self.nbytes:
            raise ValueError("shape exceeds the buffer")
        return torch.as_tensor(_DeviceArray(self.ptr, tuple(shape)), device="cuda")

    def free(self) -> None:
        """Collective release (every rank, after its last use)."""
        if self.handle:
            rc = load().jst_symm_free(self.handle)
            self.handle = None
            _lib.check(rc)


class Registration:
    """A tensor registered with every rank (jst_comm_register)."""

    def __init__(self, comm: "Comm", tensor):
        if not tensor.is_contiguous():
            raise ValueError("register a contiguous tensor")
        h = ctypes.c_void_p()
        _lib.check(load().jst_comm_register(comm.handle, tensor.data_ptr(), tensor.numel() * tensor.element_size(),
                                            ctypes.byref(h)))
        self.handle, self.tensor = h, tensor

    def deregister(self) -> None:
        """Collective (every rank, after its last use)."""
        if self.handle:
            rc = load().jst_comm_deregister(self.handle)
            self.handle = None
            _lib.check(rc)


class Comm:
    """A rank's NCCL communicator (jst_comm) on the current CUDA device."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes, timeout_s: float = 60.0):
        if len(unique_id) != ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        handle = ctypes.c_void_p()
        _lib.check(load().jst_comm_init(ctypes.byref(handle), nranks, rank, unique_id, float(timeout_s)))
        self.handle = handle
        self.nranks, self.rank = nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(ID_BYTES)
        _lib.check(load().jst_comm_get_unique_id(buf))
        return buf.raw

    @classmethod
    def from_process_group(cls, timeout_s: float = 60.0) -> "Comm":
        """Create the communicator of every rank of torch.distributed's default group."""
        import torch.distributed as dist

        rank, world = dist.get_rank(), dist.get_world_size()
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        return cls(world, rank, obj[0], timeout_s)

    def register(self, tensor) -> "Registration":
        """Collective: register a contiguous CUDA tensor with every rank so a
        row-sharded GEMM into it delivers blocks by copy engine."""
        return Registration(self, tensor)

    def symm_alloc(self, nbytes: int) -> SymmBuffer:
        """Collective: a multicast-backed buffer of nbytes on every rank."""
        return SymmBuffer(self, nbytes)

    def sync(self, stream) -> None:
        """Host wait for `stream`, bounded by the communicator deadline."""
        _lib.check(load().jst_comm_sync(self.handle, stream.cuda_stream))

    def trace(self, on: bool = True) -> None:
        """Record a timeline of the next row-sharded calls (see trace_read)."""
        _lib.check(load().jst_comm_trace(self.handle, 1 if on else 0))

    def trace_read(self) -> list[tuple[str, float]]:
        """(label, ms since the call's entry) of the last traced row-sharded call."""
        labels = ctypes.create_string_buffer(32 * 256)
        ms = (ctypes.c_double * 256)()
        n = load().jst_comm_trace_read(self.handle, labels, ms, 256)
        if n < 0:
            _lib.check(-n)
        return [(labels.raw[32 * i:32 * i + 32].split(b"\0")[0].decode(), float(ms[i])) for i in range(n)]

    def destroy(self) -> None:
        if self.handle:
            rc = load().jst_comm_destroy(self.handle)
            self.handle = None
            _lib.check(rc)

    def gemm_rowsharded(self, a_local, b, c_full, chunk_rows: int, root: int = 0, stream=None) -> None:
        """C_full = A . B with A block-cyclically row-sharded (see row_plan); b is
        broadcast in place from `root`.  Device tensors: a_local [M_local, K],
        b [K, N], c_full [M_local * nranks, N], all contiguous fp32."""
        import torch

        for t in (a_local, b, c_full):
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
                raise ValueError("operands must be contiguous float32 CUDA tensors")
        m_local, k = a_local.shape
        n = b.shape[1]
        if b.shape[0] != k or tuple(c_full.shape) != (m_local * self.nranks, n):
            raise ValueError("shape mismatch")
        st = stream if stream is not None else torch.cuda.current_stream()
        _lib.check(load().jst_gemm_rowsharded(self.handle, a_local.data_ptr(), m_local, k, b.data_ptr(), n, root,
                                              c_full.data_ptr(), chunk_rows, st.cuda_stream))

    def bmm_batchsharded(self, a_local, b_local, c_full, stream=None) -> None:
        """c_full[rank*bl:(rank+1)*bl] = a_local . b_local, then all-gathered in place."""
        import torch

        bl, m, k = a_local.shape
        n = b_local.shape[2]
        if b_local.shape[:2] != (bl, k) or tuple(c_full.shape) != (bl * self.nranks, m, n):
            raise ValueError("shape mismatch")
        st = stream if stream is not None else torch.cuda.current_stream()
        _lib.check(load().jst_bmm_batchsharded(self.handle, a_local.data_ptr(), b_local.data_ptr(), bl, m, k, n,
                                               c_full.data_ptr(), st.cuda_stream))
