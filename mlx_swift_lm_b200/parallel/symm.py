"""Symmetric memory communicator for the fused tensor-parallel kernels.

Each rank allocates one buffer of identical size (``b200_symm_alloc``), the
CUDA IPC handles are exchanged over the process group, and every rank maps
its peers' buffers (``b200_symm_open``). The resulting pointer table, region
offsets and per-rank counters are packed into a ``CommCtx`` blob (layout of
csrc/include/b200_comm.cuh) that the kernels receive by value.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from ..ops import _lib

MAX_RANKS = 8
NUM_PADS = 8
PHASES_PER_STEP = 1024

_lib.register_signatures({
    "b200_symm_alloc": (_lib.i32, [_lib.sz, C.POINTER(C.c_void_p), C.c_void_p]),
    "b200_symm_open": (_lib.i32, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "b200_symm_close": (_lib.i32, [C.c_void_p]),
    "b200_symm_free": (_lib.i32, [C.c_void_p]),
    "b200_ipc_handle_size": (_lib.i32, []),
    "b200_comm_ctx_size": (_lib.i32, []),
    "b200_comm_signal_roundtrip": (_lib.i32, [C.c_void_p, _lib.i32, C.c_void_p, C.c_void_p]),
    "b200_gemm_bf16_ag": (_lib.i32, [C.c_void_p, _lib.i32, _lib.i32, _lib.i32, _lib.i32, C.c_void_p, _lib.i32,
                                     _lib.i32, C.c_void_p, _lib.i32, C.c_void_p, _lib.i32, _lib.i32, _lib.i32,
                                     C.c_void_p]),
    "b200_gemm_bf16_rs": (_lib.i32, [C.c_void_p, _lib.i32, _lib.i32, C.c_void_p, _lib.i32, _lib.i32, _lib.i32,
                                     C.c_void_p, _lib.i32, _lib.i32, C.c_void_p, _lib.i32, _lib.i32, _lib.i32,
                                     C.c_void_p, C.c_void_p]),
    "b200_tp_combine_all": (_lib.i32, [C.c_void_p, _lib.i32, _lib.i32, C.c_void_p, C.c_void_p, _lib.f32, C.c_void_p,
                                       _lib.i32, _lib.i32, _lib.i32, C.c_void_p, C.c_void_p]),
    "b200_tp_combine_norm": (_lib.i32, [C.c_void_p, _lib.i32, _lib.i32, _lib.i32, _lib.i32, C.c_void_p, C.c_void_p,
                                        _lib.f32, _lib.i32, C.c_void_p]),
    "b200_tp_embed": (_lib.i32, [C.c_void_p, C.c_void_p, _lib.i32, C.c_void_p, _lib.i64, C.c_void_p, _lib.f32,
                                 C.c_void_p]),
    "b200_tp_argmax": (_lib.i32, [C.c_void_p, _lib.i32, _lib.i32, C.c_void_p, _lib.i64, _lib.i32, _lib.i32, _lib.i32,
                                  C.c_void_p, C.c_void_p, C.c_void_p]),
}, status_tags=("symm", "tp_fused"))


class CommCtxStruct(C.Structure):
    _fields_ = [("rank", C.c_int), ("world", C.c_int), ("base", C.c_void_p * MAX_RANKS),
                ("pads_off", C.c_uint64), ("recv_off", C.c_uint64), ("h_off", C.c_uint64), ("xarg_off", C.c_uint64),
                ("rows_per_rank", C.c_int), ("hidden", C.c_int), ("max_rows", C.c_int),
                ("step_ptr", C.c_void_p), ("expect_local", C.c_void_p), ("ticket", C.c_void_p)]


def _align(n, a=256):
    return (n + a - 1) // a * a


def open_symmetric(group, rank: int, world: int, device, nbytes: int):
    """Allocate a zeroed device buffer of `nbytes` on every rank of `group`
    and map every peer's buffer (CUDA IPC handles exchanged over the group).
    Returns (local pointer, [pointer of rank j's buffer for j in range(world)])."""
    L = _lib.lib()
    with torch.cuda.device(device):
        ptr = C.c_void_p()
        hsz = L.b200_ipc_handle_size()
        handle = (C.c_char * hsz)()
        _lib.check(L.b200_symm_alloc(nbytes, C.byref(ptr), handle), "symm_alloc")
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        peers = []
        for j, h in enumerate(handles):
            if j == rank:
                peers.append(ptr.value)
                continue
            pp = C.c_void_p()
            hb = (C.c_char * hsz).from_buffer_copy(h)
            _lib.check(L.b200_symm_open(hb, C.byref(pp)), f"symm_open peer {j}")
            peers.append(pp.value)
    return ptr.value, peers


def close_symmetric(rank: int, local_ptr, peer_ptrs):
    L = _lib.lib()
    for j, p in enumerate(peer_ptrs):
        if j != rank and p:
            L.b200_symm_close(p)
    if local_ptr:
        L.b200_symm_free(local_ptr)


class SymmetricComm:
    """Symmetric buffer + signal pads for one tensor-parallel group."""

    def __init__(self, group, rank: int, world: int, device, hidden: int, rows_per_rank: int, max_rows: int = 256):
        assert world <= MAX_RANKS
        assert rows_per_rank % 8 == 0, "rows per rank must be a multiple of 8 (TMA swizzle atoms)"
        self.group, self.rank, self.world = group, rank, world
        self.device = torch.device(device)
        self.hidden, self.rpr, self.max_rows = hidden, rows_per_rank, max_rows
        L = _lib.lib()
        assert L.b200_comm_ctx_size() == C.sizeof(CommCtxStruct), "CommCtx layout mismatch"
        pads = NUM_PADS * MAX_RANKS * 4
        # fp32 partial rows: [2][world (source)][world * rows_per_rank][hidden] (every rank's
        # partials of every row; the owner-only layout uses the first rows_per_rank rows)
        recv = 2 * world * world * rows_per_rank * hidden * 4
        hbuf = 2 * world * rows_per_rank * hidden * 2
        xarg = 2 * world * max_rows * 8
        self.pads_off = 0
        self.recv_off = _align(pads)
        self.h_off = _align(self.recv_off + recv)
        self.xarg_off = _align(self.h_off + hbuf)
        self.nbytes = _align(self.xarg_off + xarg)
        self.local_ptr, self.peer_ptrs = open_symmetric(group, rank, world, self.device, self.nbytes)
        self.step = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.expect = torch.zeros(NUM_PADS * MAX_RANKS, dtype=torch.int32, device=self.device)
        self.ticket = torch.zeros(4, dtype=torch.int32, device=self.device)
        s = CommCtxStruct()
        s.rank, s.world = rank, world
        for j in range(MAX_RANKS):
            s.base[j] = self.peer_ptrs[j] if j < world else 0
        s.pads_off, s.recv_off, s.h_off, s.xarg_off = self.pads_off, self.recv_off, self.h_off, self.xarg_off
        s.rows_per_rank, s.hidden, s.max_rows = rows_per_rank, hidden, max_rows
        s.step_ptr, s.expect_local, s.ticket = self.step.data_ptr(), self.expect.data_ptr(), self.ticket.data_ptr()
        self.ctx = s
        self.ctx_ptr = C.cast(C.pointer(self.ctx), C.c_void_p)
        self.phase = 0
        self.rs_count = 0
        self.ag_count = 0
        self.arg_count = 0
        dist.barrier(group=group)

    # step / phase bookkeeping ------------------------------------------------
    def begin_step(self, step: int | None = None):
        """Advance the device step counter (outside CUDA graphs) and restart
        phases. The update is a stream-ordered device op, so a host running
        ahead of the device cannot skip or repeat an epoch."""
        if step is None:
            self.step.add_(1)
        else:
            self.step.fill_(step)
        self.phase = 0

    def next_phase(self) -> int:
        p = self.phase
        self.phase += 1
        assert self.phase < PHASES_PER_STEP
        return p

    def self_test(self) -> bool:
        """Bounded signal round trip between all ranks."""
        L = _lib.lib()
        st = torch.zeros(1, dtype=torch.int32, device=self.device)
        _lib.check(L.b200_comm_signal_roundtrip(self.ctx_ptr, 7, st.data_ptr(), _lib.stream_ptr(self.device)),
                   "signal_roundtrip")
        torch.cuda.synchronize(self.device)
        return bool(st.item())

    def close(self):
        close_symmetric(self.rank, self.local_ptr, self.peer_ptrs)
        self.peer_ptrs, self.local_ptr = [], None
