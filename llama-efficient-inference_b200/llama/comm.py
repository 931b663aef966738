"""Tensor-parallel all-reduce + residual add over NVLink peer memory (li4_allreduce_add).

Replaces, for the decode step's small row-parallel outputs, the NCCL all-reduce
after wo / w2 and the residual add that follows it (the reference's
TransformerBlock.forward, llama/model.py:358-362, under tensor parallelism).
Each rank allocates one buffer with the kernel library (two partial slots and
a flag array), exports it with a CUDA IPC handle, gathers the other ranks'
handles through the process group, and maps their buffers.  A row-parallel
GEMV writes its fp16 partial straight into this rank's slot (`slot_ptr`), then
`all_reduce_add` sums the slots of all ranks over NVLink and adds the residual
in one launch.  Calls alternate the two slots; every rank must make the same
sequence of calls.

The same buffer also holds two receive buffers for the fused form
(`push_fusion`): the row-parallel GEMV itself stores its fp16 partial, as
8-byte words that carry the call's epoch, into every peer's receive buffer
and finishes the sum and the residual in its own launch
(LI4_EPI_ALLREDUCE_RESIDUAL), with no separate all-reduce kernel.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _native as native

_ALIGN = 256


def _round_up(v: int, a: int = _ALIGN) -> int:
    return (v + a - 1) // a * a


class NvlinkAllReduce:
    """One communication buffer per rank of `group`, mapped by every other rank."""

    def __init__(self, group, max_elems: int, device: torch.device, ctas: int = 16, key_rows: int = 64):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= 8:
            raise ValueError(f"NvlinkAllReduce takes 1..8 ranks, got {self.world}")
        self.device, self.ctas, self.max_elems = device, ctas, max_elems
        lib = native.lib()
        self.slot_bytes = _round_up(2 * max_elems)
        self.flag_bytes = _round_up(4 * ctas * self.world)
        # fused form: per receive buffer, every rank's words [world][max_elems / 2] of 8 bytes
        self.recv_bytes = _round_up(self.world * ((max_elems + 1) // 2) * 8)
        # greedy step (argmax_allreduce): every rank's key words [2][world][key_rows][2] of 8 bytes
        self.key_rows = key_rows
        self.key_bytes = _round_up(2 * self.world * key_rows * 2 * 8)
        total = 2 * self.slot_bytes + self.flag_bytes + 2 * self.recv_bytes + self.key_bytes
        with torch.cuda.device(device):
            base = ctypes.c_void_p()
            native.check(lib.li4_comm_alloc(total, ctypes.byref(base)), "comm_alloc")
            self._own = base.value
            handle = (ctypes.c_char * 64)()
            native.check(lib.li4_ipc_get_handle(base, ctypes.cast(handle, ctypes.c_void_p)), "ipc_get_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases, self._opened = [], []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                ptr = ctypes.c_void_p()
                buf = (ctypes.c_char * 64).from_buffer_copy(h)
                native.check(lib.li4_ipc_open_handle(ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(ptr)),
                             "ipc_open_handle")
                bases.append(ptr.value)
                self._opened.append(ptr.value)
        arr = ctypes.c_void_p * self.world
        self._slots = [arr(*[b + s * self.slot_bytes for b in bases]) for s in (0, 1)]
        self._flags = arr(*[b + 2 * self.slot_bytes for b in bases])
        self.counts = torch.zeros(ctas, dtype=torch.int32, device=device)
        recv0 = 2 * self.slot_bytes + self.flag_bytes
        self._recv = [arr(*[b + recv0 + s * self.recv_bytes for b in bases]) for s in (0, 1)]
        # per receive buffer, this rank's call count of every 16-row output tile
        self.epochs = torch.zeros(2, (max_elems + 15) // 16, dtype=torch.int32, device=device)
        self._keys = arr(*[b + recv0 + 2 * self.recv_bytes for b in bases])
        self.key_epochs = torch.zeros(key_rows, dtype=torch.int32, device=device)

    def slot_ptr(self, slot: int) -> int:
        """Device address of this rank's partial slot `slot` (0 or 1), fp16, max_elems values."""
        return self._own + slot * self.slot_bytes

    def all_reduce_add(self, slot: int, residual: torch.Tensor, out: torch.Tensor) -> None:
        """out = fp16(residual + sum over ranks of slot `slot`) on the current stream."""
        n = residual.numel()
        if n > self.max_elems or out.numel() != n or not (residual.is_contiguous() and out.is_contiguous()):
            raise RuntimeError(f"all_reduce_add: {n} contiguous values (at most {self.max_elems})")
        rc = native.lib().li4_allreduce_add(self._slots[slot], self._flags, self.counts.data_ptr(), self.ctas,
                                           self.world, self.rank, n, residual.data_ptr(), out.data_ptr(),
                                           native.stream_ptr(out.device))
        native.check(rc, "allreduce_add")

    def push_fusion(self, slot: int, residual: torch.Tensor) -> native.Fusion:
        """The li4_fusion of a row-parallel GEMV that finishes its own all-reduce + residual add
        (LI4_EPI_ALLREDUCE_RESIDUAL) through receive buffer `slot` (0 or 1): y = fp16(residual +
        fp16(sum over ranks of their fp16 partials)), the same values as all_reduce_add."""
        if residual.numel() > self.max_elems or residual.stride(-1) != 1:
            raise RuntimeError(f"push_fusion: a row-major residual of at most {self.max_elems} values")
        return native.Fusion(epilogue=native.LI4_EPI_ALLREDUCE_RESIDUAL, residual=residual.data_ptr(),
                             stride_rm=residual.stride(0), ar_recv=ctypes.cast(self._recv[slot], ctypes.c_void_p),
                             ar_recv_bytes=self.recv_bytes, ar_epochs=self.epochs[slot].data_ptr(),
                             ar_world=self.world, ar_rank=self.rank)

    def argmax_allreduce(self, logits: torch.Tensor, index_offset: int, out: torch.Tensor) -> None:
        """out[r] = torch.argmax of row r of the full logits, of which this rank holds the columns
        index_offset .. index_offset + logits.shape[1] - 1 (li4_argmax_rows_allreduce: each rank's key
        goes to every rank over NVLink, no NCCL).  fp16 / fp32 logits with contiguous rows."""
        codes = {torch.float16: native.LI4_F16, torch.float32: native.LI4_F32}
        rows, cols = logits.shape
        if logits.dtype not in codes or logits.stride(-1) != 1 or out.dtype != torch.long or rows > self.key_rows:
            raise RuntimeError(f"argmax_allreduce: fp16 / fp32 logits of at most {self.key_rows} contiguous rows, "
                               "an int64 output")
        rc = native.lib().li4_argmax_rows_allreduce(
            logits.data_ptr(), codes[logits.dtype], rows, cols, logits.stride(0), index_offset,
            ctypes.cast(self._keys, ctypes.c_void_p), self.key_bytes, self.key_epochs.data_ptr(), self.world,
            self.rank, out.data_ptr(), out.stride(0), native.stream_ptr(logits.device))
        native.check(rc, "argmax_rows_allreduce")

    def close(self) -> None:
        lib = native.lib()
        for p in self._opened:
            lib.li4_ipc_close(p)
        self._opened = []
        if self._own:
            lib.li4_comm_free(self._own)
            self._own = None
