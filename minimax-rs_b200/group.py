"""Multi-GPU groups for the MoE block: tensor parallel (TP = 2, the reference layout) and expert
parallel (W = 4 / 8), one process per GPU or several GPUs driven from one process.

The reference's TP rank group (src/tensor_parallel.rs) keeps persistent peer-visible buffers,
maps them into the other rank through CUDA IPC (64-byte handles) and reduces small hidden states
with a peer kernel, larger ones with NCCL.  Here every rank allocates one exchange region
(`mmrs_xch_bytes`), the handles travel through any all-gather (torch.distributed on gloo or
NCCL), and the MoE block itself performs the reduction over NVLink (`mmrs_moe_block_forward_group`).

Shard layout (tensor_parallel_model.rs:37-61, quantized_var_builder.rs:478-560): gate / up are
split along their rows (axis 1 of [experts][inter][hidden]), down along K (axis 2 of
[experts][hidden][inter], whole 256-element super-blocks); router and bias are replicated.
Expert parallel: rank r computes the experts e with e % W == r.
"""
from __future__ import annotations

import ctypes as C
from typing import Callable, Sequence

from . import MmrsPeerGroup, MoeError, check, lib, row_bytes

HANDLE_BYTES = 64


# --------------------------------------------------------------------------------------------
# Shard arithmetic (pure, CPU-testable)
# --------------------------------------------------------------------------------------------
def tp_rows(inter: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [r0, r1) of gate/up held by `rank`; the same range is the rank's down K range."""
    if inter % (256 * world):
        raise ValueError(f"inter {inter} does not split into whole super-blocks over {world} ranks")
    per = inter // world
    return rank * per, (rank + 1) * per


def tp_shard_gate_up(t, experts: int, inter: int, hidden: int, gguf_type: int, world: int, rank: int):
    """[experts][inter][hidden] GGUF bytes -> the rank's [experts][inter / world][hidden]."""
    r0, r1 = tp_rows(inter, world, rank)
    return t.reshape(experts, inter, row_bytes(gguf_type, hidden))[:, r0:r1].contiguous()


def tp_shard_down(t, experts: int, hidden: int, inter: int, gguf_type: int, world: int, rank: int):
    """[experts][hidden][inter] GGUF bytes -> the rank's K range [experts][hidden][inter / world]."""
    r0, r1 = tp_rows(inter, world, rank)
    bb = row_bytes(gguf_type, 256)
    return t.reshape(experts, hidden, inter // 256, bb)[:, :, r0 // 256:r1 // 256].contiguous()


def ep_owner(expert: int, world: int) -> int:
    return expert % world


def ep_local_experts(num_experts: int, world: int, rank: int) -> list[int]:
    return [e for e in range(num_experts) if e % world == rank]


class TokenCounter:
    """Monotonic operation tokens (start at 1); every rank must draw them in the same order."""

    def __init__(self):
        self.value = 0

    def next(self) -> int:
        self.value = (self.value + 1) & 0xFFFFFFFF
        if self.value == 0:
            self.value = 1
        return self.value


# --------------------------------------------------------------------------------------------
# Exchange regions
# --------------------------------------------------------------------------------------------
def exchange_bytes(ar_capacity: int) -> int:
    return lib().mmrs_xch_bytes(ar_capacity)


class PeerGroup:
    """One rank's view of the group: its own exchange region and every rank's mapping of it.

    `allgather(obj) -> list` must return the objects of all ranks in rank order (e.g.
    torch.distributed.all_gather_object); it is called once, with the 64-byte IPC handle."""

    def __init__(self, world: int, rank: int, ar_capacity: int, expert_parallel: bool,
                 allgather: Callable[[bytes], Sequence[bytes]]):
        if not 1 <= world <= 8 or not 0 <= rank < world:
            raise ValueError("world must be 1..8 and 0 <= rank < world")
        self.world, self.rank, self.expert_parallel = world, rank, bool(expert_parallel)
        self.ar_capacity = ar_capacity
        self.tokens = TokenCounter()
        L = lib()
        self._mine = C.c_void_p()
        check(L.mmrs_peer_alloc(exchange_bytes(ar_capacity), C.byref(self._mine)), "mmrs_peer_alloc")
        handle = (C.c_uint8 * HANDLE_BYTES)()
        check(L.mmrs_ipc_handle(self._mine, handle), "mmrs_ipc_handle")
        handles = list(allgather(bytes(handle)))
        if len(handles) != world:
            raise ValueError("allgather returned the wrong number of handles")
        self._opened = []
        peers = []
        for r, h in enumerate(handles):
            if r == rank:
                peers.append(self._mine.value)
                continue
            ptr = C.c_void_p()
            buf = (C.c_uint8 * HANDLE_BYTES).from_buffer_copy(h)
            check(L.mmrs_ipc_open(buf, C.byref(ptr)), "mmrs_ipc_open")
            self._opened.append(ptr)
            peers.append(ptr.value)
        self.c = MmrsPeerGroup(world, rank, self._mine, (C.c_void_p * 8)(*(peers + [None] * (8 - world))),
                               ar_capacity, int(self.expert_parallel))

    @classmethod
    def local(cls, devices: Sequence[int], ar_capacity: int, expert_parallel: bool):
        """All ranks driven from this process, rank r on device devices[r] (peer access)."""
        import torch
        world = len(devices)
        groups = [cls.__new__(cls) for _ in devices]
        L = lib()
        mines = []
        for d in devices:
            with torch.cuda.device(d):
                for o in devices:
                    if o != d:
                        check(L.mmrs_peer_enable(o), "mmrs_peer_enable")
                ptr = C.c_void_p()
                check(L.mmrs_peer_alloc(exchange_bytes(ar_capacity), C.byref(ptr)), "mmrs_peer_alloc")
                mines.append(ptr)
        for r, g in enumerate(groups):
            g.world, g.rank, g.expert_parallel, g.ar_capacity = world, r, bool(expert_parallel), ar_capacity
            g.tokens = TokenCounter()
            g._mine, g._opened = mines[r], []
            g._device = devices[r]
            ptrs = [m.value for m in mines] + [None] * (8 - world)
            g.c = MmrsPeerGroup(world, r, mines[r], (C.c_void_p * 8)(*ptrs), ar_capacity, int(expert_parallel))
        return groups

    def status(self, stream=None) -> int:
        from . import _stream
        return lib().mmrs_peer_status(C.byref(self.c), _stream(stream))

    def forward(self, layer, x, residual=None, y=None, topk_ids=None, topk_w=None, token: int | None = None,
                stream=None):
        """y = MoE(x) (+ residual) of the whole group, on this rank (see mmrs_moe_block_forward_group)."""
        import torch
        from . import _ptr, _stream
        T = x.shape[0]
        if y is None:
            y = torch.empty_like(x)
        ws = layer.workspace(T)
        # every call draws a group token, also for T == 1: the exchange flags and buffers belong
        # to the group, and a layer-local counter would let one layer's wait pass on another's flag
        tok = token if token is not None else self.tokens.next()
        rc = lib().mmrs_moe_block_forward_group(C.byref(layer.c), C.byref(self.c), x.data_ptr(), _ptr(residual),
                                                y.data_ptr(), T, _ptr(topk_ids), _ptr(topk_w), ws.data_ptr(),
                                                ws.numel(), tok, _stream(stream))
        if rc:
            raise MoeError(rc, "mmrs_moe_block_forward_group")
        return y

    def forward_host(self, layer, x_host, y_host, x_dev, y_dev, residual=None, topk_ids=None, topk_w=None,
                     token: int | None = None, stream=None):
        """y_host = MoE(x_host) (+ residual) of the whole group in one library call
        (mmrs_moe_block_forward_group_host): x_host / y_host in pinned host memory, x_dev / y_dev
        device staging buffers of the same shape; residual / topk_* as in forward()."""
        from . import _ptr, _stream
        T = x_host.shape[0]
        ws = layer.workspace(T)
        tok = token if token is not None else self.tokens.next()
        rc = lib().mmrs_moe_block_forward_group_host(C.byref(layer.c), C.byref(self.c), x_host.data_ptr(),
                                                     _ptr(residual), y_host.data_ptr(), T, x_dev.data_ptr(),
                                                     y_dev.data_ptr(), _ptr(topk_ids), _ptr(topk_w), ws.data_ptr(),
                                                     ws.numel(), tok, _stream(stream))
        if rc:
            raise MoeError(rc, "mmrs_moe_block_forward_group_host")
        return y_host

    def all_reduce(self, partial_writer, count: int, residual=None, y=None, stream=None):
        """Writes this rank's partial through partial_writer(ptr) then reduces over the group."""
        import torch
        from . import _ptr, _stream
        tok = self.tokens.next()
        buf = lib().mmrs_xch_ar_buffer(C.byref(self.c), tok)
        partial_writer(buf)
        rc = lib().mmrs_peer_all_reduce(C.byref(self.c), _ptr(residual), y.data_ptr(), count, tok, _stream(stream))
        if rc:
            raise MoeError(rc, "mmrs_peer_all_reduce")
        return y

    def close(self):
        L = lib()
        for p in self._opened:
            L.mmrs_ipc_close(p)
        self._opened = []
        if self._mine is not None and self._mine.value:
            L.mmrs_peer_free(self._mine)
        self._mine = None
