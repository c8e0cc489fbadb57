"""The multi-GPU decode-attention step with its all-gather fused into the attention kernel.

KV-head sharding (kernel_optim_b200/shard.py) leaves rank r with the attention output of its
query heads only; o_proj needs every head. Instead of a separate NCCL all-gather after attention,
``PeerGather`` lets the attention kernel itself write each finished output row into every rank's
gathered buffer over NVLink (CUDA IPC mappings of the peers' buffers, plain stores), at rank r's
columns [r*nq_l*128, (r+1)*nq_l*128), so the buffer is [B, nq*128] in head order and feeds o_proj
as is. The last CTA of rank r raises flag[r] = epoch + 1 in every rank's flag array, then waits
(bounded at 1 s; KOPT_DEV_ERR_TIMEOUT in the attention's error word on expiry) until all ranks'
flags for this call are up in its own array and advances the epoch, so the call's completion on its
stream means the whole gathered block is in local memory; o_proj follows in stream order.

Buffer reuse: a rank may start the next call while a slower peer still reads the previous call's
rows, so calls rotate over buffer slots. Writing call c+2 into a slot happens after this rank's call
c+1 completed, which needs every peer's call c+1 to have started, which those peers launch after
their o_proj of call c, so two slots suffice. Eager calls alternate through ``next_slot``; a CUDA
graph replays the same slot sequence every time, so ``slot_of`` gives its last call a third slot
when the count is odd.

Every rank must make the same calls in the same order (warm-up included): the flags count calls,
and a rank that skips one makes the others' next call run out of its wait with the error bit set
(no hang).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import Gather, KoptError, check
from .fused import _ptr, _require_cuda, _stream

_FLAGS_BYTES = 256        # flags[world] int32, written by the peers
_LOCAL_BYTES = 256        # epoch int32 (this rank only)
SLOTS = 3


class _DeviceArray:
    """A raw device allocation exposed through __cuda_array_interface__ (zero copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def _view(ptr: int, shape, dtype, device) -> torch.Tensor:
    if dtype == torch.bfloat16:
        return torch.as_tensor(_DeviceArray(ptr, shape, "<i2"), device=device).view(torch.bfloat16)
    return torch.as_tensor(_DeviceArray(ptr, shape, "<i4"), device=device)


def slot_of(call: int, calls_per_replay: int) -> int:
    """Slot of the call-th call (0-based) of a sequence replayed as a whole (a CUDA graph):
    alternates 0/1 and gives the last call slot 2 when the count is odd, so two uses of one slot
    are always at least two calls apart, also across replays."""
    if calls_per_replay % 2 and calls_per_replay > 1 and call == calls_per_replay - 1:
        return 2
    return call % 2


class PeerGather:
    """Per-rank state of the fused attention + all-gather: every rank's gathered buffers (this
    rank's local, the peers' mapped over NVLink), the flag arrays and this rank's epoch.

    B rows of row_elems = nq * 128 bf16 per slot. Collective: every rank of `group` constructs it
    (all_gather_object of the IPC handles) and later calls ``close`` together.
    """

    def __init__(self, B: int, row_elems: int, device, group=None):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise KoptError("PeerGather needs a CUDA device (no CPU path)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if not 1 <= self.world <= _lib.MAX_RANKS:
            raise KoptError(f"the fused gather supports 1..{_lib.MAX_RANKS} ranks, not {self.world}")
        if row_elems % (8 * self.world):
            raise KoptError("row_elems must split into 16-byte aligned rank columns")
        self.B, self.row_elems = B, row_elems
        self.slot_bytes = (B * row_elems * 2 + 255) // 256 * 256
        total = _FLAGS_BYTES + _LOCAL_BYTES + SLOTS * self.slot_bytes
        L = _lib.lib()
        dev = self.device.index
        base = ctypes.c_void_p()
        check(L.kopt_ipc_alloc(dev, total, ctypes.byref(base)), "kopt_ipc_alloc")
        self._base = base.value
        self._peers: list[int] = []
        try:
            handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            check(L.kopt_ipc_get_handle(ctypes.c_void_p(self._base), handle), "kopt_ipc_get_handle")
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
            bases = []
            for w, h in enumerate(handles):
                if w == self.rank:
                    bases.append(self._base)
                    continue
                peer = ctypes.c_void_p()
                buf = ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES)
                check(L.kopt_ipc_open(dev, buf, ctypes.byref(peer)), "kopt_ipc_open")
                self._peers.append(peer.value)
                bases.append(peer.value)
        except Exception:
            self._free_local()
            raise
        self._next = 0
        local = self._base + _FLAGS_BYTES
        self.epoch = _view(local, (1,), torch.int32, self.device)
        self.flags = _view(self._base, (self.world,), torch.int32, self.device)
        self.out = [_view(self._slot_ptr(self._base, s), (B, row_elems), torch.bfloat16, self.device)
                    for s in range(SLOTS)]
        self._desc = []
        for s in range(SLOTS):
            g = Gather()
            for w in range(self.world):
                g.out[w] = self._slot_ptr(bases[w], s)
                g.flags[w] = bases[w]
            g.epoch = local
            g.rank, g.world, g.row_elems = self.rank, self.world, row_elems
            self._desc.append(g)
        # every rank's buffers are mapped and zeroed before anyone writes into them
        dist.barrier(group=group)

    def _slot_ptr(self, base: int, s: int) -> int:
        return base + _FLAGS_BYTES + _LOCAL_BYTES + s * self.slot_bytes

    def descriptor(self, slot: int) -> Gather:
        return self._desc[slot]

    def next_slot(self) -> int:
        """Slot for the next eager call: alternates 0/1 over every eager call made through this
        object (a CUDA graph bakes in ``slot_of`` per captured call instead)."""
        s = self._next
        self._next ^= 1
        return s

    def attend(self, attn, qkv, q_norm_w, k_norm_w, cos, sin, cache, layer, pos, slot: int,
               q_out=None) -> torch.Tensor:
        """One fused step of ``attn`` (a PagedDecodeAttention for this rank's heads) whose output
        lands in slot `slot` of every rank. Returns this rank's gathered [B, nq*128] rows of that
        slot, complete once the call has completed on the current stream. Wait timeouts show in
        ``attn.read_error()``."""
        for t, n in ((qkv, "qkv"), (q_norm_w, "q_norm_w"), (k_norm_w, "k_norm_w"), (cos, "cos"),
                     (sin, "sin")):
            _require_cuda(t, n)
        _require_cuda(pos, "pos", torch.int32)
        if attn.B != self.B or attn.nq * attn.d * self.world != self.row_elems:
            raise KoptError("the attention shape does not match the gather buffers")
        if qkv.shape != (attn.B, (attn.nq + 2 * attn.nkv) * attn.d):
            raise KoptError("qkv must be [B, (nq+2nkv)d]")
        stream = _stream(qkv.device)
        check(_lib.lib().kopt_decode_attn_fused_gather(
            ctypes.byref(attn.plan), _ptr(qkv), _ptr(q_norm_w), _ptr(k_norm_w), _ptr(cos),
            _ptr(sin), cos.shape[0], ctypes.byref(attn._cache(cache, layer)), _ptr(pos),
            ctypes.byref(self._desc[slot]), _ptr(q_out), _ptr(attn.ws),
            ctypes.c_float(attn.scale), ctypes.c_float(attn.eps), stream),
            "kopt_decode_attn_fused_gather")
        return self.out[slot]

    def _free_local(self):
        L = _lib.lib()
        for p in self._peers:
            L.kopt_ipc_close(self.device.index, ctypes.c_void_p(p))
        self._peers = []
        if self._base:
            L.kopt_ipc_free(self.device.index, ctypes.c_void_p(self._base))
            self._base = 0

    def close(self) -> None:
        """Collective: unmap the peers' buffers, then free this rank's once no peer maps it."""
        if not self._base:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.out, self.flags, self.epoch = [], None, None
        L = _lib.lib()
        for p in self._peers:
            L.kopt_ipc_close(self.device.index, ctypes.c_void_p(p))
        self._peers = []
        dist.barrier(group=self.group)
        L.kopt_ipc_free(self.device.index, ctypes.c_void_p(self._base))
        self._base = 0
