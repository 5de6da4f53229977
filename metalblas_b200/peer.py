"""Peer (NVLink) buffers for the fused product-and-gather, one process per GPU.

The reference is single-device.  Its sharded form here (``shard.py``) splits a
large GEMM along N, or a bmm along the batch, and gathers the output over
NVLink.  The gather is not a separate collective: the tcgen05 kernel's
epilogue stores every finished tile into this GPU's C and, with plain 16-byte
``st.global`` over NVLink, into every other GPU's copy of C at the same offset
(``mb_gemm_peer`` in include/metalblas_b200.h).  This module provides the
memory for that: a :class:`PeerBuffer` is one device buffer per rank, mapped
into every other rank's address space with CUDA IPC (``mb_ipc_get_handle`` /
``mb_ipc_open``), and a stream-ordered :func:`barrier` after which every rank's
peer stores of the step have landed.

Where every rank's GPU supports NVSwitch multicast, the buffer is instead
torch's symmetric memory bound to one multicast object (``multicast_ptr``):
the kernel then writes each finished tile once through the multicast address
(``multimem.st``) and the switch replicates it to every GPU, so each GPU sends
its output once instead of once per peer.  That is the default from four
ranks on (``MULTICAST_MIN_WORLD``); ``METALBLAS_NVLS=1`` forces it at any size
and ``METALBLAS_NVLS=0`` keeps the plain CUDA-IPC peer mappings.  A rank that
dies while its memory is bound to a multicast object can fault the other
ranks' GPUs, so the owners release the buffers (:func:`release_arenas`) before
leaving the process group, on error paths too.

Reuse rule: a step writes into every rank's buffer, so a step must not start
writing a slot that a peer may still be reading.  :class:`PeerBuffer` keeps two
slots and callers alternate them (:meth:`PeerBuffer.next_slot`): the barrier
that ends step i on every rank orders all ranks' work queued before step i
(on the same stream) ahead of step i + 1, so step i + 1 may overwrite the slot
of step i - 1.  A result is therefore valid until two sharded calls later on
the same buffer.
"""
from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from . import _lib

HANDLE_BYTES = 64
_PAYLOAD = HANDLE_BYTES + 8   # handle + int64 byte offset of the buffer in its allocation
SLOT_ALIGN = 4096


def world_of(group=None) -> tuple[int, int]:
    """(world size, rank); a process without a process group is world 1."""
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _comm_device(group, device):
    """Where a collective's tensors must live for this group's backend."""
    try:
        backend = dist.get_backend(group)
    except (RuntimeError, ValueError):
        backend = "gloo"
    return device if str(backend).lower() == "nccl" else torch.device("cpu")


def slot_bytes(nbytes: int) -> int:
    """Bytes one slot occupies (rounded so every slot starts 4 KiB-aligned)."""
    return (int(nbytes) + SLOT_ALIGN - 1) // SLOT_ALIGN * SLOT_ALIGN


def pack_payload(handle: bytes, offset: int) -> torch.Tensor:
    """One rank's exchange record: the IPC handle bytes and its int64 offset."""
    if len(handle) != HANDLE_BYTES:
        raise ValueError(f"IPC handle must be {HANDLE_BYTES} bytes")
    raw = bytes(handle) + int(offset).to_bytes(8, "little", signed=True)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).clone()


def unpack_payload(t: torch.Tensor) -> tuple[bytes, int]:
    raw = bytes(t.cpu().numpy().tobytes())
    return raw[:HANDLE_BYTES], int.from_bytes(raw[HANDLE_BYTES:_PAYLOAD], "little", signed=True)


def exchange(payload: torch.Tensor, group, device) -> list[torch.Tensor]:
    """All ranks' payloads (rank order), through one all-gather."""
    world, _ = world_of(group)
    dev = _comm_device(group, device)
    src = payload.to(dev)
    out = torch.empty(world * _PAYLOAD, dtype=torch.uint8, device=dev)
    dist.all_gather_into_tensor(out, src, group=group)
    out = out.cpu()
    return [out[r * _PAYLOAD:(r + 1) * _PAYLOAD] for r in range(world)]


# Smallest world that takes the multicast buffer by default.  A multimem store
# reaches every member, the writer's own GPU included, so each GPU receives
# the whole output (N/N) instead of the peers' share ((N-1)/N): at two GPUs that
# doubles the inbound bytes for no saving, while from four GPUs on each GPU
# sends its share once instead of N-1 times.
MULTICAST_MIN_WORLD = 4


def _multicast_wanted(world: int) -> bool:
    """METALBLAS_NVLS=1 forces the multicast buffer, 0 disables it; unset, it
    is used from MULTICAST_MIN_WORLD ranks on."""
    v = os.environ.get("METALBLAS_NVLS", "")
    if v in ("0", "1"):
        return v == "1"
    return world >= MULTICAST_MIN_WORLD


def _agree_all(flag: bool, group, device) -> bool:
    """True when `flag` holds on every rank (one MIN all-reduce)."""
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=_comm_device(group, device))
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(int(t.item()))


def _multicast_supported(device) -> bool:
    try:
        S = torch._C._distributed_c10d._SymmetricMemory
        return bool(S.has_multicast_support(torch._C._autograd.DeviceType.CUDA, torch.device(device).index))
    except (AttributeError, RuntimeError, TypeError):
        return False


class PeerBuffer:
    """One device buffer of ``nslots`` slots of ``nbytes`` per rank, with every
    other rank's buffer mapped into this process.

    ``addr(slot, rank)`` is the device address, valid in this process, of
    ``rank``'s slot; ``view(slot, dtype, shape)`` is this rank's slot as a tensor.
    Collective: every rank of ``group`` constructs it with the same sizes, in
    the same order relative to other collectives."""

    def __init__(self, nbytes: int, device: torch.device, group=None, nslots: int = 2):
        if not torch.cuda.is_available():
            raise RuntimeError("PeerBuffer needs CUDA devices (one process per GPU)")
        self.group = group
        self.world, self.rank = world_of(group)
        self.device = torch.device(device)
        self.slot = slot_bytes(nbytes)
        self.nslots = int(nslots)
        self._turn = 0
        self._bases: list[int] = []
        self._base_addr = [0] * self.world
        self._symm = None
        self.mc_base = 0   # multicast address of this buffer's first byte, 0 without one
        if self.world > 1 and _multicast_wanted(self.world) and self.world - 1 <= _lib.MB_MAX_PEERS:
            # every rank must take the same branch: symmetric memory is collective
            if _agree_all(_multicast_supported(self.device), group, self.device):
                self._init_multicast(group)
        if self._symm is not None:
            return
        self.local = torch.empty(self.slot * self.nslots, dtype=torch.uint8, device=self.device)
        self._base_addr[self.rank] = self.local.data_ptr()
        if self.world > 1:
            lib = _lib.load()
            handle = (ctypes.c_ubyte * HANDLE_BYTES)()
            off = ctypes.c_int64()
            with torch.cuda.device(self.device):
                _lib.raise_for(lib.mb_ipc_get_handle(ctypes.c_void_p(self.local.data_ptr()), handle,
                                                     ctypes.byref(off)), "mb_ipc_get_handle")
            recs = exchange(pack_payload(bytes(handle), off.value), group, self.device)
            with torch.cuda.device(self.device):
                for r, rec in enumerate(recs):
                    if r == self.rank:
                        continue
                    h, o = unpack_payload(rec)
                    base = ctypes.c_void_p()
                    hbuf = (ctypes.c_ubyte * HANDLE_BYTES).from_buffer_copy(h)
                    _lib.raise_for(lib.mb_ipc_open(hbuf, ctypes.byref(base)), "mb_ipc_open")
                    self._bases.append(base.value)
                    self._base_addr[r] = base.value + o

    def _init_multicast(self, group) -> None:
        """Symmetric memory bound to a multicast object, or nothing (the
        caller then maps plain IPC buffers).  Each step that can fail on one
        rank alone is followed by an agreement, so every rank takes the same
        branch and no rank waits in a collective the others have left."""
        import torch.distributed._symmetric_memory as symm_mem
        try:
            t = symm_mem.empty(self.slot * self.nslots, dtype=torch.uint8, device=self.device)
        except (RuntimeError, ValueError):
            t = None
        if not _agree_all(t is not None, group, self.device):
            return
        try:
            hdl = symm_mem.rendezvous(t, group if group is not None else dist.group.WORLD)
            ptrs = [int(q) for q in hdl.buffer_ptrs]
            off = t.data_ptr() - ptrs[self.rank]
            mc = int(hdl.multicast_ptr)
            ok = mc != 0 and off % 16 == 0
        except (RuntimeError, ValueError):
            ok = False
        if not _agree_all(ok, group, self.device):
            return   # plain IPC mappings instead (every rank agrees)
        self.local, self._symm = t, hdl
        self._base_addr = [q + off for q in ptrs]
        self.mc_base = mc + off

    def mc_addr(self, slot: int, byte_offset: int = 0) -> int:
        """Multicast address of this rank's slot (+ byte_offset), or 0."""
        return self.mc_base + slot * self.slot + byte_offset if self.mc_base else 0

    def next_slot(self) -> int:
        """The slot the next step should write (alternates)."""
        s = self._turn
        self._turn = (self._turn + 1) % self.nslots
        return s

    def addr(self, slot: int, rank: int) -> int:
        return self._base_addr[rank] + slot * self.slot

    def peer_addrs(self, slot: int, byte_offset: int = 0) -> list[int]:
        """Addresses of every other rank's slot (+ byte_offset), in rank order."""
        return [self.addr(slot, r) + byte_offset for r in range(self.world) if r != self.rank]

    def view(self, slot: int, dtype: torch.dtype, shape) -> torch.Tensor:
        n = 1
        for s in shape:
            n *= int(s)
        esz = torch.empty((), dtype=dtype).element_size()
        if n * esz > self.slot:
            raise ValueError(f"view of {n * esz} bytes exceeds the {self.slot}-byte slot")
        return self.local[slot * self.slot: slot * self.slot + n * esz].view(dtype).view(*shape)

    def close(self) -> None:
        """Unmap the peers' buffers, or release the multicast-bound symmetric
        memory (callers barrier first so no rank still writes into a buffer
        whose owner frees it afterwards)."""
        if self._symm is not None:
            torch.cuda.synchronize(self.device)
            self._symm = None
            self.local = None
            self.mc_base = 0
            return
        if not self._bases:
            return
        lib = _lib.load()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for b in self._bases:
                lib.mb_ipc_close(ctypes.c_void_p(b))
        self._bases = []


_ARENAS: dict = {}


def arena(nbytes: int, device: torch.device, group=None) -> PeerBuffer:
    """The shared two-slot peer buffer of (group, device), grown to at least
    ``nbytes`` per slot.  Growing is collective: all ranks make the same calls
    in the same order, as they do for the sharded products that use it."""
    key = (id(group), torch.device(device).index)
    buf = _ARENAS.get(key)
    if buf is None or buf.slot < nbytes:
        if buf is not None:
            barrier(group, device)
            buf.close()
        buf = PeerBuffer(nbytes, device, group)
        _ARENAS[key] = buf
    return buf


def release_arenas() -> None:
    """Unmap and drop every arena (before destroying the process group)."""
    for buf in _ARENAS.values():
        buf.close()
    _ARENAS.clear()


_FLAGS: dict = {}


def barrier(group=None, device=None) -> None:
    """Stream-ordered barrier: a one-word all-reduce on the current stream.  When
    it completes on a rank, every rank's work queued before it (its peer stores
    included: each kernel's writes are performed before the kernel retires) has
    finished."""
    world, _ = world_of(group)
    if world <= 1:
        return
    dev = _comm_device(group, device if device is not None else torch.device("cuda", torch.cuda.current_device()))
    key = (id(group), str(dev))
    flag = _FLAGS.get(key)
    if flag is None:
        flag = _FLAGS[key] = torch.zeros(1, dtype=torch.int32, device=dev)
    dist.all_reduce(flag, group=group)
