"""Host side of the fused KV-slab exchange (include/m4b.h, m4b_exchange_*): one process per GPU.

``PeerExchange`` allocates this GPU's receive buffer, swaps CUDA IPC handles with the other
ranks over ``torch.distributed`` (set-up only; the data path uses no library collective), and
opens every peer's buffer.  Per layer the caller runs

    part = m4.kqkv_partials(kcache_slab, qcur, mask_slab, scale)   # this GPU's split records
    x.publish(part)                        # merge + store the record into every peer (NVLink)
    x.combine_wvb(w_uv, out=..., attn_out=...)   # wait for all records, merge, W_UV (one kernel)

Both calls are plain launches on the current stream and can be captured in a CUDA graph.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import m4

IPC_HANDLE_BYTES = 64

_lib = m4.lib()
_lib.m4b_exchange_create.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]
_lib.m4b_exchange_ipc_handle.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
_lib.m4b_exchange_open.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
_lib.m4b_exchange_open_local.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.c_int]
_lib.m4b_exchange_detach.argtypes = [ctypes.c_void_p]
_lib.m4b_exchange_destroy.argtypes = [ctypes.c_void_p]
_lib.m4b_exchange_publish.argtypes = [ctypes.c_void_p, ctypes.POINTER(m4.PhaseArgs), ctypes.c_void_p]
_lib.m4b_exchange_combine_wvb.argtypes = [ctypes.c_void_p, ctypes.POINTER(m4.PhaseArgs),
                                          ctypes.c_void_p]
_lib.m4b_exchange_merge_wvb.argtypes = [ctypes.c_void_p, ctypes.POINTER(m4.PhaseArgs),
                                         ctypes.c_void_p]


class PeerExchange:
    def __init__(self, world: int, rank: int, group=None):
        """Collective over ``group``: every rank constructs its exchange at the same point."""
        self.world, self.rank = world, rank
        h = ctypes.c_void_p()
        m4._check(_lib.m4b_exchange_create(world, rank, ctypes.byref(h)), "m4b_exchange_create")
        self._h = h
        mine = (ctypes.c_char * IPC_HANDLE_BYTES)()
        m4._check(_lib.m4b_exchange_ipc_handle(self._h, mine), "m4b_exchange_ipc_handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(mine), group=group)
        blob = (ctypes.c_char * (IPC_HANDLE_BYTES * world)).from_buffer_copy(b"".join(handles))
        m4._check(_lib.m4b_exchange_open(self._h, blob), "m4b_exchange_open")

    def publish(self, partials: torch.Tensor, flags: int = 0) -> None:
        a = m4.PhaseArgs()
        a.src[1] = m4.gtensor(partials, [m4.PART_STRIDE, m4.HEADS, partials.shape[0], 1])
        a.flags = flags
        m4._check(_lib.m4b_exchange_publish(self._h, ctypes.byref(a), m4._stream()),
                  "m4b_exchange_publish")

    def combine_wvb(self, w_uv: torch.Tensor, out: torch.Tensor, attn_out: torch.Tensor | None = None,
                    flags: int = 0) -> torch.Tensor:
        a = m4.PhaseArgs()
        a.src[0] = m4.gtensor(w_uv, list(reversed(w_uv.shape)))
        if attn_out is not None:
            a.src[2] = m4._heads_desc(attn_out, m4.LATENT)
        a.dst = m4._heads_desc(out, m4.VHEAD)
        a.flags = flags
        m4._check(_lib.m4b_exchange_combine_wvb(self._h, ctypes.byref(a), m4._stream()),
                  "m4b_exchange_combine_wvb")
        return out

    def merge_wvb(self, partials: torch.Tensor, w_uv: torch.Tensor, out: torch.Tensor,
                  attn_out: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
        """publish + combine_wvb in one launch (m4b_exchange_merge_wvb)."""
        a = m4.PhaseArgs()
        a.src[0] = m4.gtensor(w_uv, list(reversed(w_uv.shape)))
        a.src[1] = m4.gtensor(partials, [m4.PART_STRIDE, m4.HEADS, partials.shape[0], 1])
        if attn_out is not None:
            a.src[2] = m4._heads_desc(attn_out, m4.LATENT)
        a.dst = m4._heads_desc(out, m4.VHEAD)
        a.flags = flags
        m4._check(_lib.m4b_exchange_merge_wvb(self._h, ctypes.byref(a), m4._stream()),
                  "m4b_exchange_merge_wvb")
        return out

    def close(self, group=None) -> None:
        """Collective: unmap the peers, meet every rank, then free this GPU's buffer."""
        if self._h:
            rc = _lib.m4b_exchange_detach(self._h)
            dist.barrier(group=group)
            rc2 = _lib.m4b_exchange_destroy(self._h)
            self._h = None
            m4._check(rc or rc2, "m4b_exchange close")
