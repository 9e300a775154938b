"""Peer-memory regions for the expert-parallel exchange (NVLink P2P, no collective library).

One process per GPU.  Every rank allocates one device buffer holding, for each
expert-parallel layer:

* a receive region: ``G`` chunks of ``cap + 1`` fp16 rows (chunk ``s`` from
  source rank ``s``; its last row carries ``s``'s expert counts), exactly what
  the dispatch all-to-all would deliver;
* a return region: ``G`` chunks of ``cap`` rows (chunk ``s`` from owner rank
  ``s``), what the combine all-to-all would deliver;
* two int32 flag arrays ``[G]`` (dispatch, return), written by the peers;
* this rank's own sequence numbers, CTA completion counters and the two words
  of the fused front launch's grid barrier.

The buffer's CUDA IPC handle is exchanged once over the process group (host
objects, ``all_gather_object``) and each peer's buffer is mapped with
``cudaIpcOpenMemHandle`` (plain peer mappings: no multicast object is
created).  The kernels (``moe_ep_front_p2p`` or ``moe_ep_dispatch_p2p``,
``moe_ep_return_partials_p2p`` or ``moe_ep_return_p2p``) then store token rows straight into the owners' receive
regions and results straight into the sources' return regions, and signal
with per-exchange sequence numbers (one system-scope fence, then the flag stores); every wait is bounded
(``moe_set_wait_limit_ns``).

Regions are per layer, so consecutive layers never reuse a region while a
slower peer may still be reading it; a whole decode step separates two uses
of the same region, and every layer's exchanges order the ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

_ALIGN = 256


def _align(v: int) -> int:
    return (v + _ALIGN - 1) // _ALIGN * _ALIGN


def _check(ret, what: str):
    """cuda-python returns (status, *values): raise on a bad status, return the values."""
    err = ret[0] if isinstance(ret, tuple) else ret
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: {err}")
    if not isinstance(ret, tuple) or len(ret) == 1:
        return None
    return ret[1] if len(ret) == 2 else ret[1:]


@dataclass(frozen=True)
class LayerRegions:
    """Every address one layer's two exchanges use (device addresses as ints)."""
    recv_table: int   # [G] uint64: each rank's receive region
    back_table: int   # [G] uint64: each rank's return region
    dflag_table: int  # [G] uint64: each rank's dispatch flags
    rflag_table: int  # [G] uint64: each rank's return flags
    recv: torch.Tensor  # this rank's receive region, fp16 rows [G*(cap+1), hidden]
    back: torch.Tensor  # this rank's return region, fp16 rows [G*cap, hidden]
    dflags: int
    rflags: int
    seq_d: int
    seq_r: int
    done_d: int
    done_r: int
    bar: int


class PeerExchange:
    """Per-layer exchange regions of ``world`` ranks, mapped into every rank."""

    def __init__(self, layers: int, world: int, rank: int, cap: int, hidden: int, group=None,
                 device=None) -> None:
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt

        self.layers, self.world, self.rank, self.cap, self.hidden = layers, world, rank, cap, hidden
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else \
            torch.device(device)
        G = world
        self.recv_bytes = _align(G * (cap + 1) * hidden * 2)
        self.back_bytes = _align(G * cap * hidden * 2)
        self.flag_bytes = _align(2 * G * 4)
        self.local_bytes = _align(6 * 4)  # seq[2], done[2], bar[2]
        self.layer_bytes = self.recv_bytes + self.back_bytes + self.flag_bytes + self.local_bytes
        total = self.layer_bytes * layers
        # Zeroed: flags, sequence numbers and completion counters start at 0.
        self.buf = torch.zeros(total, dtype=torch.uint8, device=self.device)
        ptr = self.buf.data_ptr()
        base, _size = _check(drv.cuMemGetAddressRange(ptr), "cuMemGetAddressRange")
        base = int(base)
        handle = _check(rt.cudaIpcGetMemHandle(base), "cudaIpcGetMemHandle")
        mine = (bytes(handle.reserved), ptr - base)
        gathered: list = [None] * world
        dist.all_gather_object(gathered, mine, group=group)
        self._opened = []
        addrs = []
        for r, (hbytes, off) in enumerate(gathered):
            if r == rank:
                addrs.append(ptr)
                continue
            h = rt.cudaIpcMemHandle_t()
            h.reserved = hbytes
            peer_base = _check(rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess),
                               "cudaIpcOpenMemHandle")
            self._opened.append(int(peer_base))
            addrs.append(int(peer_base) + off)
        self.peer_addrs = addrs
        tabs = []
        for l in range(layers):
            lo = l * self.layer_bytes
            tabs.append([[a + lo for a in addrs],                                        # recv
                         [a + lo + self.recv_bytes for a in addrs],                      # back
                         [a + lo + self.recv_bytes + self.back_bytes for a in addrs],    # flags d
                         [a + lo + self.recv_bytes + self.back_bytes + 4 * G for a in addrs]])
        # device tables [layers, 4, G] of uint64 addresses
        self.tables = torch.tensor(tabs, dtype=torch.int64, device=self.device)
        self._layers: dict = {}
        torch.distributed.barrier(group=group)

    # -- per-layer addresses -------------------------------------------------------------
    def _off(self, l: int) -> int:
        return l * self.layer_bytes

    def peer_table(self, l: int, which: int) -> int:
        """Device address of the [G] uint64 table: 0 recv, 1 back, 2 dispatch flags, 3 return flags."""
        return self.tables[l, which].data_ptr()

    def recv_rows(self, l: int) -> torch.Tensor:
        """This rank's receive region of layer ``l`` as fp16 rows [G*(cap+1), hidden]."""
        o = self._off(l)
        n = self.world * (self.cap + 1) * self.hidden
        return self.buf[o:o + 2 * n].view(torch.float16).view(self.world * (self.cap + 1),
                                                              self.hidden)

    def back_rows(self, l: int) -> torch.Tensor:
        """This rank's return region of layer ``l`` as fp16 rows [G*cap, hidden]."""
        o = self._off(l) + self.recv_bytes
        n = self.world * self.cap * self.hidden
        return self.buf[o:o + 2 * n].view(torch.float16).view(self.world * self.cap, self.hidden)

    def own_flags(self, l: int, d: int) -> int:
        return self.buf.data_ptr() + self._off(l) + self.recv_bytes + self.back_bytes + 4 * self.world * d

    def seq(self, l: int, d: int) -> int:
        return self.buf.data_ptr() + self._off(l) + self.recv_bytes + self.back_bytes + \
            self.flag_bytes + 4 * d

    def done(self, l: int, d: int) -> int:
        return self.seq(l, d) + 8

    def bar(self, l: int) -> int:
        """The grid-barrier words (arrivals, generation) of layer ``l``'s front launch."""
        return self.seq(l, 0) + 16

    def layer(self, l: int) -> LayerRegions:
        """Layer ``l``'s addresses, computed once (the regions never move), so that a call
        on the host does no tensor indexing to find them."""
        got = self._layers.get(l)
        if got is None:
            got = LayerRegions(self.peer_table(l, 0), self.peer_table(l, 1), self.peer_table(l, 2),
                               self.peer_table(l, 3), self.recv_rows(l), self.back_rows(l),
                               self.own_flags(l, 0), self.own_flags(l, 1), self.seq(l, 0),
                               self.seq(l, 1), self.done(l, 0), self.done(l, 1), self.bar(l))
            self._layers[l] = got
        return got

    def close(self) -> None:
        from cuda.bindings import runtime as rt

        for p in self._opened:
            rt.cudaIpcCloseMemHandle(p)
        self._opened = []
