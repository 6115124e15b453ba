"""Multi-GPU probe host logic: the NVLink ring and all-to-all exchanges.

One process per GPU (torchrun).  Every rank owns a send and a receive buffer
of `nbytes` allocated with cmb_p2p_alloc; the ranks swap CUDA IPC handles of
their receive buffers through torch.distributed, map the peers' buffers, and
then write straight into them with the library's peer-store kernel, its
bulk-copy kernel, its copy-engine scatter or both engines at once (hybrid).  torch.distributed carries only the handle exchange,
barriers and the max-over-ranks timing reduction: the data path uses no
collective library.

Plans (all offsets in bytes):
  ring:      rank r sends its whole buffer to rank (r + 1) % N.
  alltoall:  the buffer is N chunks; rank r sends chunk j to rank j, which
             stores it at chunk position r (chunk r stays local).  Rank r
             lists its jobs staggered, peers r+1, r+2, ... first and its own
             chunk last, so at every position of the job list each rank
             receives from exactly one sender (the order the copy engines
             visit them when the jobs share one stream).
"""

import ctypes
from typing import List, NamedTuple


class Job(NamedTuple):
    src_off: int
    dst_rank: int
    dst_off: int
    nbytes: int


class Source(NamedTuple):
    recv_off: int
    src_rank: int
    src_off: int
    nbytes: int


def chunk_bytes(world: int, nbytes: int) -> int:
    if nbytes % (16 * world):
        raise ValueError(f"{nbytes} bytes do not split into {world} 16-byte aligned chunks")
    return nbytes // world


def plan(mode: str, rank: int, world: int, nbytes: int) -> List[Job]:
    """Copies rank `rank` issues."""
    if mode == "ring":
        return [Job(0, (rank + 1) % world, 0, nbytes)]
    if mode == "alltoall":
        c = chunk_bytes(world, nbytes)
        order = [(rank + 1 + k) % world for k in range(world)]
        return [Job(j * c, j, rank * c, c) for j in order]
    raise ValueError(mode)


def sources(mode: str, rank: int, world: int, nbytes: int) -> List[Source]:
    """What rank `rank`'s receive buffer holds afterwards, and from where."""
    if mode == "ring":
        return [Source(0, (rank - 1) % world, 0, nbytes)]
    if mode == "alltoall":
        c = chunk_bytes(world, nbytes)
        return [Source(i * c, i, rank * c, c) for i in range(world)]
    raise ValueError(mode)


def egress_bytes(mode: str, rank: int, world: int, nbytes: int) -> int:
    """Bytes rank `rank` sends to other GPUs (local copies excluded)."""
    return sum(j.nbytes for j in plan(mode, rank, world, nbytes) if j.dst_rank != rank)


def parse_hybrid(method: str):
    """"hybrid_<P>_<S>": the copy engines take P/1000 of each job on S
    internal streams, the SMs' peer stores the rest."""
    parts = method.split("_")
    if len(parts) != 3 or parts[0] != "hybrid":
        raise ValueError(method)
    permille, streams = int(parts[1]), int(parts[2])
    if not (0 <= permille <= 1000 and 1 <= streams <= 8):
        raise ValueError(method)
    return permille, streams


class PeerExchange:
    """Send/receive buffers of this rank and the mapped receive buffers of
    all peers.  `ranks` provides rank, world, barrier() and dist."""

    def __init__(self, ranks, nbytes: int, seed: int):
        import torch

        from . import capi

        self.capi, self.lib, self.torch = capi, capi.lib, torch
        self.ranks, self.nbytes, self.seed = ranks, nbytes, seed
        # receive buffers are mapped by peers: a whole cudaMalloc allocation
        self.recv = self._alloc(nbytes)
        self._send_t = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        self._scratch_t = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        self._count_t = torch.zeros(1, dtype=torch.int64, device="cuda")
        self.send = ctypes.c_void_p(self._send_t.data_ptr())
        self.scratch = ctypes.c_void_p(self._scratch_t.data_ptr())
        self.count = ctypes.c_void_p(self._count_t.data_ptr())
        self.capi.check("cmb_fill_bytes", self.send, nbytes, ctypes.c_uint64(seed + ranks.rank), None)
        torch.cuda.synchronize()
        hb = self.lib.cmb_ipc_handle_bytes()
        handle = (ctypes.c_uint8 * hb)()
        self.capi.check("cmb_ipc_get_handle", self.recv, handle)
        mine = bytes(handle)
        allh = [None] * ranks.world
        ranks.dist.all_gather_object(allh, mine)
        self.peer_recv = []
        for r, h in enumerate(allh):
            if r == ranks.rank:
                self.peer_recv.append(self.recv)
            else:
                p = ctypes.c_void_p()
                hbuf = (ctypes.c_uint8 * hb).from_buffer_copy(h)
                self.capi.check("cmb_ipc_open", hbuf, ctypes.byref(p))
                self.peer_recv.append(p)
        ranks.barrier()

    def _alloc(self, n: int) -> ctypes.c_void_p:
        p = ctypes.c_void_p()
        self.capi.check("cmb_p2p_alloc", n, ctypes.byref(p))
        return p

    def launch(self, mode: str, method: str, stream) -> None:
        jobs = plan(mode, self.ranks.rank, self.ranks.world, self.nbytes)
        n = len(jobs)
        dst = (ctypes.c_void_p * n)(*[self.peer_recv[j.dst_rank].value + j.dst_off for j in jobs])
        src = (ctypes.c_void_p * n)(*[self.send.value + j.src_off for j in jobs])
        nb = (ctypes.c_size_t * n)(*[j.nbytes for j in jobs])
        if method == "store":
            self.capi.check("cmb_p2p_scatter_store", dst, src, nb, n, 0, stream)
        elif method == "bulk":
            self.capi.check("cmb_p2p_scatter_bulk", dst, src, nb, n, 0, None, stream)
        elif method == "copy_engine":
            self.capi.check("cmb_p2p_scatter_copy_engine", dst, src, nb, n, stream)
        elif method == "copy_engine_1stream":
            self.capi.check("cmb_p2p_scatter_copy_engine_tuned", dst, src, nb, n, 1, stream)
        elif method == "copy_engine_2stream":
            self.capi.check("cmb_p2p_scatter_copy_engine_tuned", dst, src, nb, n, 2, stream)
        elif method.startswith("hybrid_"):
            permille, streams = parse_hybrid(method)
            self.capi.check("cmb_p2p_scatter_hybrid", dst, src, nb, n, permille, streams, stream)
        else:
            raise ValueError(method)

    def mismatches(self, mode: str, stream) -> int:
        """Differing words between the receive buffer and what the plan says
        it must hold (each source regenerated from its rank's seed)."""
        total = 0
        for s in sources(mode, self.ranks.rank, self.ranks.world, self.nbytes):
            self.capi.check("cmb_fill_bytes", self.scratch, self.nbytes,
                            ctypes.c_uint64(self.seed + s.src_rank), stream)
            self.capi.check("cmb_compare_bytes", ctypes.c_void_p(self.recv.value + s.recv_off),
                            ctypes.c_void_p(self.scratch.value + s.src_off), s.nbytes, self.count,
                            stream)
            self.torch.cuda.synchronize()
            total += int(self._count_t.item())
        return total

    def close(self) -> None:
        self.ranks.barrier()
        for r, p in enumerate(self.peer_recv):
            if r != self.ranks.rank:
                self.capi.check("cmb_ipc_close", p)
        self.ranks.barrier()
        self.capi.check("cmb_p2p_free", self.recv)
        del self._send_t, self._scratch_t, self._count_t
