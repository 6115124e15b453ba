"""GPU parity of the dependent-load chase (reference src/memory_chase.cu,
include/memory_chase.h): the final index equals the oracle's host walk."""

import ctypes

import numpy as np
import pytest

from oracle import ptr
from tests.helpers import dptr, stream_handle

pytestmark = pytest.mark.gpu


def _run(cuda, cmb, links_np, warmup, hops, bypass_l1=1):
    d = cuda.from_numpy(links_np.view(np.int32)).cuda()
    out = cuda.zeros(4, dtype=cuda.int64, device="cuda")
    cmb.check("cmb_chase_run", dptr(d), links_np.size, ctypes.c_uint64(warmup),
              ctypes.c_uint64(hops), bypass_l1, dptr(out), stream_handle(cuda))
    return [int(v) for v in out.cpu().numpy().view(np.uint64)]


@pytest.mark.parametrize("slots,warmup,hops", [(1, 0, 5), (64, 3, 1000), (4096, 1024, 4096 * 3 + 7)])
@pytest.mark.parametrize("bypass", [1, 0])
def test_chase_endpoint_matches_walk(cuda, cmb, orc, slots, warmup, hops, bypass):
    links = np.empty(slots * 32, np.uint32)
    cmb.check("cmb_chase_build_links", ctypes.c_void_p(links.ctypes.data), links.nbytes,
              ctypes.c_uint64(9))
    cycles, idx, ns, status = _run(cuda, cmb, links, warmup, hops, bypass)
    assert status == 0
    assert idx == orc.orc_chase_walk(ptr(links), warmup + hops, 0)
    assert cycles > 0 and ns > 0


def test_chase_full_footprint(cuda, cmb, orc):
    """Config: 512 MiB (2^22 slots), Sattolo cycle; endpoint vs host walk.
    2^20 timed hops here (the bench runs 2^24)."""
    nbytes = 512 << 20
    links = np.empty(nbytes // 4, np.uint32)
    cmb.check("cmb_chase_build_links", ctypes.c_void_p(links.ctypes.data), nbytes,
              ctypes.c_uint64(0xC0DA))
    hops = 1 << 20
    cycles, idx, ns, status = _run(cuda, cmb, links, 1024, hops)
    assert status == 0
    assert idx == orc.orc_chase_walk(ptr(links), 1024 + hops, 0)
    ns_per_hop = ns / hops
    assert 100 < ns_per_hop < 5000, ns_per_hop  # DRAM latency, not a cache hit


def test_chase_rejects_corrupt_links(cuda, cmb):
    links = np.empty(64 * 32, np.uint32)
    cmb.check("cmb_chase_build_links", ctypes.c_void_p(links.ctypes.data), links.nbytes,
              ctypes.c_uint64(1))
    links[5 * 32] = 0xFFFFFF00  # out of range: the walk must not start
    cycles, idx, ns, status = _run(cuda, cmb, links, 0, 100)
    assert status == 1 and cycles == 0 and idx == 0


def test_chase_rejects_bad_words(cuda, cmb):
    d = cuda.zeros(64, dtype=cuda.int32, device="cuda")
    out = cuda.zeros(4, dtype=cuda.int64, device="cuda")
    assert cmb.lib.cmb_chase_run(dptr(d), 33, 0, 1, 1, dptr(out), stream_handle(cuda)) == 1
