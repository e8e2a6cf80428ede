"""lxb_decode_noalloc: the decode for hosts that cannot give the library device memory while
they run (a server that carves all device memory into one pool at start-up, or a host whose
allocator is not CUDA-aware and only passes the buffers it owns). Its scratch is a fixed array
inside the library instead of a caller buffer. Through the C ABI, two calls in a row must give
exactly what lxb_decode gives with a caller-allocated scratch: the same predictions and the same
final states, bit for bit (the tolerance of every other decode test here).

This file is collected last on purpose, and works in a fresh process as well as after the
other tests (the first call on a device sets the array's address up)."""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from linuxformer_b200 import chip as C  # noqa: E402
from linuxformer_b200._lib import S_ERRORS, check, lib  # noqa: E402


def _noalloc(dec, ds, forced, n):
    f = torch.tensor([forced], dtype=torch.int32, device=dec.dev)
    preds = torch.empty((1, n), dtype=torch.int32, device=dec.dev)
    st = torch.cuda.current_stream(dec.dev).cuda_stream
    check(lib().lxb_decode_noalloc(dec.plan, ds.ptrs.data_ptr(), ds.bitmaps.data_ptr(), 1,
                                   dec.embed.data_ptr(), 1, f.data_ptr(), f.shape[1], n,
                                   preds.data_ptr(), None, st), "lxb_decode_noalloc")
    torch.cuda.synchronize(dec.dev)
    assert (dec.status().status & S_ERRORS) == 0
    return preds[0].cpu().numpy()


def test_noalloc_matches_allocating_decode():
    from linuxformer_b200.runtime import Decoder

    chip = C.c1(0)
    st0 = C.c1_state(chip, 0)
    dec = Decoder(chip, cluster=16)
    assert lib().lxb_scratch_bytes(dec.plan, 1) <= 4 << 20
    a = dec.states([st0])  # lxb_decode, scratch allocated by the caller
    b = dec.states([st0])  # lxb_decode_noalloc, the library's fixed array
    la = lb = 0
    for n in (37, 29):     # two calls in a row, each continuing its stream
        pa, _ = dec.run(a, [[la]], n)
        pa = pa[0].cpu().numpy()
        pb = _noalloc(dec, b, [lb], n)
        assert (pa == pb).all()
        la, lb = int(pa[-1]), int(pb[-1])
    sa, sb = a.host(0), b.host(0)
    assert np.array_equal(sa.conv, sb.conv)
    assert not (sa.recurrent != sb.recurrent).any()


def test_noalloc_rejects_requests_beyond_its_array():
    from linuxformer_b200.runtime import Decoder

    chip = C.c1(0)
    dec = Decoder(chip, cluster=16)
    n = 1
    while lib().lxb_scratch_bytes(dec.plan, n) <= 4 << 20:
        n *= 2
    f = torch.zeros((n, 1), dtype=torch.int32, device=dec.dev)
    preds = torch.empty((n, 1), dtype=torch.int32, device=dec.dev)
    dummy = torch.zeros(16, dtype=torch.int64, device=dec.dev)
    rc = lib().lxb_decode_noalloc(dec.plan, dummy.data_ptr(), dummy.data_ptr(), 0,
                                  dec.embed.data_ptr(), n, f.data_ptr(), 1, 1, preds.data_ptr(),
                                  None, torch.cuda.current_stream(dec.dev).cuda_stream)
    assert rc == -5  # LXB_E_TOOBIG, before anything is launched
    assert lib().lxb_error_string(rc).decode().startswith("the request needs more scratch")
