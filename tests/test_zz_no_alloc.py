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
    """forced: one list per stream (equal lengths); returns the predictions [streams, n]."""
    S = ds.n_streams
    f = torch.tensor(forced, dtype=torch.int32, device=dec.dev).view(S, -1)
    preds = torch.empty((S, n), dtype=torch.int32, device=dec.dev)
    st = torch.cuda.current_stream(dec.dev).cuda_stream
    check(lib().lxb_decode_noalloc(dec.plan, ds.ptrs.data_ptr(), ds.bitmaps.data_ptr(), 1,
                                   dec.embed.data_ptr(), S, f.data_ptr(), f.shape[1], n,
                                   preds.data_ptr(), None, st), "lxb_decode_noalloc")
    torch.cuda.synchronize(dec.dev)
    assert (dec.status().status & S_ERRORS) == 0
    return preds.cpu().numpy()


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
        pb = _noalloc(dec, b, [[lb]], n)[0]
        assert (pa == pb).all()
        la, lb = int(pa[-1]), int(pb[-1])
    sa, sb = a.host(0), b.host(0)
    assert np.array_equal(sa.conv, sb.conv)
    assert not (sa.recurrent != sb.recurrent).any()


def test_noalloc_two_plans_in_turn():
    """Two plans with different machine states take turns on the one array with launches of the
    same lengths (1 token each, then 11 each): the array keeps the last call's contents, and the
    head helpers' exchange words in it must not let one plan take the other's stale head input or
    maximum. Each plan's stream equals lxb_decode's with a caller buffer, bit for bit."""
    from linuxformer_b200.runtime import Decoder

    chip = C.c1(0)
    sts = [C.c1_state(chip, 0), C.c1_state(chip, 6)]
    decs = [Decoder(chip, cluster=16), Decoder(chip, cluster=16)]
    ref = [d.states([st]) for d, st in zip(decs, sts)]
    nal = [d.states([st]) for d, st in zip(decs, sts)]
    last_r, last_n = [0, 3], [0, 3]
    for n in (1, 1, 11, 11):
        for k in (0, 1):
            pb = _noalloc(decs[k], nal[k], [[last_n[k]]], n)[0]
            pa, _ = decs[k].run(ref[k], [[last_r[k]]], n)
            pa = pa[0].cpu().numpy()
            assert (pa == pb).all(), (k, n)
            last_r[k], last_n[k] = int(pa[-1]), int(pb[-1])
    for k in (0, 1):
        sa, sb = ref[k].host(0), nal[k].host(0)
        assert np.array_equal(sa.conv, sb.conv)
        assert not (sa.recurrent != sb.recurrent).any()


def test_noalloc_several_streams():
    """Three streams in one call (no head helpers, the larger ring layout), twice in a row:
    the same predictions and states as lxb_decode."""
    from linuxformer_b200.runtime import Decoder

    chip = C.c1(0)
    dec = Decoder(chip, cluster=16)
    assert lib().lxb_scratch_bytes(dec.plan, 3) <= 4 << 20
    sts = [C.c1_state(chip, s) for s in (0, 1, 2)]
    a, b = dec.states(sts), dec.states(sts)
    fa = fb = [[0], [9], [100]]
    for n in (13, 17):
        pa, _ = dec.run(a, fa, n)
        pa = pa.cpu().numpy()
        pb = _noalloc(dec, b, fb, n)
        assert (pa == pb).all()
        fa = [[int(x)] for x in pa[:, -1]]
        fb = [[int(x)] for x in pb[:, -1]]
    for s in range(3):
        sa, sb = a.host(s), b.host(s)
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
