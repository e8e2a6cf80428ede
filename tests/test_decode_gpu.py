"""The CUDA decode (liblxb.so through its C ABI) against the CPU oracle and the reference's own
stock stream. Bit-exact: token streams, conv windows and recurrent states (values compared as
floats, so -0 and +0 agree: the stock forward itself differs from the sparse path only in a
zero's sign, lx/csrc/mega.cu:276)."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from linuxformer_b200 import chip as C  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

GOLD = __import__("pathlib").Path(__file__).parent / "golden"


def _decoder(chip, cluster):
    from linuxformer_b200.runtime import Decoder

    return Decoder(chip, cluster=cluster)


def _same_state(dev_states, s, host_state):
    got = dev_states.host(s)
    assert np.array_equal(got.conv, host_state.conv), "conv windows differ"
    diff = got.recurrent != host_state.recurrent
    assert not diff.any(), f"{int(diff.sum())} recurrent values differ"


def test_c1_matches_oracle(c1_chip):
    n = 40
    dec = _decoder(c1_chip, 16)
    st0 = C.c1_state(c1_chip, 0)
    ds = dec.states([st0])
    preds, inputs = dec.run(ds, [[0]], n)
    host = st0.copy()
    p, i, _ = Oracle(c1_chip).decode(host, [0], n)
    assert (preds[0].cpu().numpy() == p).all()
    assert (inputs[0].cpu().numpy() == i).all()
    _same_state(ds, 0, host)


def test_c1_stock_stream_512(c1_chip):
    """512 greedy tokens equal the reference's stock forward (tests/golden/c1_decode.npz)."""
    g = np.load(GOLD / "c1_decode.npz")
    dec = _decoder(c1_chip, 16)
    ds = dec.states([C.c1_state(c1_chip, 0)])
    preds, inputs = dec.run(ds, [[0]], 512)
    assert (preds[0].cpu().numpy() == g["preds"]).all()
    got = ds.host(0)
    assert np.array_equal(got.conv, g["conv"])
    assert np.abs(got.recurrent[:, [5, 77]] - g["rec_heads"]).max() <= 1e-9


def test_streams_are_independent(c1_chip):
    """Three machines with their own states and forced prefixes, one launch: each equals its
    own oracle run."""
    n = 24
    dec = _decoder(c1_chip, 16)
    sts = [C.c1_state(c1_chip, s) for s in (0, 3, 4)]
    forced = [[0, 5, 9], [17, 17, 3], [4095, 1, 2]]
    ds = dec.states(sts)
    preds, _ = dec.run(ds, forced, n)
    o = Oracle(c1_chip)
    for s in range(3):
        host = sts[s].copy()
        p, _, _ = o.decode(host, forced[s], n)
        assert (preds[s].cpu().numpy() == p).all()
        _same_state(ds, s, host)


def test_bad_token_sets_status(c1_chip):
    """A forced token outside the embedding is clamped and reported, not read out of bounds."""
    from linuxformer_b200._lib import LxbError

    dec = _decoder(c1_chip, 16)
    ds = dec.states([C.c1_state(c1_chip, 0)])
    with pytest.raises(LxbError, match="device status"):
        dec.run(ds, [[0, 5000]], 4)
    preds, _ = dec.run(ds, [[0]], 2)  # the plan stays usable
    assert preds.shape == (1, 2)


@pytest.mark.parametrize("cluster", [16, 8])
def test_c2_matches_oracle(cluster):
    """The 37-layer chip-shaped stack (a 20,000-row head to keep the oracle quick), on clusters
    of 16 and of 8 CTAs: streams, conv windows and recurrent states bit-identical."""
    chip = C.c2(1, vocab=20000)
    st0 = C.c2_state(chip, 1)
    n = 48
    dec = _decoder(chip, cluster)
    ds = dec.states([st0])
    preds, _ = dec.run(ds, [[0]], n)
    host = st0.copy()
    p, _, _ = Oracle(chip).decode(host, [0], n)
    assert (preds[0].cpu().numpy() == p).all()
    _same_state(ds, 0, host)


@pytest.mark.parametrize("which", ["c1", "c2"])
def test_chained_short_launches(c1_chip, which):
    """Launches of 1, 2, 5, 3 and 7 steps, each continuing from the last prediction (as
    Linux.run_alone chains Mega.run): the lazily kept conv windows are rebuilt at every launch's
    end, including launches shorter than the window; the whole equals one continuous run."""
    chip = c1_chip if which == "c1" else C.c2(1, vocab=20000)
    st0 = C.c1_state(chip, 0) if which == "c1" else C.c2_state(chip, 1)
    dec = _decoder(chip, 16)
    ds = dec.states([st0])
    got, last = [], 0
    for n in (1, 2, 5, 3, 7):
        preds, _ = dec.run(ds, [[last]], n)
        p = preds[0].cpu().numpy().tolist()
        got += p
        last = p[-1]
    host = st0.copy()
    want, _, _ = Oracle(chip).decode(host, [0], len(got))
    assert got == want.tolist()
    _same_state(ds, 0, host)


def test_head_helpers_match_and_fall_back():
    """The output head with helper clusters, without them, and with helpers that never answer
    (a drill: the decoding cluster's bounded wait runs out, it takes their rows itself and flags
    LXB_S_HELPER): the same stream as the oracle every time."""
    from linuxformer_b200._lib import S_HELPER, lib

    chip = C.c2(1, vocab=20000)
    st0 = C.c2_state(chip, 1)
    n = 12
    p, _, _ = Oracle(chip).decode(st0.copy(), [0], n)
    for helpers in (7, 0, -3):
        dec = _decoder(chip, 16)
        assert lib().lxb_plan_set_head_helpers(dec.plan, helpers) == 0
        ds = dec.states([st0])
        preds, _ = dec.run(ds, [[0]], n)
        assert (preds[0].cpu().numpy() == p).all(), helpers
        flagged = bool(dec.status().status & S_HELPER)
        assert flagged == (helpers < 0 and dec.max_clusters > 1), (helpers, dec.status().status)


def test_two_plans_share_one_scratch(c1_chip):
    """Two plans (the same chip, different machine states) take turns on ONE scratch buffer,
    with launches of equal lengths: 1 token each, then 9 tokens each. The head helpers' exchange
    words in that buffer are tagged per launch, so neither plan may take the other's stale head
    input or maximum; both streams equal their own oracle runs bit for bit."""
    import torch

    sts = [C.c1_state(c1_chip, 0), C.c1_state(c1_chip, 5)]
    decs = [_decoder(c1_chip, 16), _decoder(c1_chip, 16)]
    dss = [d.states([st]) for d, st in zip(decs, sts)]
    shared = decs[0].scratch(1)
    got = [[], []]
    last = [0, 7]
    for n in (1, 1, 9, 9):
        for k in (0, 1):
            f = torch.tensor([[last[k]]], dtype=torch.int32, device=decs[k].dev)
            preds = torch.empty((1, n), dtype=torch.int32, device=decs[k].dev)
            decs[k].launch(dss[k].ptrs, dss[k].bitmaps, f, n, preds, None, scratch=shared)
            p = preds[0].cpu().numpy().tolist()
            got[k] += p
            last[k] = p[-1]
    o = Oracle(c1_chip)
    for k, first in ((0, 0), (1, 7)):
        host = sts[k].copy()
        want, _, _ = o.decode(host, [first], len(got[k]))
        assert got[k] == want.tolist(), k
        _same_state(dss[k], 0, host)


def test_c2_full_head_matches_stock_stream():
    """The bench's config 2 (the full 459,982-row head) on the GPU: the 32 greedy tokens of the
    reference's own stock forward (tests/golden/c2_decode.npz), and the final conv windows and
    recurrent states bit for bit those of the CPU restatement on the same stream (which holds
    them to the stock forward's within the tolerance test_oracle_golden states)."""
    g = np.load(GOLD / "c2_decode.npz")
    chip = C.c2(1)
    assert str(g["digest"]) == chip.digest()
    st0 = C.c2_state(chip, 1)
    n = len(g["preds"])
    dec = _decoder(chip, 16)
    ds = dec.states([st0])
    preds, _ = dec.run(ds, [[0]], n)
    assert (preds[0].cpu().numpy() == g["preds"]).all()
    host = st0.copy()
    Oracle(chip).decode(host, [0], n)
    _same_state(ds, 0, host)
