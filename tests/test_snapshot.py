"""Snapshots in the reference's file layout (linuxformer_b200.snapshot): a file written by the
reference's own writer (tests/golden/snapshot_ref.safetensors, made by
tests/golden/make_snapshot.py) reads back bit for bit, our files read back and, where the
reference's checkout is present, load with the reference's own reader; the bitwise diff finds
every changed element; on a GPU a decoded stream's state goes through a file and back."""

import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from linuxformer_b200 import chip as C
from linuxformer_b200 import snapshot

GOLD = Path(__file__).parent / "golden"
REF = Path(os.environ["LXB_REFERENCE"]) / "lx" if os.environ.get("LXB_REFERENCE") else None


def _fixture():
    spec = importlib.util.spec_from_file_location("make_snapshot", GOLD / "make_snapshot.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m.fixture()


def _same_bits(a, b) -> bool:
    return snapshot.diff(a, b)["elements_differ"] == 0


def test_reads_the_reference_writers_file():
    state, host, ref = _fixture()
    d = snapshot.load(GOLD / "snapshot_ref.safetensors")
    assert _same_bits(d["state"], state)
    assert {k: d[k] for k in host} == host
    assert vars(d["ref"]) == ref
    assert type(d["ref"].ram) is bytearray and type(d["ref"].out) is bytes


@pytest.mark.parametrize("suffix", [".safetensors", ".pt"])
def test_round_trip(tmp_path, suffix, c1_chip):
    st = C.c1_state(c1_chip, 0)
    state = snapshot.of_host(st)
    ref = {"pc": 4, "ram": bytearray(b"\x01\x02"), "out": b"hi"}
    p = tmp_path / f"s{suffix}"
    snapshot.save(p, state, next=5, last=6, n=7, waiting=False, ref=ref)
    d = snapshot.load(p)
    assert _same_bits(d["state"], state)
    assert (d["next"], d["last"], d["n"], d["waiting"]) == (5, 6, 7, False)
    assert vars(d["ref"]) == ref
    back = snapshot.to_host(d["state"])
    assert np.array_equal(back.conv, st.conv)
    assert np.array_equal(back.recurrent.view(np.uint32), st.recurrent.view(np.uint32))


@pytest.mark.skipif(REF is None or not REF.exists(),
                    reason="LXB_REFERENCE (the reference checkout) is not set")
def test_the_references_reader_loads_our_file(tmp_path):
    state, host, ref = _fixture()
    p = tmp_path / "ours.safetensors"
    snapshot.save(p, state, ref=ref, **host)
    sys.path.insert(0, str(REF))
    try:
        from lx.session import load_safe
    except Exception as e:  # (its dependencies missing here)
        pytest.skip(f"the reference's session module does not import: {e}")
    d = load_safe(p)
    assert _same_bits(d["state"], state)
    assert {k: d[k] for k in host} == host
    assert {k: vars(d["ref"])[k] for k in ref} == ref  # (its Machine class has properties)


def test_diff_counts_bits():
    a = [(torch.zeros(4, 4, dtype=torch.bfloat16), torch.zeros(2, 3))]
    b = [(a[0][0].clone(), a[0][1].clone())]
    assert snapshot.diff(a, b)["elements_differ"] == 0
    b[0][1][1, 2] = -0.0                       # -0 differs from +0 bitwise
    b[0][0][3, 1] = 1.0
    r = snapshot.diff(a, b)
    assert r["elements"] == 22 and r["elements_differ"] == 2
    assert {(d["state"], tuple(d["index"])) for d in r["differences"]} == {
        ("conv", (3, 1)), ("recurrent", (1, 2))}
    with pytest.raises(ValueError):
        snapshot.diff(a, [(a[0][0], torch.zeros(3, 2))])


@pytest.mark.gpu
def test_decoded_stream_survives_a_file(tmp_path, c1_chip):
    """Decode 12 tokens, save the stream's state, decode 12 more; load the file into fresh states
    and decode the same 12: the same predictions and a bit-identical final state."""
    from linuxformer_b200.runtime import Decoder

    dec = Decoder(c1_chip, cluster=16)
    ds = dec.states([C.c1_state(c1_chip, 0)])
    p0, _ = dec.run(ds, [[0]], 12)
    nxt = int(p0[0, -1])
    snapshot.save(tmp_path / "mid.safetensors", snapshot.of_states(ds, 0), next=nxt, n=12)
    p1, _ = dec.run(ds, [[nxt]], 12)
    d = snapshot.load(tmp_path / "mid.safetensors")
    ds2 = dec.states(1)
    snapshot.into(ds2, 0, d["state"])
    p2, _ = dec.run(ds2, [[d["next"]]], 12)
    assert torch.equal(p1, p2)
    r = snapshot.diff(snapshot.of_states(ds, 0), snapshot.of_states(ds2, 0))
    assert r["elements_differ"] == 0, r["differences"][:3]
