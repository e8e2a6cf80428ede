"""The CUDA decode on the real compiled circuit (tests/golden/real_chip.npz): the model alone,
fed its own predictions from GO, reproduces the reference machine's token trace across chained
launches, and its states stay bit-identical to the CPU restatement's."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from linuxformer_b200 import chip as C  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402


def test_real_matches_oracle_states(real_chip):
    from linuxformer_b200.runtime import Decoder

    n = 64
    tr = real_chip.meta["fixture"]["trace"]
    st0 = C.real_state(real_chip)
    dec = Decoder(real_chip, cluster=16)
    ds = dec.states([st0])
    preds, inputs = dec.run(ds, [[int(tr[0])]], n)
    host = st0.copy()
    p, i, _ = Oracle(real_chip).decode(host, [int(tr[0])], n)
    assert (preds[0].cpu().numpy() == p).all()
    assert (inputs[0].cpu().numpy() == i).all()
    got = ds.host(0)
    assert np.array_equal(got.conv, host.conv), "conv windows differ"
    assert not (got.recurrent != host.recurrent).any(), "recurrent states differ"


def test_real_reproduces_the_machine(real_chip):
    """65,536 tokens in launches of 8,192 (each continuing from the last prediction, as
    Linux.run_alone chains Mega.run) equal the reference machine's trace."""
    from linuxformer_b200.runtime import Decoder

    chip = real_chip
    tr = chip.meta["fixture"]["trace"]
    dec = Decoder(chip, cluster=16)
    ds = dec.states([C.real_state(chip)])
    T, n = 8192, 65536
    got = []
    nxt = int(tr[0])
    for _ in range(n // T):
        preds, _ = dec.run(ds, [[nxt]], T)
        p = preds[0].cpu().numpy()
        got.append(p)
        nxt = int(p[-1])
    got = np.concatenate(got)
    bad = np.nonzero(got != tr[1:n + 1])[0]
    assert len(bad) == 0, f"first difference at token {bad[0] + 1} of {n}"
    assert dec.status().status == 0


def test_real_matches_stock_forward(real_chip):
    """32 tokens from GO against the reference's stock forward (tests/golden/real_decode.npz):
    the tokens and, after them, every layer's conv windows and recurrent state bit for bit (-0
    written as +0)."""
    import hashlib
    from pathlib import Path

    from linuxformer_b200.runtime import Decoder

    g = np.load(Path(__file__).parent / "golden" / "real_decode.npz")
    dec = Decoder(real_chip, cluster=16)
    ds = dec.states([C.real_state(real_chip)])
    preds, inputs = dec.run(ds, [[int(g["inputs"][0])]], len(g["preds"]))
    assert (preds[0].cpu().numpy() == g["preds"]).all()
    assert (inputs[0].cpu().numpy() == g["inputs"]).all()
    st = ds.host(0)
    cv = np.where((st.conv & 0x7FFF) == 0, 0, st.conv).astype(np.uint16)
    rv = np.where(st.recurrent == 0, np.float32(0), st.recurrent).astype(np.float32)
    for L in range(real_chip.n_layers):
        assert hashlib.sha256(np.ascontiguousarray(cv[L]).tobytes()).hexdigest() == g["conv_sha"][L]
        assert (hashlib.sha256(np.ascontiguousarray(rv[L]).view(np.uint32).tobytes()).hexdigest()
                == g["rec_sha"][L]), f"layer {L}'s recurrent state"
