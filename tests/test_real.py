"""The real compiled circuit (tests/golden/real_chip.npz, built by the reference's own compiler and
machine model, tests/golden/make_real.py) on the CPU: the state rebuilt from the fixture is the
reference's own snapshot bit for bit, and the CPU restatement decoding the model alone from GO
reproduces the reference machine's token trace (as the reference's tools/mega_boot.py checks its
megakernel against the same machine)."""

import hashlib

import numpy as np

from linuxformer_b200 import chip as C
from oracle.oracle import Oracle


def test_state_is_the_reference_snapshot(real_chip):
    st = C.real_state(real_chip)
    m = real_chip.meta
    assert hashlib.sha256(st.recurrent.tobytes()).hexdigest() == m["state_sha256"]
    assert not st.conv.any()


def test_structure(real_chip):
    """The sizes the reference reports for its megakernel on this circuit
    (lx/results/mega_check_start.json: 5.87M CSR entries over 497 items, 360,883 channels, a
    head of 31 dense and 191 sparse columns holding 4,133,751 entries)."""
    from linuxformer_b200 import tables as T

    assert real_chip.n_layers == 37 and real_chip.n_vocab == 459982
    cnt = np.bincount(real_chip.head.indices, minlength=C.H)
    dense = np.nonzero(cnt == real_chip.n_vocab)[0]
    sparse = np.nonzero((cnt > 0) & (cnt < real_chip.n_vocab))[0]
    assert len(dense) == 31 and len(sparse) == 191
    assert int(cnt[sparse].sum()) == 4133751
    _, st = T.build_image(real_chip, 16)
    assert st["items"] == 497 and st["chans"] == 360883
    assert st["head_dense"] == 31 and st["head_sparse_nnz"] == 4133751


def test_oracle_reproduces_the_machine(real_chip):
    tr = real_chip.meta["fixture"]["trace"]
    n = 48
    st = C.real_state(real_chip)
    preds, inputs, _ = Oracle(real_chip).decode(st, [int(tr[0])], n)
    assert inputs[0] == real_chip.meta["go"]
    assert (preds == tr[1:n + 1]).all(), np.nonzero(preds != tr[1:n + 1])[0][:5]


def test_oracle_matches_stock_bit_for_bit():
    """The reference's own stock forward on the real circuit (tests/golden/real_decode.npz: the
    HF decoder layers run as lx.hf.chip_forward runs them, 32 tokens from GO one per call, its
    predictions the machine's trace): every token identical, and after them every layer's conv
    windows and recurrent state identical bit for bit (-0 written as +0: a product with a zero
    weight or input that the sparse path never forms can differ in a zero's sign only). Here the
    stock CPU GEMM's summation order makes no difference: the circuit's sums are exact."""
    from pathlib import Path

    g = np.load(Path(__file__).parent / "golden" / "real_decode.npz")
    chip = C.real()
    st = C.real_state(chip)
    preds, inputs, _ = Oracle(chip).decode(st, [int(g["inputs"][0])], len(g["preds"]))
    assert (preds == g["preds"]).all() and (inputs == g["inputs"]).all()
    cv = np.where((st.conv & 0x7FFF) == 0, 0, st.conv).astype(np.uint16)
    rv = np.where(st.recurrent == 0, np.float32(0), st.recurrent).astype(np.float32)
    for L in range(chip.n_layers):
        assert hashlib.sha256(np.ascontiguousarray(cv[L]).tobytes()).hexdigest() == g["conv_sha"][L]
        assert (hashlib.sha256(np.ascontiguousarray(rv[L]).view(np.uint32).tobytes()).hexdigest()
                == g["rec_sha"][L]), f"layer {L}'s recurrent state"
