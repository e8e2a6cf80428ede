"""The CPU restatement (oracle/) against the reference's own stock forward.

tests/golden/c1_decode.npz holds what lx.hf.chip_forward + lx.hf.head_argmax (transformers'
torch GDN path, CPU) produced for config 1 (tests/golden/make_golden.py). The oracle must give
the same greedy tokens, bit-identical residuals and conv windows, and recurrent states within
TOL_REC (the stock sums its fp32 reductions in torch's CPU order; the oracle in the fixed order
the kernels share)."""

import numpy as np
import pytest

from linuxformer_b200 import chip as C
from oracle.oracle import Oracle, lib

GOLD = __import__("pathlib").Path(__file__).parent / "golden"
TOL_REC = 1e-9  # max-abs over recurrent-state values of magnitude <= ~1e-2


def test_generator_matches_fixture(c1_chip):
    g = np.load(GOLD / "c1_decode.npz")
    assert c1_chip.digest() == str(g["digest"])


def test_oracle_decode_matches_stock(c1_chip):
    g = np.load(GOLD / "c1_decode.npz")
    st = C.c1_state(c1_chip, 0)
    n = 96  # a prefix keeps the CPU suite quick; the full 512 run is test_oracle_decode_full
    preds, inputs, marg, rs = Oracle(c1_chip).decode(st, [0], n, resid=True)
    assert (preds == g["preds"][:n]).all()
    assert (inputs == g["inputs"][:n]).all()
    gr = C.bf16_float(g["resid"])
    assert np.array_equal(rs[:8].view(np.uint32), gr.view(np.uint32))


@pytest.mark.slow
def test_oracle_decode_full(c1_chip):
    g = np.load(GOLD / "c1_decode.npz")
    st = C.c1_state(c1_chip, 0)
    preds, inputs, marg = Oracle(c1_chip).decode(st, [0], 512)
    assert (preds == g["preds"]).all()
    assert np.array_equal(st.conv, g["conv"])
    heads = st.recurrent[:, [5, 77]]
    assert np.abs(heads - g["rec_heads"]).max() <= TOL_REC
    sums = st.recurrent.astype(np.float64).sum(axis=(2, 3))
    assert np.abs(sums - g["rec_sum"]).max() <= 1e-6


def test_math_functions_close_to_libm():
    """The shared exp/log1p/silu/sigmoid are within 2 ulp of numpy's float64 math."""
    L = lib()
    xs = np.concatenate([np.linspace(-100, 88, 20001), np.linspace(-1, 1, 2001),
                         [0.0, -0.0, 1e-30, -1e-30, 20.0, 20.5]]).astype(np.float32)
    for f, ref in ((L.lxo_exp, np.exp), (L.lxo_silu, lambda v: v / (1 + np.exp(-v))),
                   (L.lxo_sigmoid, lambda v: 1 / (1 + np.exp(-v)))):
        got = np.array([f(float(v)) for v in xs], np.float32)
        want = ref(xs.astype(np.float64)).astype(np.float32)
        # below -88.7 exp(-x) overflows: x / (1 + exp(-x)) is -0 there, as torch computes it
        fin = np.isfinite(want) & (np.abs(want) > 1e-37) & (xs > -88.0)
        ulp = np.abs(got[fin].view(np.int32).astype(np.int64) - want[fin].view(np.int32))
        assert ulp.max() <= 2, (f, ulp.max())
    ys = np.concatenate([np.logspace(-30, 8, 4001), [0.0]]).astype(np.float32)
    got = np.array([L.lxo_log1p(float(v)) for v in ys], np.float32)
    want = np.log1p(ys.astype(np.float64)).astype(np.float32)
    ulp = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32))
    assert ulp.max() <= 3
