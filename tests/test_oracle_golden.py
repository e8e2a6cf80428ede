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


def _bf16_order(x: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> integers in value order (adjacent values differ by 1: ulps)."""
    x = x.astype(np.int64)
    return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)


def test_oracle_matches_stock_on_config_2():
    """Config 2 (37 layers, the full 459,982-row head, the seeded RAM/ROM state) against the
    reference's own stock forward (tests/golden/c2_decode.npz, 32 greedy tokens one per call):
    every token identical and the two kept memory heads' states bit for bit. The stock forward
    sums in_proj_qkv's 15-entry value-channel rows in its CPU GEMM's blocked order, the oracle
    (and the kernel) sequentially, so a projection can round to a neighbouring bf16 value: at most
    32 of the ~348,000 nonzero conv windows may differ, each value by at most 16 bf16 ulps, and a
    key's write with such a value moves its head's state: every (layer, value head) sum within
    1% of the head's absolute sum."""
    g = np.load(GOLD / "c2_decode.npz")
    chip = C.c2(1)
    assert str(g["digest"]) == chip.digest()
    st = C.c2_state(chip, 1)
    preds, inputs, _ = Oracle(chip).decode(st, [0], len(g["preds"]))
    assert (preds == g["preds"]).all()
    assert (inputs == g["inputs"]).all()
    for (L, vh), h in zip(g["head_ids"], g["heads"]):
        assert not (st.recurrent[L, vh] != h).any()
    a, b = g["conv"], st.conv
    diff = (a != b) & (((a | b) & 0x7FFF) != 0)  # (+0 and -0 are the same value)
    assert int(diff.any(-1).sum()) <= 32
    assert np.abs(_bf16_order(a[diff]) - _bf16_order(b[diff])).max(initial=0) <= 16
    vs = st.recurrent.astype(np.float64).sum(axis=(2, 3))
    assert (np.abs(vs - g["rec_vh_sum"]) <= 0.01 * g["rec_vh_abs"] + 1e-30).all()
