"""Verified mode (the reference's Session.verify over its chunked prefill): the CPU restatement
pinned to the reference's own chunked forward (tests/golden/c1_prefill.npz, made by
tests/golden/make_golden.py), the verifier's bookkeeping, and on a GPU the kernel through the
Mega drop-in against the same fixture."""

from types import SimpleNamespace

import numpy as np
import pytest

from linuxformer_b200 import chip as C
from linuxformer_b200.verify import Verifier

GOLD = __import__("pathlib").Path(__file__).parent / "golden"


def test_oracle_matches_stock_chunked_prefill(c1_chip):
    """Two 256-token chunks from the seeded state, each one recurrent pass with every input
    forced: the stock chunked forward's predictions and conv windows bit for bit, its recurrent
    states within 1e-9 (they are sums in another order)."""
    from oracle.oracle import Oracle

    g = np.load(GOLD / "c1_prefill.npz")
    assert str(g["digest"]) == c1_chip.digest()
    st = C.c1_state(c1_chip, 0)
    o = Oracle(c1_chip)
    for k in range(2):
        ids = g[f"ids{k}"].astype(np.int32)
        p, _, _ = o.decode(st, ids, len(ids))
        assert (p == g[f"preds{k}"]).all()
        assert np.array_equal(st.conv, g[f"conv{k}"])
        assert np.abs(st.recurrent[:, [5, 77]] - g[f"rec_heads{k}"]).max() <= 1e-9


class _Fixed:
    """A stand-in for Mega: predictions from a table of the next token per input."""

    def __init__(self, nxt):
        self.nxt, self.calls = nxt, []

    def run(self, forced, n):
        assert len(forced) == n
        self.calls.append(list(forced))
        return [self.nxt.get(t, 0) for t in forced]


def test_verifier_bookkeeping():
    nxt = {1: 2, 2: 3, 3: 9, 4: 5, 5: 6, 6: 7, 9: 1}
    m = _Fixed(nxt)
    v = Verifier(m, chunk=2, go=1)
    r = v.verify([2, 3, 4])  # GO prepended: 1 2 3 4; predictions 2 3 9 5
    assert m.calls == [[1, 2], [3, 4]]
    assert r["predicted"].tolist() == [2, 3, 9, 5]
    assert r["wrong"] == 1 and r["first_wrong"] == [(3, 4, 9)]
    r = v.verify([5, 6])  # the previous call predicted 5 for the first token: right
    assert r["wrong"] == 0 and r["predicted"].tolist() == [6, 7] and v.next == 7
    r = v.verify([8])  # 7 was predicted
    assert r["first_wrong"] == [(0, 8, 7)]
    v2 = Verifier(_Fixed(nxt), typed=lambda t: t == 4, go=None)
    r = v2.verify([1, 2, 3, 4])  # 4 is typed: its wrong prediction is not counted
    assert r["wrong"] == 0


@pytest.mark.gpu
def test_verify_on_the_kernel_matches_stock_prefill(c1_chip):
    """Two 256-token verify calls through the Mega drop-in on the reference's own model and
    cache: the stock chunked forward's predictions and conv windows, recurrent states within
    1e-9."""
    import torch
    from transformers import DynamicCache

    from linuxformer_b200.mega import Mega

    g = np.load(GOLD / "c1_prefill.npz")
    model = C.to_hf(c1_chip).to("cuda")
    st0 = C.c1_state(c1_chip, 0)
    cache = DynamicCache(config=model.config)
    for L in range(c1_chip.n_layers):
        cache.update_conv_state(torch.zeros((1, C.CONV, 4), dtype=torch.bfloat16, device="cuda"), L)
        lay = cache.layers[L]
        lay.recurrent_states = torch.from_numpy(st0.recurrent[L].copy())[None].to("cuda")
        lay.is_recurrent_states_initialized = True
    fast = SimpleNamespace(n_chip=c1_chip.n_layers, w_head=model.lm_head.weight)
    v = Verifier(Mega(fast, model, cache, 0), chunk=100)  # chunks of 100: three launches a call
    for k in range(2):
        r = v.verify(g[f"ids{k}"].tolist())
        assert r["predicted"].tolist() == g[f"preds{k}"].tolist()
        conv = np.stack([cache.layers[L].conv_states[0].view(torch.int16).cpu().numpy()
                         .view(np.uint16) for L in range(c1_chip.n_layers)])
        assert np.array_equal(conv, g[f"conv{k}"])
        rec = np.stack([cache.layers[L].recurrent_states[0].cpu().numpy()
                        for L in range(c1_chip.n_layers)])
        assert np.abs(rec[:, [5, 77]] - g[f"rec_heads{k}"]).max() <= 1e-9


def test_oracle_matches_stock_chunked_prefill_8192(c1_chip):
    """Config 3's first chunk (8,192 ids, seed 2) through the reference's own chunked forward
    (tests/golden/c1_prefill8k.npz): the forced per-token oracle gives the same predictions for
    the first 2,048 positions (a prefix keeps the CPU suite quick; the GPU test runs all 8,192)."""
    from oracle.oracle import Oracle

    g = np.load(GOLD / "c1_prefill8k.npz")
    assert str(g["digest"]) == c1_chip.digest()
    n = 2048
    p, _, _ = Oracle(c1_chip).decode(C.c1_state(c1_chip, 0), g["ids"][:n].astype(np.int32), n)
    assert (p == g["preds"][:n]).all()
