"""Config 5's host side (linuxformer_b200.text), CPU only: the Gated DeltaNet padding pinned to
the reference's own merge.pad_gdn (tests/golden/c5_pad.npz, made by make_golden.py c5pad), the
packing of a config-5-shaped model, the fact that makes skipping the padding exact (the stock
forward leaves the padded heads, key rows and channels at exactly zero), and the stop-string
bookkeeping of TextDecoder.generate."""

from pathlib import Path

import numpy as np
import pytest
import torch

from linuxformer_b200 import text as T
from oracle.text_stock import steps, zero_cache

GOLD = Path(__file__).resolve().parent / "golden" / "c5_pad.npz"


def _expect(n, idx):
    a = np.full(n, -1)
    a[idx] = np.arange(len(idx))
    return a


def test_pad_maps_match_the_reference_pad_gdn():
    d = np.load(GOLD)
    rows, vrows, heads = T.pad_maps()
    assert (d["qkv"] == _expect(T.CONV, rows)).all()
    assert (d["conv"] == _expect(T.CONV, rows)).all()
    assert (d["z"] == _expect(T.NV * T.VD, vrows)).all()
    assert (d["out"] == _expect(T.NV * T.VD, vrows)).all()
    for k in ("b", "a", "dt_bias", "A_log"):
        assert (d[k] == _expect(T.NV, heads)).all(), k


@pytest.fixture(scope="module")
def small():
    """Three GDN layers and one attention layer of config 5's shape, a 512-row vocabulary."""
    return T.random_model(seed=4, n_layers=4, vocab=512, device="cpu")


def test_pack_keeps_exactly_the_live_rows(small):
    t = T.pack(small)
    rows, vrows, heads = (torch.as_tensor(a) for a in T.pad_maps())
    ga = small.model.layers[0].linear_attn
    d = t["layers"][0]
    assert d["type"] == 0 and d["w1"].shape == (T.W1_GDN, T.H)
    assert torch.equal(d["w1"][:8192], ga.in_proj_qkv.weight[rows])
    assert torch.equal(d["w1"][8192:12288], ga.in_proj_z.weight[vrows])
    assert torch.equal(d["w1"][12288:12320], ga.in_proj_b.weight[heads])
    assert torch.equal(d["w1"][12320:], ga.in_proj_a.weight[heads])
    assert torch.equal(d["conv"], ga.conv1d.weight.reshape(T.CONV, 4)[rows])
    assert torch.equal(d["wo"], ga.out_proj.weight[:, vrows])
    assert torch.equal(d["A_log"], ga.A_log.float()[heads])
    assert d["flags"] == 0  # a bf16 gated-norm weight
    mlp = small.model.layers[0].mlp
    assert torch.equal(d["wgu"][0::2], mlp.gate_proj.weight)
    assert torch.equal(d["wgu"][1::2], mlp.up_proj.weight)
    at = small.model.layers[3].self_attn
    d = t["layers"][3]
    assert d["type"] == 1 and d["w1"].shape == (T.W1_ATT, T.H)
    assert torch.equal(d["w1"], torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight]))
    assert torch.equal(d["wo"], at.o_proj.weight)
    assert t["head"].data_ptr() == t["embed"].data_ptr()  # tied


def test_pack_rejects_nonzero_padding(small):
    ga = small.model.layers[1].linear_attn
    _, vrows, _ = T.pad_maps()
    pad_row = sorted(set(range(T.NV * T.VD)) - set(vrows.tolist()))[0]
    with torch.no_grad():
        ga.in_proj_z.weight[pad_row, 7] = 1.0
        try:
            with pytest.raises(T.Unsupported, match="padding"):
                T.pack(small)
        finally:
            ga.in_proj_z.weight[pad_row, 7] = 0.0


def test_padding_stays_zero_in_the_stock_forward(small):
    """What the kernel skips is exactly zero in the stock forward: padded value heads' states,
    the padded key rows of live heads, the padded conv channels."""
    cache = zero_cache(small)
    steps(small, [1, 2, 3, 4, 5], cache, logits=False)
    rows, _, heads = T.pad_maps()
    pad_heads = sorted(set(range(T.NV)) - set(heads.tolist()))
    pad_ch = sorted(set(range(T.CONV)) - set(rows.tolist()))
    for L in range(3):
        rec = cache.layers[L].recurrent_states[0]
        assert not rec[pad_heads].any()
        assert not rec[heads][:, T.QKD:].any()
        assert rec[heads][:, :T.QKD].abs().sum() > 0
        conv = cache.layers[L].conv_states[0]
        assert not conv[pad_ch].any()
        assert conv[rows].abs().sum() > 0


def test_stop_strings():
    class Tok:
        def decode(self, ids):
            return "".join(chr(97 + i % 26) for i in ids)

    new = [0, 1, 2, 3, 4]  # "abcde"
    assert T._cut_at_stop(new, ["cd"], Tok()) == [0, 1, 2, 3]
    assert T._cut_at_stop(new, ["zz"], Tok()) == new
    assert T._stopped(new, ["bc"], Tok()) and not T._stopped(new, ["q"], Tok())
    assert not T._stopped(new, None, Tok())
