"""The drop-in for lx.mega.Mega: its tables come from the stock model's own weights, and it
decodes in place on the reference's HF cache tensors."""

from types import SimpleNamespace

import numpy as np
import pytest

from linuxformer_b200 import chip as C

GOLD = __import__("pathlib").Path(__file__).parent / "golden"


def test_chip_from_model_is_lossless(c1_chip):
    from linuxformer_b200.mega import chip_from_model

    back = chip_from_model(C.to_hf(c1_chip), c1_chip.n_layers)
    for a, b in zip(c1_chip.layers, back.layers):
        for f in ("qkv", "z", "b", "a", "out", "gate", "up", "down"):
            x, y = getattr(a, f), getattr(b, f)
            assert np.array_equal(x.indptr, y.indptr) and np.array_equal(x.indices, y.indices)
            assert np.array_equal(x.data, y.data), f
        for f in ("conv", "A_log", "dt_bias", "gnorm", "ln_in", "ln_post"):
            assert np.array_equal(getattr(a, f), getattr(b, f)), f
    assert np.array_equal(back.embed, c1_chip.embed)
    assert np.array_equal(back.head.indices, c1_chip.head.indices)
    assert np.array_equal(back.final_norm, c1_chip.final_norm) and back.eps == c1_chip.eps


@pytest.mark.gpu
def test_mega_shim_decodes_the_stock_stream_in_place(c1_chip):
    """Mega(fast, model, cache, offset).run(forced, n) on the reference's own model and cache:
    the stock stream (tests/golden/c1_decode.npz), the cache updated in place, inputs reported."""
    import torch
    from transformers import DynamicCache

    from linuxformer_b200.mega import Mega

    g = np.load(GOLD / "c1_decode.npz")
    model = C.to_hf(c1_chip).to("cuda")
    st0 = C.c1_state(c1_chip, 0)
    cache = DynamicCache(config=model.config)
    for L in range(c1_chip.n_layers):
        cache.update_conv_state(torch.zeros((1, C.CONV, 4), dtype=torch.bfloat16, device="cuda"), L)
        lay = cache.layers[L]
        lay.recurrent_states = torch.from_numpy(st0.recurrent[L].copy())[None].to("cuda")
        lay.is_recurrent_states_initialized = True
    fast = SimpleNamespace(n_chip=c1_chip.n_layers, w_head=model.lm_head.weight)
    m = Mega(fast, model, cache, 0)
    inputs = torch.zeros(200, dtype=torch.int32, device="cuda")
    p1 = m.run([0], 100, inputs=inputs)
    p2 = m.run([p1[-1]], 60)  # the next launch continues the stream (Linux.run_alone's pattern)
    assert p1 == g["preds"][:100].tolist()
    assert p2 == g["preds"][100:160].tolist()
    assert inputs[:100].tolist() == g["inputs"][:100].tolist()
    conv = np.stack([cache.layers[L].conv_states[0].view(torch.int16).cpu().numpy().view(np.uint16)
                     for L in range(c1_chip.n_layers)])
    assert conv.shape == (c1_chip.n_layers, C.CONV, 4)
