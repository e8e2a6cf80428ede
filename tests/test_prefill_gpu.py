"""The chunked prefill (liblxb.so's lxb_prefill through its C ABI) against the CPU oracle and the
reference's own chunked forward.

A chunk of T tokens through lxb_prefill must equal T steps of the per-token oracle with every
input forced (oracle.decode(state, forced=tokens, n=T)), bit for bit: every prediction, the conv
windows and the recurrent states (compared as floats, so -0 and +0 agree, as in the decode
tests). Against the reference's stock chunked forward (tests/golden/c1_prefill*.npz, made by
tests/golden/make_golden.py): the same predictions and conv windows, recurrent states within
1e-9 (the stock sums its chunked products in another order)."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from linuxformer_b200 import chip as C  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402

GOLD = __import__("pathlib").Path(__file__).parent / "golden"
TOL_REC = 1e-9


def _prefill(chip):
    from linuxformer_b200.prefill import Prefill

    return Prefill(chip)


def _states(chip, st):
    from linuxformer_b200.runtime import Decoder  # noqa: F401  (the same device layout)

    dev = torch.device("cuda")
    rec = torch.from_numpy(st.recurrent.copy()).to(dev)
    conv = torch.from_numpy(st.conv.view(np.int16).copy()).to(dev)
    ptrs = torch.tensor([[rec[L].data_ptr(), conv[L].data_ptr()] for L in range(chip.n_layers)],
                        dtype=torch.int64, device=dev)
    return rec, conv, ptrs


def _same(rec, conv, host):
    assert np.array_equal(conv.cpu().numpy().view(np.uint16), host.conv), "conv windows differ"
    got = rec.cpu().numpy()
    diff = got != host.recurrent
    assert not diff.any(), f"{int(diff.sum())} recurrent values differ"


def _ids(n, vocab, seed=2):
    return np.random.default_rng(seed).integers(0, vocab, n).astype(np.int32)


@pytest.mark.parametrize("T", [1, 3, 5, 67, 300])
def test_c1_chunk_matches_oracle(c1_chip, T):
    """Chunks shorter than the conv window, than a recurrence tile, and ragged ones: the
    predictions, conv windows and recurrent states of T forced decode steps."""
    st0 = C.c1_state(c1_chip, 0)
    ids = _ids(T, c1_chip.n_vocab)
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, st0)
    preds, first = pf.run(ptrs, ids)
    host = st0.copy()
    want, _, _ = Oracle(c1_chip).decode(host, ids, T)
    assert (preds.cpu().numpy() == want).all()
    ok = want[:-1] == ids[1:]
    assert first == (int(np.argmin(ok)) if not ok.all() else -1)
    _same(rec, conv, host)


def test_c1_chained_chunks_match_one_run(c1_chip):
    """Chunks of 1000, 7 and 1, 2 and 1500 tokens in a row (each continuing the state) equal
    one forced run of all 2510 tokens."""
    st0 = C.c1_state(c1_chip, 0)
    ids = _ids(2510, c1_chip.n_vocab, seed=5)
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, st0)
    got, a = [], 0
    for n in (1000, 7, 1, 2, 1500):
        p, _ = pf.run(ptrs, ids[a:a + n])
        got += p.cpu().numpy().tolist()
        a += n
    host = st0.copy()
    want, _, _ = Oracle(c1_chip).decode(host, ids, len(ids))
    assert got == want.tolist()
    _same(rec, conv, host)


def test_c1_chunk_8192_matches_oracle(c1_chip):
    """One config-3 chunk of 8,192 tokens (ids uniform over the vocabulary, seed 2)."""
    st0 = C.c1_state(c1_chip, 0)
    ids = _ids(8192, c1_chip.n_vocab)
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, st0)
    preds, _ = pf.run(ptrs, ids)
    host = st0.copy()
    want, _, _ = Oracle(c1_chip).decode(host, ids, len(ids))
    assert (preds.cpu().numpy() == want).all()
    _same(rec, conv, host)


def test_c1_matches_stock_chunked_prefill(c1_chip):
    """The reference's own chunked forward (two 256-token chunks, tests/golden/c1_prefill.npz):
    predictions and conv windows bit for bit, recurrent states within 1e-9."""
    g = np.load(GOLD / "c1_prefill.npz")
    assert str(g["digest"]) == c1_chip.digest()
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, C.c1_state(c1_chip, 0))
    for k in range(2):
        preds, _ = pf.run(ptrs, g[f"ids{k}"])
        assert (preds.cpu().numpy() == g[f"preds{k}"]).all()
        assert np.array_equal(conv.cpu().numpy().view(np.uint16), g[f"conv{k}"])
        assert np.abs(rec.cpu().numpy()[:, [5, 77]] - g[f"rec_heads{k}"]).max() <= TOL_REC


@pytest.mark.skipif(not (GOLD / "c1_prefill8k.npz").exists(), reason="fixture not generated")
def test_c1_8192_matches_stock_chunked_prefill(c1_chip):
    """The reference's own chunked forward on one 8,192-token chunk of config 3's ids
    (tests/golden/c1_prefill8k.npz): every prediction, the conv windows; states within 1e-9."""
    g = np.load(GOLD / "c1_prefill8k.npz")
    assert str(g["digest"]) == c1_chip.digest()
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, C.c1_state(c1_chip, 0))
    preds, _ = pf.run(ptrs, g["ids"])
    assert (preds.cpu().numpy() == g["preds"]).all()
    assert np.array_equal(conv.cpu().numpy().view(np.uint16), g["conv"])
    assert np.abs(rec.cpu().numpy()[:, [5, 77]] - g["rec_heads"]).max() <= TOL_REC


def test_self_consistent_trace_has_no_mismatch(c1_chip):
    """The greedy stream itself as the proposed trace (the all-correct case of verified mode):
    every prediction is the next token, the first mismatch is -1, and the state after the
    prefill equals the decode's."""
    from linuxformer_b200.runtime import Decoder

    st0 = C.c1_state(c1_chip, 0)
    dec = Decoder(c1_chip, cluster=16)
    ds = dec.states([st0])
    n = 1200
    preds, inputs = dec.run(ds, [[0]], n)
    trace = inputs[0].cpu().numpy()
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, st0)
    p2, first = pf.run(ptrs, trace, chunk=500)
    assert first == -1
    assert (p2.cpu().numpy() == preds[0].cpu().numpy()).all()
    got = ds.host(0)
    _same(rec, conv, got)


def test_c2_matches_oracle():
    """The 37-layer chip-shaped stack (a 20,000-row head: dense code columns; 16 live rows per
    key head; layers without an MLP; two decaying layers)."""
    chip = C.c2(1, vocab=20000)
    st0 = C.c2_state(chip, 1)
    ids = _ids(200, chip.n_vocab, seed=7)
    pf = _prefill(chip)
    rec, conv, ptrs = _states(chip, st0)
    preds, _ = pf.run(ptrs, ids, chunk=150)
    host = st0.copy()
    want, _, _ = Oracle(chip).decode(host, ids, len(ids))
    assert (preds.cpu().numpy() == want).all()
    _same(rec, conv, host)


def test_bad_token_sets_status(c1_chip):
    from linuxformer_b200._lib import LxbError

    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, C.c1_state(c1_chip, 0))
    with pytest.raises(LxbError, match="device status"):
        pf.run(ptrs, [0, 5, 4096, 3])
    p, _ = pf.run(ptrs, [1, 2])  # the plan stays usable
    assert p.shape == (2,)


def test_fast_dropin_on_the_references_model(c1_chip):
    """lx.fast.Fast's interface on the reference's own HF model and cache, as Session.verify
    calls it (embed, forward, head_argmax per chunk): the stock chunked forward's predictions
    (tests/golden/c1_prefill.npz); decode() of one token equals a chunk of one."""
    from transformers import DynamicCache

    from linuxformer_b200.prefill import Fast

    g = np.load(GOLD / "c1_prefill.npz")
    model = C.to_hf(c1_chip).to("cuda")
    st0 = C.c1_state(c1_chip, 0)
    cache = DynamicCache(config=model.config)
    for L in range(c1_chip.n_layers):
        cache.update_conv_state(torch.zeros((1, C.CONV, 4), dtype=torch.bfloat16, device="cuda"), L)
        lay = cache.layers[L]
        lay.recurrent_states = torch.from_numpy(st0.recurrent[L].copy())[None].to("cuda")
        lay.is_recurrent_states_initialized = True
    fast = Fast(model, c1_chip.n_layers)
    for k in range(2):
        ids = torch.from_numpy(g[f"ids{k}"]).to("cuda")
        e = model.model.embed_tokens(ids[None])
        pred = fast.head_argmax(fast.forward(e, cache)[0])
        assert pred.tolist() == g[f"preds{k}"].tolist()
    # one more token: decode (T = 1) against a fresh chunk of one on a copy of the state
    conv = [cache.layers[L].conv_states[0].clone() for L in range(c1_chip.n_layers)]
    rec = [cache.layers[L].recurrent_states[0].clone() for L in range(c1_chip.n_layers)]
    e = model.model.embed_tokens(torch.tensor([[11]], device="cuda"))
    h1 = fast.decode(e[0], cache)
    for L in range(c1_chip.n_layers):
        cache.layers[L].conv_states[0].copy_(conv[L])
        cache.layers[L].recurrent_states[0].copy_(rec[L])
    h2 = fast.forward(e, cache)[0]
    assert torch.equal(h1.view(torch.int16), h2.view(torch.int16))


def test_layers_and_head_calls_equal_the_fused_call(c1_chip):
    """lxb_prefill_layers (embedded rows in, rows out) followed by lxb_prefill_head gives what
    lxb_prefill gives on the token ids: the same predictions and the same state; the per-stage
    timing reports every stage of the chunk."""
    ids = _ids(777, c1_chip.n_vocab, seed=9)
    st0 = C.c1_state(c1_chip, 0)
    pf = _prefill(c1_chip)
    rec_a, conv_a, ptrs_a = _states(c1_chip, st0)
    pf.set_timing(True)
    pa, _ = pf.run(ptrs_a, ids)
    split = pf.timing()
    pf.set_timing(False)
    assert {"rows", "norm", "gates", "scan", "recur", "gnorm", "out", "mlp", "down", "head",
            "reduce"} <= set(split)
    assert split["recur"][1] == c1_chip.n_layers and split["norm"][1] == 2 * c1_chip.n_layers + 1
    rec_b, conv_b, ptrs_b = _states(c1_chip, st0)
    emb = pf.embed.view(torch.bfloat16)[torch.from_numpy(ids).long().to(pf.dev)].contiguous()
    h = pf.layers(ptrs_b, emb)
    pb = pf.head(h)
    torch.cuda.synchronize()
    assert torch.equal(pa, pb)
    assert torch.equal(conv_a, conv_b)
    assert torch.equal(rec_a.view(torch.int32), rec_b.view(torch.int32))


def test_c1_chunk_in_views_matches_the_forced_decode(c1_chip):
    """A chunk long enough to run as four views on four streams (16,384 tokens: 4 x 4,096), each
    view's state part chained to the previous one's, the decay scans ordered on the plan's second
    stream. The trace is the decode's own greedy stream with one token changed just after the
    first view boundary: the predictions and the final state equal the decode kernel's with every
    input forced (itself bit-identical to the CPU restatement), and the first mismatch is the
    position before the changed token, found across the views."""
    from linuxformer_b200.runtime import Decoder

    n = 16384
    st0 = C.c1_state(c1_chip, 0)
    dec = Decoder(c1_chip, cluster=16)
    _, inputs = dec.run(dec.states([st0]), [[0]], n)
    trace = inputs[0].cpu().numpy().copy()
    trace[4097] = (trace[4097] + 1) % c1_chip.n_vocab
    ds = dec.states([st0])
    want, _ = dec.run(ds, [trace.tolist()], n)
    pf = _prefill(c1_chip)
    rec, conv, ptrs = _states(c1_chip, st0)
    preds, first = pf.run(ptrs, trace)
    assert (preds.cpu().numpy() == want[0].cpu().numpy()).all()
    assert first == 4096
    _same(rec, conv, ds.host(0))


def test_fast_runs_unsupported_circuits_through_the_decode_kernel():
    """A circuit the prefill kernels do not take (here config 1 with 40 tapped query rows in one
    key head; the real circuit's memory heads have 256): Fast runs it through the decode kernel,
    every input forced, so Session.verify's calls still work. Predictions, conv windows and
    recurrent states equal the CPU restatement's forced decode bit for bit; head_argmax takes
    only the rows forward returned."""
    from transformers import DynamicCache

    from linuxformer_b200._lib import LxbError
    from linuxformer_b200.prefill import Fast

    chip = C.c1(0)
    ly = chip.layers[0]
    ly.conv = ly.conv.copy()
    ly.conv[:40, 3] = C.bf16_bits(np.float32(0.5))
    model = C.to_hf(chip).to("cuda")
    st0 = C.c1_state(chip, 0)
    cache = DynamicCache(config=model.config)
    for L in range(chip.n_layers):
        cache.update_conv_state(torch.zeros((1, C.CONV, 4), dtype=torch.bfloat16, device="cuda"), L)
        lay = cache.layers[L]
        lay.recurrent_states = torch.from_numpy(st0.recurrent[L].copy())[None].to("cuda")
        lay.is_recurrent_states_initialized = True
    fast = Fast(model, chip.n_layers)
    assert fast.pf is None and "live rows" in fast.unsupported
    ids = np.random.default_rng(5).integers(0, chip.n_vocab, 96).astype(np.int32)
    got = []
    for a in (0, 64):  # two chunks, the state carried in the cache
        e = model.model.embed_tokens(torch.from_numpy(ids[a:a + 64]).long().to("cuda")[None])
        h = fast.forward(e, cache)[0]
        got += fast.head_argmax(h).tolist()
        with pytest.raises(LxbError):
            fast.head_argmax(e[0])
    host = st0.copy()
    want, _, _ = Oracle(chip).decode(host, ids, len(ids))
    assert got == want.tolist()
    for L in range(chip.n_layers):
        conv = cache.layers[L].conv_states[0].view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(conv, host.conv[L])
        assert not (cache.layers[L].recurrent_states[0].cpu().numpy() != host.recurrent[L]).any()
