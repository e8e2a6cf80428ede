"""Golden vectors from the reference's own stock forward, run on CPU in the build container.

The reference's decode and verify paths call ``lx.hf.chip_forward`` (the stock
``Qwen3_5DecoderLayer`` modules, layer by layer) and ``lx.hf.head_argmax``
(lx/lx/hf.py:169-184; lx/lx/session.py:95-100, 140-146). Without fla/causal_conv1d (the CPU case)
transformers runs its torch paths: ``torch_causal_conv1d_update``, ``torch_recurrent_gated_delta_rule``
(decode) and ``torch_chunk_gated_delta_rule`` (prefill). This script imports the reference from
its checkout, builds the seeded config-1 stack as a stock model, seeds fp32 recurrent states as
``Fast.init_cache`` does (lx/lx/fast.py:420-430), and records:

- ``c1_decode.npz``: 512 greedy tokens from token 0 (the reference's model-alone decode, one
  token per call as ``Session.step`` runs it), each step's top-2 bf16 logit margin, the final conv
  windows, per-value-head checksums of the final recurrent states plus two full value heads, and
  the residual after the chip layers for the first 8 steps;
- ``c1_prefill.npz``: two 256-token chunks of seeded random ids run as chunked prefill (the
  verified mode), the argmax at every position, the same state summaries after each chunk;
- ``c1_prefill8k.npz``: one 8,192-token chunk of config 3's ids (uniform over the vocabulary,
  seed 2) run as chunked prefill from the seeded state: the argmax and its top-2 margin at every
  position, the final conv windows and state summaries;
- ``c5_pad.npz``: config 5's Gated DeltaNet padding by the reference's own ``merge.pad_gdn``
  (lx/lx/merge.py:82-120) applied to Qwen-shaped weights whose entries encode their own row (or
  column): for every padded tensor, the Qwen row each padded row came from (-1: zero padding);
- ``c2_decode.npz``: config 2 (the 37-layer chip-shaped stack, the full 459,982-row head, the
  seeded RAM/ROM state) decoded greedily for 32 tokens from token 0 by the stock forward, one
  token per call: the tokens, each step's top-2 margin, the final conv windows (all layers),
  SHA-256 digests of every layer's conv windows and recurrent state (bits, -0 written as +0),
  per-(layer, value head) sums and absolute sums of the final recurrent state, and the whole
  final state of two memory value heads;
- ``real_decode.npz``: the real compiled circuit (``real_chip.npz``) decoded by the stock forward
  from GO for 32 tokens, one per call (the predictions must be the reference machine's trace):
  the tokens, their top-2 margins, the same per-layer digests and per-head sums.

Run where the reference's checkout is (its directory in LXB_REFERENCE); the tests only read the
.npz files:

    LXB_REFERENCE=<checkout> python tests/golden/make_golden.py [decode] [prefill] [prefill8k] [c2]
        [c5pad] [real]
"""

import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
REF = os.environ.get("LXB_REFERENCE")

from linuxformer_b200 import chip as C  # noqa: E402

N_DEC = 512
PRE_T = 256
PRE_8K = 8192


def new_cache(model, st: C.State):
    from transformers import DynamicCache

    cache = DynamicCache(config=model.config)
    for L in range(st.recurrent.shape[0]):
        conv = torch.from_numpy(st.conv[L].view(np.int16).copy()).view(torch.bfloat16)[None]
        cache.update_conv_state(conv, L)
        lay = cache.layers[L]
        # fp32 recurrent state (this transformers' lazy init would make it bf16)
        lay.recurrent_states = torch.from_numpy(st.recurrent[L].copy())[None]
        lay.is_recurrent_states_initialized = True
    return cache


def summarize(cache, n_layers):
    conv = np.stack([cache.layers[L].conv_states[0].view(torch.int16).numpy().view(np.uint16)
                     for L in range(n_layers)])
    rec = np.stack([cache.layers[L].recurrent_states[0].float().numpy() for L in range(n_layers)])
    sums = rec.astype(np.float64).sum(axis=(2, 3))           # [L, NV]
    abss = np.abs(rec.astype(np.float64)).sum(axis=(2, 3))
    heads = rec[:, [5, 77]]                                   # two full value heads per layer
    return conv, sums, abss, heads


def margins(logits: torch.Tensor) -> np.ndarray:
    top = torch.topk(logits.float(), 2, dim=-1).values
    return (top[..., 0] - top[..., 1]).numpy()


@torch.no_grad()
def main(parts):
    if not REF:
        sys.exit("set LXB_REFERENCE to the reference checkout's directory")
    sys.path.insert(0, REF + "/lx")
    from lx import hf as ref_hf  # the reference's stock forward

    torch.manual_seed(0)
    torch.set_num_threads(os.cpu_count())
    if "c5pad" in parts:
        c5_pad()
    if "c2" in parts:
        c2_decode(ref_hf)
    if "real" in parts:
        real_decode(ref_hf)
    if not {"decode", "prefill", "prefill8k"} & set(parts):
        return
    chip = C.c1(0)
    model = C.to_hf(chip)
    st0 = C.c1_state(chip, 0)
    n = chip.n_layers
    emb = model.model.embed_tokens
    if "decode" in parts:
        decode(ref_hf, chip, model, st0, n, emb)
    if "prefill" in parts:
        prefill(ref_hf, chip, model, st0, n, emb)
    if "prefill8k" in parts:
        prefill8k(ref_hf, chip, model, st0, n, emb)


def decode(ref_hf, chip, model, st0, n, emb):
    # --- model-alone decode --------------------------------------------------------------
    cache = new_cache(model, st0)
    tok, toks, preds, marg, resid = 0, [], [], [], []
    t0 = time.time()
    for i in range(N_DEC):
        h = ref_hf.chip_forward(model, emb(torch.tensor([[tok]])), cache, n)[0]
        logits = torch.nn.functional.linear(model.model.norm(h), model.lm_head.weight)
        p = int(ref_hf.head_argmax(model, h)[0])
        assert p == int(logits.argmax(-1)[0])
        toks.append(tok)
        preds.append(p)
        marg.append(float(margins(logits)[0]))
        if i < 8:
            resid.append(h[0].view(torch.int16).numpy().view(np.uint16).copy())
        tok = p
    dt = time.time() - t0
    conv, sums, abss, heads = summarize(cache, n)
    np.savez_compressed(HERE / "c1_decode.npz", digest=chip.digest(), inputs=np.array(toks),
                        preds=np.array(preds), margin=np.array(marg, np.float32),
                        resid=np.stack(resid), conv=conv, rec_sum=sums, rec_abs=abss,
                        rec_heads=heads, cpu_s=dt)
    print(f"decode: {N_DEC} tokens in {dt:.1f}s, min margin {min(marg):.3g}")


def prefill(ref_hf, chip, model, st0, n, emb):
    # --- verified-mode prefill (chunked) -------------------------------------------------
    cache = new_cache(model, st0)
    rng = np.random.default_rng(2)
    out = {}
    for c in range(2):
        ids = rng.integers(0, chip.n_vocab, PRE_T)
        t0 = time.time()
        h = ref_hf.chip_forward(model, emb(torch.from_numpy(ids)[None]), cache, n)[0]
        logits = torch.nn.functional.linear(model.model.norm(h), model.lm_head.weight)
        p = ref_hf.head_argmax(model, h).numpy()
        dt = time.time() - t0
        conv, sums, abss, heads = summarize(cache, n)
        out.update({f"ids{c}": ids, f"preds{c}": p, f"margin{c}": margins(logits),
                    f"conv{c}": conv, f"rec_sum{c}": sums, f"rec_abs{c}": abss,
                    f"rec_heads{c}": heads, f"cpu_s{c}": dt})
        print(f"prefill chunk {c}: {PRE_T} tokens in {dt:.1f}s")
    np.savez_compressed(HERE / "c1_prefill.npz", digest=chip.digest(), **out)


def prefill8k(ref_hf, chip, model, st0, n, emb):
    # --- one config-3 chunk: 8,192 ids uniform over the vocabulary (seed 2) --------------
    ids = np.random.default_rng(2).integers(0, chip.n_vocab, PRE_8K)
    cache = new_cache(model, st0)
    t0 = time.time()
    h = ref_hf.chip_forward(model, emb(torch.from_numpy(ids)[None]), cache, n)[0]
    p = ref_hf.head_argmax(model, h).numpy()
    logits = torch.cat([torch.nn.functional.linear(model.model.norm(h[a:a + 1024]),
                                                   model.lm_head.weight)
                        for a in range(0, PRE_8K, 1024)])
    dt = time.time() - t0
    conv, sums, abss, heads = summarize(cache, n)
    np.savez_compressed(HERE / "c1_prefill8k.npz", digest=chip.digest(), ids=ids, preds=p,
                        margin=margins(logits), conv=conv, rec_sum=sums, rec_abs=abss,
                        rec_heads=heads, cpu_s=dt)
    print(f"prefill 8k: {PRE_8K} tokens in {dt:.1f}s")


N_C2 = 32
N_REAL = 32


def c2_heads(chip):
    """Two memory value heads (layer, value head) whose whole final state the fixture keeps:
    the first memory key head's first value head, and a later layer's fifth."""
    mem = chip.meta["memory_heads"]
    (l0, k0), (l1, k1) = mem[0], mem[len(mem) // 2]
    return ((l0, k0 * 8), (l1, k1 * 8 + 5))


def c2_digests(conv, rec):
    """SHA-256 per layer of the conv windows' and the recurrent state's bits, with -0 written as
    +0 (the stock forward and the sparse path may differ in a zero's sign only: a product with a
    zero weight or input that the sparse path never forms)."""
    import hashlib

    cv = np.where((conv & 0x7FFF) == 0, 0, conv).astype(np.uint16)
    rv = np.where(rec == 0, np.float32(0), rec).astype(np.float32)
    cd = [hashlib.sha256(np.ascontiguousarray(cv[L]).tobytes()).hexdigest()
          for L in range(conv.shape[0])]
    rd = [hashlib.sha256(np.ascontiguousarray(rv[L]).view(np.uint32).tobytes()).hexdigest()
          for L in range(rec.shape[0])]
    return np.array(cd), np.array(rd)


def c2_decode(ref_hf):
    # --- config 2: the 37-layer stack with its full head, one token per call -------------
    chip = C.c2(1)
    st0 = C.c2_state(chip, 1)
    t0 = time.time()
    model = C.to_hf(chip)
    print(f"c2 stock model built in {time.time() - t0:.0f}s")
    n = chip.n_layers
    emb = model.model.embed_tokens
    cache = new_cache(model, st0)
    tok, toks, preds, marg = 0, [], [], []
    t0 = time.time()
    for i in range(N_C2):
        h = ref_hf.chip_forward(model, emb(torch.tensor([[tok]])), cache, n)[0]
        logits = torch.nn.functional.linear(model.model.norm(h), model.lm_head.weight)
        p = int(ref_hf.head_argmax(model, h)[0])
        assert p == int(logits.argmax(-1)[0])
        toks.append(tok)
        preds.append(p)
        marg.append(float(margins(logits)[0]))
        tok = p
    dt = time.time() - t0
    conv = np.stack([cache.layers[L].conv_states[0].view(torch.int16).numpy().view(np.uint16)
                     for L in range(n)])
    rec = np.stack([cache.layers[L].recurrent_states[0].float().numpy() for L in range(n)])
    cd, rd = c2_digests(conv, rec)
    hid = c2_heads(chip)
    np.savez_compressed(HERE / "c2_decode.npz", digest=chip.digest(), inputs=np.array(toks),
                        preds=np.array(preds), margin=np.array(marg, np.float32),
                        conv=conv, conv_sha=cd, rec_sha=rd,
                        rec_vh_sum=rec.astype(np.float64).sum(axis=(2, 3)),
                        rec_vh_abs=np.abs(rec.astype(np.float64)).sum(axis=(2, 3)),
                        heads=np.stack([rec[L, vh] for L, vh in hid]), head_ids=np.array(hid),
                        cpu_s=dt)
    print(f"c2 decode: {N_C2} tokens in {dt:.1f}s, min margin {min(marg):.3g}")


def real_decode(ref_hf):
    # --- the real compiled circuit (real_chip.npz): the model alone from GO, one per call ----
    chip = C.real()
    st0 = C.real_state(chip)
    tr = chip.meta["fixture"]["trace"]
    t0 = time.time()
    import dataclasses

    # the stock model's vocabulary is the head's rows (the embedding's padding rows past them,
    # PAD among them, are never an input)
    model = C.to_hf(dataclasses.replace(chip, embed=chip.embed[:chip.n_vocab]))
    print(f"real stock model built in {time.time() - t0:.0f}s")
    n = chip.n_layers
    emb = model.model.embed_tokens
    cache = new_cache(model, st0)
    tok, toks, preds, marg = int(tr[0]), [], [], []
    t0 = time.time()
    for i in range(N_REAL):
        h = ref_hf.chip_forward(model, emb(torch.tensor([[tok]])), cache, n)[0]
        logits = torch.nn.functional.linear(model.model.norm(h), model.lm_head.weight)
        p = int(ref_hf.head_argmax(model, h)[0])
        assert p == int(logits.argmax(-1)[0])
        toks.append(tok)
        preds.append(p)
        marg.append(float(margins(logits)[0]))
        tok = p
    dt = time.time() - t0
    assert preds == tr[1:N_REAL + 1].tolist(), "the stock forward left the machine's trace"
    conv = np.stack([cache.layers[L].conv_states[0].view(torch.int16).numpy().view(np.uint16)
                     for L in range(n)])
    rec = np.stack([cache.layers[L].recurrent_states[0].float().numpy() for L in range(n)])
    cd, rd = c2_digests(conv, rec)
    np.savez_compressed(HERE / "real_decode.npz", inputs=np.array(toks), preds=np.array(preds),
                        margin=np.array(marg, np.float32), conv_sha=cd, rec_sha=rd,
                        rec_vh_sum=rec.astype(np.float64).sum(axis=(2, 3)),
                        rec_vh_abs=np.abs(rec.astype(np.float64)).sum(axis=(2, 3)), cpu_s=dt)
    print(f"real decode: {N_REAL} tokens in {dt:.1f}s, min margin {min(marg):.3g}")


def c5_pad():
    from lx import merge as ref_merge

    q = {"linear_num_key_heads": 16, "linear_key_head_dim": 128, "linear_num_value_heads": 32,
         "linear_value_head_dim": 128}
    hdim = 4  # the hidden size does not enter the padding

    def rows(n, cols):  # every entry of row i is i + 1 (exact in fp32)
        return (torch.arange(n, dtype=torch.float32) + 1)[:, None].expand(n, cols).contiguous()

    w = {"in_proj_qkv.weight": rows(8192, hdim), "conv1d.weight": rows(8192, 4).view(8192, 1, 4),
         "in_proj_z.weight": rows(4096, hdim), "in_proj_b.weight": rows(32, hdim),
         "in_proj_a.weight": rows(32, hdim), "dt_bias": torch.arange(32.0) + 1,
         "A_log": torch.arange(32.0) + 1, "norm.weight": torch.ones(128),
         "out_proj.weight": rows(4096, hdim).t().contiguous()}
    out = ref_merge.pad_gdn(w, q, nk=16, dk=256, nv=128, dv=128)

    def src(t):
        return (t[:, 0] if t.dim() > 1 else t).to(torch.int64).numpy() - 1

    np.savez_compressed(
        HERE / "c5_pad.npz",
        qkv=src(out["in_proj_qkv.weight"]), conv=src(out["conv1d.weight"].reshape(-1, 4)),
        z=src(out["in_proj_z.weight"]), b=src(out["in_proj_b.weight"]),
        a=src(out["in_proj_a.weight"]), dt_bias=src(out["dt_bias"]), A_log=src(out["A_log"]),
        out=src(out["out_proj.weight"].t()))
    print("c5 pad: written")


if __name__ == "__main__":
    main(sys.argv[1:] or ["decode", "prefill", "prefill8k", "c2", "c5pad", "real"])
