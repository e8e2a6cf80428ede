"""The reference's model-alone decoder interface, on the B200 kernels.

A drop-in for ``lx.mega.Mega`` (lx/lx/mega.py:198-574): the same constructor and ``run`` call,
the same cache tensors updated in place, the same returned predictions. ``Linux.boot_alone``
(lx/lx/linux.py:209-227), ``lx.chat --alone`` and ``tools/mega_boot.py`` switch to it by
importing this class instead:

    from linuxformer_b200.mega import Mega
    m = Mega(fast, model, cache, offset)
    preds = m.run(forced, n)       # n steps: inputs forced[0..], then each step's prediction

What the reference's host packs per launch (CSR/CSC tables, per-CTA blobs, a phase schedule)
this class builds once, through linuxformer_b200.tables, from the model's chip layers; the
decode itself is liblxb.so's (include/lxb.h). There is no CPU fallback: without a CUDA device
or the built library the constructor raises.
"""

from __future__ import annotations

import numpy as np
import torch

from . import chip as C
from ._lib import S_ERRORS
from .runtime import Decoder, state_pointers


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.bfloat16).contiguous().view(torch.int16).cpu().numpy().view(
        np.uint16)


def _sparse(w: torch.Tensor) -> C.Sparse:
    """A dense bf16 weight's nonzeros as CSR (rows, ascending columns), without densifying on
    the host twice."""
    w = w.detach()
    nz = (w != 0).nonzero()
    rows, cols = nz[:, 0], nz[:, 1]
    vals = w[rows, cols]
    return C.Sparse.from_coo(tuple(w.shape), rows.cpu().numpy(), cols.cpu().numpy(), _bits(vals))


def chip_from_model(model, n_chip: int, rows: slice | None = None, offset: int = 0) -> C.Chip:
    """The chip layers of a stock Qwen3_5ForCausalLM (the reference's chip-only or merged
    model) as a linuxformer_b200 Chip: every projection's nonzeros, the conv taps, the per-head
    parameters, the norms, the embedding and the head rows (``rows``: the chip vocabulary's
    slice of the merged model's head, as Session passes it, lx/lx/session.py:65)."""
    layers = []
    for L in range(n_chip):
        ly = model.model.layers[L]
        ga = ly.linear_attn
        assert ga.head_k_dim == C.KD and ga.head_v_dim == C.VD and ga.num_k_heads == C.NK \
            and ga.num_v_heads == C.NV and ga.conv_kernel_size == C.TAPS, "not the chip shape"
        layers.append(C.Layer(
            qkv=_sparse(ga.in_proj_qkv.weight), conv=_bits(ga.conv1d.weight[:, 0, :]),
            z=_sparse(ga.in_proj_z.weight), b=_sparse(ga.in_proj_b.weight),
            a=_sparse(ga.in_proj_a.weight), out=_sparse(ga.out_proj.weight),
            A_log=_bits(ga.A_log), dt_bias=_bits(ga.dt_bias), gnorm=_bits(ga.norm.weight),
            ln_in=_bits(ly.input_layernorm.weight), ln_post=_bits(ly.post_attention_layernorm.weight),
            gate=_sparse(ly.mlp.gate_proj.weight), up=_sparse(ly.mlp.up_proj.weight),
            down=_sparse(ly.mlp.down_proj.weight)))
    head = model.lm_head.weight if rows is None else model.lm_head.weight[rows]
    emb = model.model.embed_tokens.weight
    assert emb.shape[1] == C.H
    return C.Chip(name="model", layers=layers, embed=_bits(emb),
                  head=_sparse(head), final_norm=_bits(model.model.norm.weight),
                  eps=float(model.config.rms_norm_eps), offset=offset)


class Mega:
    """lx.mega.Mega's interface (lx/lx/mega.py:198-574) on liblxb.so."""

    def __init__(self, fast, model, cache, offset: int, ncta: int | None = None,
                 subprof: bool = False, spec: bool = True, pair_layers=None) -> None:
        n_chip = fast.n_chip
        rows = slice(offset, offset + fast.w_head.shape[0]) if offset else None
        dev = next(model.parameters()).device
        chip = chip_from_model(model, n_chip, rows, offset)
        emb = model.model.embed_tokens.weight
        assert emb.dtype == torch.bfloat16 and emb.is_contiguous()
        chip.embed = chip.embed[:, :0]  # the kernel reads the model's own embedding (its rows count)
        self.dec = Decoder(chip, cluster=ncta or 16, device=dev, embed=emb.view(torch.int16))
        self.dev, self.fast, self.model, self.cache, self.offset = dev, fast, model, cache, offset
        self.n_chip = n_chip
        self.stats = dict(self.dec.stats, smem=self.dec.staging()["smem_bytes"])
        self.bitmaps = torch.zeros((1, n_chip, C.NV, 8), dtype=torch.int32, device=dev)
        self.scratch = self.dec.scratch(1)
        self.prof = None

    def _state_ptrs(self) -> torch.Tensor:
        rs, cs = [], []
        for L in range(self.n_chip):
            cl = self.cache.layers[L]
            r, c = cl.recurrent_states[0], cl.conv_states[0]
            assert r.is_contiguous() and c.is_contiguous() and r.dtype == torch.float32
            assert c.dtype == torch.bfloat16 and c.shape[-1] == C.TAPS
            rs.append(r)
            cs.append(c)
        return state_pointers([rs], [cs], self.dev)

    def sync_bitmaps(self) -> None:
        """The nonzero-row bitmaps are rebuilt from the states on every run (in the kernel)."""

    @torch.no_grad()
    def run(self, forced: list[int], n: int, dbg=None, dbg_tok: int = 0, dbg_items=None,
            prof: torch.Tensor | None = None, inputs: torch.Tensor | None = None) -> list[int]:
        """n steps; step i's input is forced[i] (i < len(forced)) or step i - 1's prediction.
        Returns the n predictions (chip token ids); ``inputs`` (n,) int32 receives each step's
        input as embedded; ``prof`` (int64 [cluster, sections]) accumulates the per-section
        cycle counters (the reference's per-phase counters)."""
        assert len(forced) >= 1
        if dbg is not None or dbg_items is not None:
            raise NotImplementedError("per-phase residual dumps: use the oracle (oracle/)")
        f = torch.tensor([forced], dtype=torch.int32, device=self.dev)
        preds = torch.empty((1, n), dtype=torch.int32, device=self.dev)
        inp = inputs[:n].view(1, n) if inputs is not None else None
        if prof is not None:
            self.dec.set_profile(prof.view(1, *prof.shape[-2:]))
        try:
            self.dec.launch(self._state_ptrs(), self.bitmaps, f, n, preds, inp,
                            sync_bitmaps=True, scratch=self.scratch)
            out = preds[0].tolist()  # syncs
        finally:
            if prof is not None:
                self.dec.set_profile(None)
        e = self.dec.status()
        if e.status & S_ERRORS:
            raise RuntimeError(f"mega failed: device status {e.status:#x} at step {e.first_step}")
        return out
