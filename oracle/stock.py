"""TEST INFRASTRUCTURE ONLY: the reference's stock forward on the CPU, used by bench.py's CPU
baseline and reference arm (and nothing in the product path).

The reference's CPU path for the chip layers is its stock forward: ``lx.hf.chip_forward`` calls
the model's ``Qwen3_5DecoderLayer`` modules one after another (lx/lx/hf.py:169-176) and
``lx.hf.head_argmax`` takes the first argmax of the tied head over the final norm
(lx/lx/hf.py:179-184). Without fla and causal_conv1d (the CPU case) transformers runs its torch
functions for the GDN: torch_causal_conv1d_update and torch_recurrent_gated_delta_rule for one
token, F.conv1d and torch_chunk_gated_delta_rule for a chunk (modeling_qwen3_5.py in transformers
5.5.0; the reference pins 5.19.0). This module restates those two loops over the same modules,
with the torch functions forced (should fla import on the machine, its GPU kernels must not be
called on CPU tensors) and fp32 recurrent states seeded as ``Fast.init_cache`` seeds them
(lx/lx/fast.py:420-430).

    m = StockCPU(chip)                       # the chip as a stock bf16 model on the CPU
    cache = m.cache(state)                   # a DynamicCache from a chip.State
    preds = m.decode(cache, first_token, n)  # greedy, one token per call (Session.step)
    preds = m.prefill(cache, ids)            # one chunk (Session.verify's stock branch)

In transformers 5.5.0 a multi-token forward starts from a zero recurrent state and a zero conv
window (``initial_state=None``, ``F.pad`` of the chunk's inputs), so ``prefill`` measures the
stock chunked forward's cost, not a state carried across chunks.
"""

from __future__ import annotations

import os

import numpy as np
import torch


def _force_torch_paths(model) -> None:
    import transformers.models.qwen3_5.modeling_qwen3_5 as M

    for layer in model.model.layers:
        ga = getattr(layer, "linear_attn", None)
        if ga is None:
            continue
        ga.causal_conv1d_fn = None
        ga.causal_conv1d_update = M.torch_causal_conv1d_update
        ga.chunk_gated_delta_rule = M.torch_chunk_gated_delta_rule
        ga.recurrent_gated_delta_rule = M.torch_recurrent_gated_delta_rule
        if not isinstance(ga.norm, M.Qwen3_5RMSNormGated):
            w = ga.norm.weight.detach().clone()
            ga.norm = M.Qwen3_5RMSNormGated(ga.head_v_dim, eps=ga.layer_norm_epsilon)
            ga.norm.weight.data.copy_(w)


class StockCPU:
    def __init__(self, chip, threads: int | None = None) -> None:
        from linuxformer_b200 import chip as C

        self.threads = threads or len(os.sched_getaffinity(0))
        torch.set_num_threads(self.threads)
        self.chip = chip
        self.model = C.to_hf(chip)
        _force_torch_paths(self.model)
        self.n = chip.n_layers

    def cache(self, st):
        from transformers import DynamicCache

        cache = DynamicCache(config=self.model.config)
        for L in range(self.n):
            conv = torch.from_numpy(st.conv[L].view(np.int16).copy()).view(torch.bfloat16)[None]
            cache.update_conv_state(conv, L)
            lay = cache.layers[L]
            lay.recurrent_states = torch.from_numpy(st.recurrent[L].copy())[None]
            lay.is_recurrent_states_initialized = True
        return cache

    @torch.no_grad()
    def _layers(self, h, cache):
        for layer in self.model.model.layers[:self.n]:
            h = layer(h, position_embeddings=None, attention_mask=None, position_ids=None,
                      past_key_values=cache)
        return h

    @torch.no_grad()
    def _head(self, h, block: int = 2048):
        w = self.model.lm_head.weight
        return torch.cat([torch.nn.functional.linear(self.model.model.norm(h[a:a + block]),
                                                     w).argmax(-1)
                          for a in range(0, h.shape[0], block)])

    @torch.no_grad()
    def decode(self, cache, first: int, n: int) -> np.ndarray:
        emb = self.model.model.embed_tokens
        tok, out = int(first), []
        for _ in range(n):
            h = self._layers(emb(torch.tensor([[tok]])), cache)[0]
            tok = int(self._head(h)[0])
            out.append(tok)
        return np.array(out, np.int32)

    @torch.no_grad()
    def prefill(self, cache, ids) -> np.ndarray:
        emb = self.model.model.embed_tokens
        h = self._layers(emb(torch.as_tensor(np.asarray(ids, np.int64))[None]), cache)[0]
        return self._head(h).numpy().astype(np.int32)
