"""TEST INFRASTRUCTURE ONLY: the reference's text path for config 5, used by the text decode's
parity tests and by bench.py's CPU baseline and reference arm (never by the product path).

The reference runs text through the stock HF forward of a Qwen3_5ForCausalLM
(``merge.text_view``, then ``generate``: lx/lx/merge.py:251-280, lx/lx/chat.py:62-73). Here the
same stock modules run token by token with a DynamicCache whose GDN layers start from zero fp32
states (the recurrent path from the first token, as ``Fast.init_cache`` seeds the chip's,
lx/lx/fast.py:420-430) and with transformers' torch GDN functions (no fla / causal_conv1d
kernels), so the comparison is with the stock decode step itself:

    cache = zero_cache(model)
    hidden, logits = steps(model, ids, cache)     # the final norm's output and the logits per step
"""

from __future__ import annotations

import torch


def zero_cache(model):
    from transformers import DynamicCache

    cfg = model.config
    dev = model.model.embed_tokens.weight.device
    cache = DynamicCache(config=cfg)
    nk, kd = cfg.linear_num_key_heads, cfg.linear_key_head_dim
    nv, vd = cfg.linear_num_value_heads, cfg.linear_value_head_dim
    conv = 2 * nk * kd + nv * vd
    for L, t in enumerate(cfg.layer_types):
        if t != "linear_attention":
            continue
        cache.update_conv_state(torch.zeros(1, conv, cfg.linear_conv_kernel_dim,
                                            dtype=torch.bfloat16, device=dev), L)
        lay = cache.layers[L]
        lay.recurrent_states = torch.zeros(1, nv, kd, vd, dtype=torch.float32, device=dev)
        lay.is_recurrent_states_initialized = True
    return cache


@torch.no_grad()
def steps(model, ids, cache, logits: bool = True):
    """Feed ``ids`` one at a time; returns the final norm's output [n, hidden] (fp32) and, with
    ``logits``, the head's bf16 logits as fp32 [n, vocab]."""
    dev = model.model.embed_tokens.weight.device
    ids = torch.as_tensor(ids, dtype=torch.long, device=dev).reshape(-1)
    hs, lg = [], []
    for i in range(len(ids)):
        h = model.model(input_ids=ids[None, i:i + 1], past_key_values=cache,
                        use_cache=True).last_hidden_state[0, -1]
        hs.append(h.float())
        if logits:
            lg.append(model.lm_head(h).float())
    return torch.stack(hs), (torch.stack(lg) if logits else None)


@torch.no_grad()
def cpu_copy(model, threads: int | None = None):
    """The same model on the host (weights copied from the device), for the CPU baseline."""
    import os

    from transformers import Qwen3_5ForCausalLM

    torch.set_num_threads(threads or len(os.sched_getaffinity(0)))
    with torch.device("meta"):
        m = Qwen3_5ForCausalLM(model.config).to(torch.bfloat16)
    m = m.to_empty(device="cpu")
    m.tie_weights()
    src = dict(model.named_parameters(remove_duplicate=False))
    for name, p in m.named_parameters():  # a tied parameter once, under its first name
        p.data.copy_(src[name].data.to(p.dtype), non_blocking=False)
    m.model.rotary_emb = type(model.model.rotary_emb)(config=model.config)
    from linuxformer_b200.text import force_torch_paths

    force_torch_paths(m)
    return m.eval()
