"""Config 5: the Qwen3.5-4B-shaped text path, its Gated DeltaNet layers zero-padded to the chip
shape, decoded at batch 1 by one persistent kernel (csrc/text.cu).

The reference merges the chip layers into Qwen3.5-4B and pads Qwen's GDN weights to the chip's
shape (lx/lx/merge.py:82-120, ``pad_gdn``; config in lx/lx/hf.py:25-38 and merge.py:160-185):
key dim 128 -> 256 and 32 -> 128 value heads, Qwen's value head h (of key head h // 2) becoming
value head (h // 2) * 8 + h % 2, and ``rms_norm_eps`` scaled by 128 / 256 (5e-7). Its text then
runs through the stock HF forward. This module builds that model shape with random weights
(``random_model``), packs the non-padding parts of a model's weights for the kernel
(``pack``), and decodes with ``TextDecoder``, which skips the padding structurally: zero rows and
columns of the padded projections are never read, and the padded value heads (zero value, zero
z, zero out_proj columns, zero initial state) are never touched, since their state stays zero
and their output is exactly 0.

    model = random_model(seed=4)                  # stock Qwen3_5ForCausalLM, bf16, on cuda
    dec = TextDecoder(model, max_pos=4608)        # packs the weights, owns the caches
    preds = dec.run(prompt_ids, n_new)            # prompt forced, then greedy; predictions

Shapes (Qwen3.5-4B text config): 32 layers, three GDN layers then one gated full-attention layer
(16 query heads, 4 key/value heads, head dim 256, partial rotary 0.25, output gate), hidden
2560, SwiGLU 9216, vocabulary 248,320 with the head tied to the embedding.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

H = 2560
N_LAYERS = 32
VOCAB = 248320
INTER = 9216
# Qwen3.5-4B's own GDN shape, and the chip shape it is padded to
QNK, QKD, QNV, QVD = 16, 128, 32, 128
NK, KD, NV, VD = 16, 256, 128, 128
QR, PR = QNV // QNK, NV // NK          # value heads per key head: 2 (Qwen), 8 (padded)
CONV = 2 * NK * KD + NV * VD           # 24,576 padded conv channels
# gated full attention
NQ, NKV, HD = 16, 4, 256
ROT = HD // 4                          # partial_rotary_factor 0.25
THETA = 10_000_000
EPS = 1e-6 * QKD / KD                  # 5e-7, as the reference scales it for the padded key dim
STD = 0.02
W1_GDN = 2 * QNK * QKD + QNV * QVD + QNV * QVD + 2 * QNV   # q, k, v, z, b, a rows: 12,352
W1_ATT = NQ * 2 * HD + 2 * NKV * HD                        # q (+ gate), k, v rows: 10,240


def layer_types(n_layers: int = N_LAYERS) -> list[str]:
    """Qwen3.5-4B's pattern: every fourth layer is full attention."""
    return ["full_attention" if i % 4 == 3 else "linear_attention" for i in range(n_layers)]


def hf_config(n_layers: int = N_LAYERS, vocab: int = VOCAB):
    from transformers import Qwen3_5TextConfig

    cfg = Qwen3_5TextConfig(
        hidden_size=H, num_hidden_layers=n_layers, layer_types=layer_types(n_layers),
        vocab_size=vocab, intermediate_size=INTER, hidden_act="silu",
        linear_key_head_dim=KD, linear_value_head_dim=VD, linear_num_key_heads=NK,
        linear_num_value_heads=NV, linear_conv_kernel_dim=4,
        num_attention_heads=NQ, num_key_value_heads=NKV, head_dim=HD, attn_output_gate=True,
        rope_parameters={"rope_type": "default", "rope_theta": THETA,
                         "partial_rotary_factor": ROT / HD, "mrope_section": [11, 11, 10],
                         "mrope_interleaved": True},
        max_position_embeddings=262144, rms_norm_eps=EPS, tie_word_embeddings=True,
        attention_bias=False)
    cfg._attn_implementation = "sdpa"
    return cfg


def pad_maps():
    """The padded model's row indices of Qwen's GDN rows (the padding rule of
    lx/lx/merge.py:82-120, restated): ``rows`` the conv / in_proj_qkv channels of Qwen's q, k
    (key-head major) and v channels; ``vrows`` the value dims (in_proj_z rows, out_proj
    columns); ``heads`` the value heads (in_proj_b / in_proj_a rows, A_log, dt_bias)."""
    vmap = [(h // QR) * PR + h % QR for h in range(QNV)]
    qk = [j * KD + i for j in range(NK) for i in range(QKD)]
    rows = qk + [NK * KD + x for x in qk] + [2 * NK * KD + vh * VD + i for vh in vmap
                                             for i in range(VD)]
    vrows = [vh * VD + i for vh in vmap for i in range(VD)]
    return np.array(rows), np.array(vrows), np.array(vmap)


# --- the random-init workload -----------------------------------------------------------------
def random_model(seed: int = 4, n_layers: int = N_LAYERS, vocab: int = VOCAB,
                 device: str = "cuda"):
    """A stock Qwen3_5ForCausalLM of config 5's shape with seeded random weights, bf16, on
    ``device``: every projection, conv tap and the (tied) embedding N(0, 0.02); the RMSNorm
    gains 0 (the (1 + w) form); the gated norms' weights 1, dt_bias 1 and A_log = log U(0, 16)
    (transformers' own initialisation, modeling_qwen3_5.py:786-813); the GDN weights drawn in
    Qwen's 32-value-head shape and zero-padded. Each tensor has its own generator seed
    (seed, index), so a tensor's values do not depend on the others'; on cuda the generator is
    torch's Philox, the same on every B200."""
    from transformers import Qwen3_5ForCausalLM

    cfg = hf_config(n_layers, vocab)
    with torch.device("meta"):
        model = Qwen3_5ForCausalLM(cfg).to(torch.bfloat16)
    model = model.to_empty(device=device)
    model.tie_weights()
    rows, vrows, heads = (torch.as_tensor(a, device=device) for a in pad_maps())
    k = [0]

    def gen():
        k[0] += 1
        return torch.Generator(device=device).manual_seed(seed * 1_000_003 + k[0])

    def normal(shape):
        return (torch.randn(shape, generator=gen(), device=device) * STD).to(torch.bfloat16)

    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(normal((vocab, H)))
        for i, layer in enumerate(model.model.layers):
            layer.input_layernorm.weight.zero_()
            layer.post_attention_layernorm.weight.zero_()
            if cfg.layer_types[i] == "linear_attention":
                ga = layer.linear_attn
                for p in (ga.in_proj_qkv.weight, ga.conv1d.weight, ga.in_proj_z.weight,
                          ga.in_proj_b.weight, ga.in_proj_a.weight, ga.out_proj.weight,
                          ga.A_log, ga.dt_bias):
                    p.zero_()
                ga.in_proj_qkv.weight.index_copy_(0, rows, normal((len(rows), H)))
                ga.conv1d.weight.index_copy_(0, rows, normal((len(rows), 1, 4)))
                ga.in_proj_z.weight.index_copy_(0, vrows, normal((len(vrows), H)))
                ga.in_proj_b.weight.index_copy_(0, heads, normal((QNV, H)))
                ga.in_proj_a.weight.index_copy_(0, heads, normal((QNV, H)))
                ga.out_proj.weight.index_copy_(1, vrows, normal((H, len(vrows))))
                u = torch.rand(QNV, generator=gen(), device=device) * 16
                ga.A_log.index_copy_(0, heads, u.log().to(torch.bfloat16))
                ga.dt_bias.index_copy_(0, heads, torch.ones(QNV, device=device,
                                                            dtype=torch.bfloat16))
                ga.norm.weight.fill_(1.0)
            else:
                at = layer.self_attn
                for p in (at.q_proj.weight, at.k_proj.weight, at.v_proj.weight,
                          at.o_proj.weight):
                    p.copy_(normal(tuple(p.shape)))
                at.q_norm.weight.zero_()
                at.k_norm.weight.zero_()
            for p in (layer.mlp.gate_proj.weight, layer.mlp.up_proj.weight,
                      layer.mlp.down_proj.weight):
                p.copy_(normal(tuple(p.shape)))
        model.model.norm.weight.zero_()
    model.tie_weights()
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg).to(device)
    force_torch_paths(model)
    return model.eval()


def force_torch_paths(model) -> None:
    """transformers' torch GDN functions (no fla / causal_conv1d kernels), as the reference's
    CPU path runs them."""
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
            ga.norm.weight.data = w


# --- packing ------------------------------------------------------------------------------------
class Unsupported(ValueError):
    pass


def _check_padding_zero(name, t, keep, dim=0):
    mask = torch.ones(t.shape[dim], dtype=torch.bool, device=t.device)
    mask[keep] = False
    rest = t.index_select(dim, mask.nonzero().flatten())
    if rest.numel() and bool((rest != 0).any()):
        raise Unsupported(f"{name}: nonzero weights in the padding")


def pack(model, check_padding: bool = True) -> dict:
    """The kernel's weight tables from a config-5-shaped model (every tensor bf16 on the model's
    device, rows contiguous over the hidden dim):
      GDN layer: w1 [12,352 x 2560] = Qwen's q (key-head major), k, v, z, b, a rows; conv
        [8192 x 4] (q, k, v channels); A_log, dt_bias and the gated norm's weight [128] as fp32
        values (flags: 1 when that weight is an fp32 parameter, as in the reference's merged
        model, so its product is not rounded to bf16);
      attention layer: w1 [10,240 x 2560] = q_proj (per head its 256 query then 256 gate rows),
        k_proj, v_proj; q_norm, k_norm [256];
      both: wo [2560 x 4096] (out_proj over the live value dims / o_proj); wgu [18,432 x 2560]
        (gate row u then up row u); wd [2560 x 9216]; ln_in, ln_post [2560];
    and the final norm and the tied head / embedding [vocab x 2560] (not copied).
    ``check_padding`` verifies that every padded row and column is zero (the kernel never
    reads them)."""
    cfg = model.config
    if any(t not in ("linear_attention", "full_attention") for t in cfg.layer_types):
        raise Unsupported("layer types other than GDN and full attention")
    if (cfg.hidden_size, cfg.intermediate_size, cfg.linear_key_head_dim,
            cfg.linear_value_head_dim, cfg.linear_num_key_heads, cfg.linear_num_value_heads,
            cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim) != (
            H, INTER, KD, VD, NK, NV, NQ, NKV, HD):
        raise Unsupported("not config 5's shape")
    dev = model.model.embed_tokens.weight.device
    rows, vrows, heads = (torch.as_tensor(a, device=dev) for a in pad_maps())
    bf = torch.bfloat16
    layers = []
    for i, layer in enumerate(model.model.layers):
        d = {"type": 0 if cfg.layer_types[i] == "linear_attention" else 1}
        d["ln_in"] = layer.input_layernorm.weight.detach().to(bf).contiguous()
        d["ln_post"] = layer.post_attention_layernorm.weight.detach().to(bf).contiguous()
        if d["type"] == 0:
            ga = layer.linear_attn
            if ga.norm.weight.dtype not in (bf, torch.float32):
                raise Unsupported("the gated norm's weight must be bf16 or fp32")
            d["flags"] = 1 if ga.norm.weight.dtype == torch.float32 else 0
            qkv, z = ga.in_proj_qkv.weight.detach(), ga.in_proj_z.weight.detach()
            b, a = ga.in_proj_b.weight.detach(), ga.in_proj_a.weight.detach()
            out = ga.out_proj.weight.detach()
            if check_padding:
                _check_padding_zero("in_proj_qkv", qkv, rows)
                _check_padding_zero("conv1d", ga.conv1d.weight.detach(), rows)
                _check_padding_zero("in_proj_z", z, vrows)
                _check_padding_zero("in_proj_b", b, heads)
                _check_padding_zero("in_proj_a", a, heads)
                _check_padding_zero("out_proj", out, vrows, dim=1)
            d["w1"] = torch.cat([qkv.index_select(0, rows), z.index_select(0, vrows),
                                 b.index_select(0, heads), a.index_select(0, heads)]).to(bf)
            d["conv"] = ga.conv1d.weight.detach().reshape(CONV, 4).index_select(0, rows).to(bf)
            d["A_log"] = ga.A_log.detach().float().index_select(0, heads).contiguous()
            d["dt_bias"] = ga.dt_bias.detach().float().index_select(0, heads).contiguous()
            d["gnorm"] = ga.norm.weight.detach().float().contiguous()
            d["wo"] = out.index_select(1, vrows).to(bf).contiguous()
        else:
            at = layer.self_attn
            d["w1"] = torch.cat([at.q_proj.weight.detach(), at.k_proj.weight.detach(),
                                 at.v_proj.weight.detach()]).to(bf)
            d["qn"] = at.q_norm.weight.detach().to(bf).contiguous()
            d["kn"] = at.k_norm.weight.detach().to(bf).contiguous()
            d["wo"] = at.o_proj.weight.detach().to(bf).contiguous()
        g, u = layer.mlp.gate_proj.weight.detach(), layer.mlp.up_proj.weight.detach()
        d["wgu"] = torch.stack([g, u], 1).reshape(2 * INTER, H).to(bf).contiguous()
        d["wd"] = layer.mlp.down_proj.weight.detach().to(bf).contiguous()
        d["w1"] = d["w1"].contiguous()
        layers.append(d)
    embed = model.model.embed_tokens.weight.detach()
    head = model.lm_head.weight.detach()
    if embed.dtype != bf or head.dtype != bf or not embed.is_contiguous() \
            or not head.is_contiguous():
        raise Unsupported("the embedding and the head must be contiguous bf16")
    return {"layers": layers, "norm": model.model.norm.weight.detach().to(bf).contiguous(),
            "embed": embed, "head": head, "eps": float(cfg.rms_norm_eps)}


def rope_table(model, max_pos: int) -> torch.Tensor:
    """cos and sin of positions [0, max_pos) from the model's own rotary module, as the stock
    forward computes them (fp32 then bf16), [max_pos][2][64] bf16."""
    rot = model.model.rotary_emb
    dev = rot.inv_freq.device
    x = torch.zeros(1, dtype=torch.bfloat16, device=dev)
    pos = torch.arange(max_pos, device=dev)[None]
    cos, sin = rot(x, pos)
    return torch.stack([cos[0], sin[0]], 1).contiguous()


# --- the decoder --------------------------------------------------------------------------------
class TextDecoder:
    """Greedy batch-1 decode of a config-5 model through ``lxb_text_decode``: a prompt forced
    token by token, then the model's own argmax, the next token kept on the device. Owns the
    caches: the GDN layers' conv windows and recurrent states in the stock cache layout
    ([24,576 x 4] bf16 and [128 x 256 x 128] fp32 per layer; only the non-padding parts are
    touched) and the attention layers' key/value rows [4 x max_pos x 256] bf16 each."""

    def __init__(self, model, max_pos: int = 4608, tables: dict | None = None) -> None:
        from ._lib import lib

        self._lib = lib()
        self.model = model
        self.t = tables or pack(model)
        self.dev = self.t["embed"].device
        if self.dev.type != "cuda":
            raise RuntimeError("the text decode runs on a CUDA device")
        self.max_pos = int(max_pos)
        n = len(self.t["layers"])
        self.n_gdn = sum(1 for d in self.t["layers"] if d["type"] == 0)
        self.n_att = n - self.n_gdn
        self.rope = rope_table(model, self.max_pos)
        self.conv = torch.zeros(self.n_gdn, CONV, 4, dtype=torch.bfloat16, device=self.dev)
        self.rec = torch.zeros(self.n_gdn, NV, KD, VD, dtype=torch.float32, device=self.dev)
        self.kc = torch.zeros(self.n_att, NKV, self.max_pos, HD, dtype=torch.bfloat16,
                              device=self.dev)
        self.vc = torch.zeros_like(self.kc)
        self.pos = 0
        desc = (_TLayer * n)()
        ig = ia = 0
        for i, d in enumerate(self.t["layers"]):
            e = desc[i]
            e.type = d["type"]
            e.flags = d.get("flags", 0)
            e.w1, e.wo, e.wgu, e.wd = (d[k].data_ptr() for k in ("w1", "wo", "wgu", "wd"))
            e.ln_in, e.ln_post = d["ln_in"].data_ptr(), d["ln_post"].data_ptr()
            if d["type"] == 0:
                e.conv_w, e.A_log, e.dt_bias = (d[k].data_ptr() for k in ("conv", "A_log",
                                                                          "dt_bias"))
                e.gnorm = d["gnorm"].data_ptr()
                e.conv_state, e.rec_state = self.conv[ig].data_ptr(), self.rec[ig].data_ptr()
                ig += 1
            else:
                e.qn, e.kn = d["qn"].data_ptr(), d["kn"].data_ptr()
                e.kc, e.vc = self.kc[ia].data_ptr(), self.vc[ia].data_ptr()
                ia += 1
        plan = ctypes.c_void_p()
        emb, head = self.t["embed"], self.t["head"]
        rc = self._lib.lxb_text_plan_create(
            ctypes.cast(desc, ctypes.c_void_p), n, emb.data_ptr(), emb.shape[0], head.data_ptr(),
            head.shape[0], self.t["norm"].data_ptr(), self.rope.data_ptr(), self.max_pos,
            ctypes.c_float(self.t["eps"]), self.dev.index or 0, ctypes.byref(plan))
        if rc != 0:
            raise RuntimeError(f"lxb_text_plan_create failed: {rc}")
        self.plan = plan
        self._desc = desc
        self.scratch = torch.empty(int(self._lib.lxb_text_scratch_bytes(self.plan)),
                                   dtype=torch.uint8, device=self.dev)

    def __del__(self):
        if getattr(self, "plan", None):
            self._lib.lxb_text_plan_destroy(self.plan)
            self.plan = None

    def reset(self) -> None:
        self.conv.zero_()
        self.rec.zero_()
        self.pos = 0

    def launch(self, forced: torch.Tensor, n_tokens: int, preds: torch.Tensor,
               hidden: torch.Tensor | None = None, stream: int | None = None) -> None:
        """One launch: ``n_tokens`` steps from position ``self.pos``; step t's input is
        forced[t] for t < len(forced), else the previous step's prediction; preds[t] the
        argmax after step t (device int32 tensors); ``hidden`` (optional, fp32
        [n_tokens, n_layers + 1, 2560]) receives at each step the residual after every layer and
        then the final norm's output."""
        nl = len(self.t["layers"])
        if hidden is not None and (hidden.dtype != torch.float32 or not hidden.is_contiguous()
                                   or hidden.numel() < n_tokens * (nl + 1) * H):
            raise ValueError("hidden must be a contiguous fp32 [n_tokens, n_layers + 1, 2560] "
                             "tensor")
        n_forced = int(forced.numel())
        if n_tokens < 1 or n_forced < 1 or n_tokens > preds.numel():
            raise ValueError("need 1 <= n_tokens <= len(preds) and a first token")
        if self.pos + n_tokens > self.max_pos:
            raise ValueError(f"positions past max_pos {self.max_pos}")
        st = torch.cuda.current_stream(self.dev).cuda_stream if stream is None else stream
        rc = self._lib.lxb_text_decode(self.plan, forced.data_ptr(), n_forced, n_tokens,
                                       self.pos, preds.data_ptr(),
                                       None if hidden is None else hidden.data_ptr(),
                                       self.scratch.data_ptr(), self.scratch.numel(),
                                       ctypes.c_void_p(st))
        if rc != 0:
            raise RuntimeError(f"lxb_text_decode failed: {rc}")
        self.pos += n_tokens

    def run(self, prompt, n_new: int) -> list[int]:
        """Prompt (forced) then ``n_new`` greedy tokens; returns the predictions after every
        step (len(prompt) + n_new - 1 of them: the last prompt step's is the first new token)."""
        ids = torch.as_tensor(np.asarray(prompt, np.int32), device=self.dev)
        n = len(ids) + n_new - 1
        preds = torch.empty(n, dtype=torch.int32, device=self.dev)
        self.launch(ids, n, preds)
        return preds.tolist()

    PROFILE = ("norm", "gemv", "wait", "sync", "gdn", "att", "head", "tokens")

    def set_profile(self, prof: torch.Tensor | None) -> None:
        """Per-CTA cycle counters (int64 [grid, len(PROFILE)] on the device, added to by every
        later launch), or None to turn them off."""
        if prof is not None and (prof.dtype != torch.int64 or not prof.is_contiguous()
                                 or prof.numel() < self.grid * len(self.PROFILE)):
            raise ValueError("prof must be a contiguous int64 [grid, sections] tensor")
        rc = self._lib.lxb_text_set_profile(self.plan, None if prof is None else prof.data_ptr())
        if rc != 0:
            raise RuntimeError(f"lxb_text_set_profile failed: {rc}")
        self._prof = prof

    @property
    def grid(self) -> int:
        return int(self._lib.lxb_text_grid(self.plan))

    def status(self) -> int:
        """The plan's sticky LXB_S_* bits (token clamped, staging or grid-barrier timeout)."""
        v = ctypes.c_uint32()
        rc = self._lib.lxb_text_status(self.plan, ctypes.byref(v))
        if rc != 0:
            raise RuntimeError(f"lxb_text_status failed: {rc}")
        return int(v.value)

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens: int, do_sample: bool = False,
                 stop_strings=None, tokenizer=None, chunk: int = 64, **_):
        """The reference's text call, ``tv.generate(x, max_new_tokens=..., do_sample=False,
        stop_strings=[...], tokenizer=tok)`` (lx/lx/chat.py:69-70), greedy at batch 1 from an
        empty cache: returns [1, prompt + new] ids. With stop strings the new tokens are decoded
        ``chunk`` at a time and generation ends after the token that completes one (as
        transformers' StopStringCriteria ends it)."""
        if do_sample:
            raise ValueError("only greedy decoding (do_sample=False)")
        x = torch.as_tensor(input_ids).reshape(-1)
        ids = x.to(self.dev, torch.int32)
        self.reset()
        if max_new_tokens < 1:
            return x.view(1, -1).to(self.dev, torch.long)
        preds = torch.empty(max(len(ids), chunk), dtype=torch.int32, device=self.dev)
        self.launch(ids, len(ids), preds)  # the prompt; its last prediction is the first new
        new = [int(preds[len(ids) - 1])]
        while len(new) < max_new_tokens and not _stopped(new, stop_strings, tokenizer):
            k = min(chunk, max_new_tokens - len(new))
            self.launch(torch.tensor([new[-1]], dtype=torch.int32, device=self.dev), k, preds)
            new += preds[:k].tolist()
        if stop_strings:
            new = _cut_at_stop(new, stop_strings, tokenizer)
        out = torch.tensor(new[:max_new_tokens], dtype=torch.long, device=self.dev)
        return torch.cat([x.to(self.dev, torch.long), out]).view(1, -1)


def _stopped(new, stop_strings, tok) -> bool:
    if not stop_strings or tok is None:
        return False
    text = tok.decode(new)
    return any(s in text for s in stop_strings)


def _cut_at_stop(new, stop_strings, tok):
    """The shortest prefix of ``new`` whose text contains a stop string (all of it if none)."""
    if tok is None:
        return new
    for k in range(1, len(new) + 1):
        text = tok.decode(new[:k])
        if any(s in text for s in stop_strings):
            return new[:k]
    return new


class _TLayer(ctypes.Structure):
    """lxb_text_layer (include/lxb.h)."""
    _fields_ = [("type", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("w1", ctypes.c_uint64), ("wo", ctypes.c_uint64), ("wgu", ctypes.c_uint64),
                ("wd", ctypes.c_uint64), ("ln_in", ctypes.c_uint64), ("ln_post", ctypes.c_uint64),
                ("conv_w", ctypes.c_uint64), ("A_log", ctypes.c_uint64),
                ("dt_bias", ctypes.c_uint64), ("gnorm", ctypes.c_uint64),
                ("qn", ctypes.c_uint64), ("kn", ctypes.c_uint64),
                ("conv_state", ctypes.c_uint64), ("rec_state", ctypes.c_uint64),
                ("kc", ctypes.c_uint64), ("vc", ctypes.c_uint64)]


def _main(argv=None) -> None:
    """python -m linuxformer_b200.text [n_layers] [vocab] [prompt] [tokens]: a seeded random-init
    model (config 5's shape; fewer layers or a smaller vocabulary for small profiling cases), one
    launch of the prompt, one launch of greedy tokens after it; prints the decode rate."""
    import sys
    import time

    args = [int(x) for x in (sys.argv[1:] if argv is None else argv)]
    n_layers, vocab, n_prompt, n_new = (args + [N_LAYERS, VOCAB, 64, 64][len(args):])[:4]
    model = random_model(seed=4, n_layers=n_layers, vocab=vocab)
    dec = TextDecoder(model, max_pos=n_prompt + n_new)
    ids = torch.from_numpy(np.random.default_rng(4).integers(0, vocab, n_prompt).astype(np.int32))
    preds = torch.empty(max(n_prompt, n_new), dtype=torch.int32, device=dec.dev)
    dec.launch(ids.to(dec.dev), n_prompt, preds)
    torch.cuda.synchronize(dec.dev)
    t0 = time.perf_counter()
    dec.launch(preds[n_prompt - 1:n_prompt].clone(), n_new, preds)
    torch.cuda.synchronize(dec.dev)
    dt = time.perf_counter() - t0
    print(f"{n_layers} layers, vocab {vocab}: {n_new} tokens after a {n_prompt}-token prompt in "
          f"{dt * 1e3:.1f} ms ({n_new / dt:.1f} tok/s), status {dec.status()}")


if __name__ == "__main__":
    _main()
