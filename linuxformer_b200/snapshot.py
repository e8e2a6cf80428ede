"""Machine snapshots in the reference's file layout, and a bitwise state diff.

A snapshot holds every chip layer's conv window (bf16 [conv_dim, 4], oldest tap first) and
recurrent state (fp32 [128, 256, 128]) plus the session's host fields. The .safetensors layout is
the one of the reference's `save_safe` / `load_safe` (`lx/lx/session.py:259-292`): tensors
`conv.L` and `recurrent.L`, the machine's byte fields as uint8 tensors `ref.<name>`, and every
other field as JSON in the metadata key `lx.session` (`next`, `last`, `n`, `waiting`, `ref`,
`bytes`). Files written here load with the reference's `Session.load`, and the reference's load
here, so a stream decoded on the B200 can be handed to the reference and back.

    st = snapshot.of_states(dev_states, s=0)        # one stream of a Decoder's DeviceStates
    snapshot.save("boot.safetensors", st, next=tok, n=tokens_seen)
    d = snapshot.load("boot.safetensors")           # {"state": [(conv, rec), ...], "next": ...}
    snapshot.into(dev_states, 0, d["state"])
    r = snapshot.diff(d["state"], other["state"])   # {"elements", "elements_differ", ...}

`diff` compares bit patterns (like the reference's `tests/check_snapshots.py`: -0 differs from
+0, a NaN equals only the same NaN) and runs on whatever device the tensors are on.
"""

from __future__ import annotations

import json
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import torch

from . import chip as C

META_KEY = "lx.session"


def of_states(states, s: int = 0) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Stream s of a DeviceStates as [(conv bf16 [CONV, 4], recurrent fp32 [NV, KD, VD])] per
    layer (views of the device tensors, no copy)."""
    return [(states.conv[s, L].view(torch.bfloat16), states.recurrent[s, L])
            for L in range(states.recurrent.shape[1])]


def of_host(st: C.State) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """A host chip.State in the same form (CPU tensors sharing its memory)."""
    conv = torch.from_numpy(np.ascontiguousarray(st.conv).view(np.int16)).view(torch.bfloat16)
    rec = torch.from_numpy(np.ascontiguousarray(st.recurrent))
    return [(conv[L], rec[L]) for L in range(rec.shape[0])]


def to_host(state) -> C.State:
    """[(conv, rec)] per layer back to a host chip.State (copies)."""
    conv = np.stack([c.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
                     for c, _ in state])
    rec = np.stack([r.detach().cpu().contiguous().numpy() for _, r in state])
    return C.State(rec.astype(np.float32, copy=False), conv)


def into(states, s: int, state) -> None:
    """Copy [(conv, rec)] per layer into stream s of a DeviceStates (any device to any device).
    The launch after it must rebuild the decaying layers' bitmaps (lxb_decode with
    sync_bitmaps, the default of Decoder.launch/run)."""
    nl = states.recurrent.shape[1]
    if len(state) != nl:
        raise ValueError(f"snapshot has {len(state)} layers, the states {nl}")
    for L, (c, r) in enumerate(state):
        if tuple(c.shape) != (C.CONV, C.TAPS) or c.dtype != torch.bfloat16:
            raise ValueError(f"layer {L}: conv must be bf16 [{C.CONV}, {C.TAPS}], is "
                             f"{c.dtype} {tuple(c.shape)}")
        if tuple(r.shape) != (C.NV, C.KD, C.VD) or r.dtype != torch.float32:
            raise ValueError(f"layer {L}: recurrent must be fp32 [{C.NV}, {C.KD}, {C.VD}], is "
                             f"{r.dtype} {tuple(r.shape)}")
        states.conv[s, L].copy_(c.view(torch.int16))
        states.recurrent[s, L].copy_(r)


def save(path, state, next: int = 0, last: int = 0, n: int = 0, waiting=False,
         ref=None) -> None:
    """Write a snapshot. .safetensors: the reference's save_safe layout (no pickle); any other
    suffix: torch.save of the same dict the reference's Session.save writes (ref as a plain
    namespace). ref: the proposer machine's fields (an object or a dict; bytes fields become
    tensors), or None."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    fields = dict(vars(ref)) if ref is not None and not isinstance(ref, dict) else dict(ref or {})
    cpu = [(c.detach().cpu().contiguous(), r.detach().cpu().contiguous()) for c, r in state]
    if path.suffix != ".safetensors":
        torch.save({"state": cpu, "next": next, "last": last, "n": n, "waiting": waiting,
                    "ref": SimpleNamespace(**fields)}, path)
        return
    from safetensors.torch import save_file

    t, plain, kinds = {}, {}, {}
    for L, (c, r) in enumerate(cpu):
        t[f"conv.{L}"], t[f"recurrent.{L}"] = c, r
    for k, v in fields.items():
        if isinstance(v, (bytes, bytearray)):
            t[f"ref.{k}"] = (torch.frombuffer(bytearray(v), dtype=torch.uint8).clone() if v
                             else torch.zeros(0, dtype=torch.uint8))
            kinds[k] = type(v).__name__
        else:
            plain[k] = v
    meta = {"next": next, "last": last, "n": n, "waiting": waiting, "ref": plain, "bytes": kinds}
    save_file(t, str(path), metadata={META_KEY: json.dumps(meta)})


def load(path) -> dict:
    """Read a snapshot (either format): {"state": [(conv, rec)] per layer as CPU tensors, "next",
    "last", "n", "waiting", "ref": a namespace of the machine's fields}."""
    path = Path(path)
    if path.suffix != ".safetensors":
        d = torch.load(path, weights_only=False)
        return dict(d, state=[(c, r) for c, r in d["state"]])
    from safetensors import safe_open

    with safe_open(str(path), "pt") as f:
        md = f.metadata() or {}
        if META_KEY not in md:
            raise ValueError(f"{path}: not a session snapshot (no {META_KEY!r} metadata)")
        meta = json.loads(md[META_KEY])
        t = {k: f.get_tensor(k) for k in f.keys()}
    ref = SimpleNamespace(**meta.pop("ref"))
    for k, kind in meta.pop("bytes").items():
        b = t[f"ref.{k}"].numpy().tobytes()
        setattr(ref, k, bytearray(b) if kind == "bytearray" else b)
    n = sum(k.startswith("conv.") for k in t)
    return dict(meta, ref=ref, state=[(t[f"conv.{L}"], t[f"recurrent.{L}"]) for L in range(n)])


def _bits(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1).view({2: torch.int16, 4: torch.int32}[x.element_size()])


def diff(a, b, max_report: int = 20) -> dict:
    """Bitwise comparison of two [(conv, rec)] state lists (same shapes and dtypes; on any one
    device): element counts, differing elements, and the first max_report differences."""
    if len(a) != len(b):
        raise ValueError(f"{len(a)} layers against {len(b)}")
    res = {"layers": len(a), "elements": 0, "elements_differ": 0, "differences": []}
    for L, (sa, sb) in enumerate(zip(a, b)):
        for kind, x, y in zip(("conv", "recurrent"), sa, sb):
            if x.shape != y.shape or x.dtype != y.dtype:
                raise ValueError(f"layer {L} {kind}: {x.dtype} {tuple(x.shape)} against "
                                 f"{y.dtype} {tuple(y.shape)}")
            ne = _bits(x).ne(_bits(y.to(x.device)))
            res["elements"] += x.numel()
            k = int(ne.sum())
            res["elements_differ"] += k
            if k and len(res["differences"]) < max_report:
                idx = ne.nonzero()[:max_report - len(res["differences"]), 0].tolist()
                xf, yf = x.reshape(-1), y.reshape(-1)
                for i in idx:
                    at = np.unravel_index(i, tuple(x.shape))
                    res["differences"].append({"layer": L, "state": kind,
                                               "index": [int(j) for j in at],
                                               "a": float(xf[i]), "b": float(yf[i])})
    return res
