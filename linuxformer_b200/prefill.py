"""The chunked prefill (verified mode) on the B200 kernels, and the reference's ``Fast`` interface
on it.

    pf = Prefill(chip)                              # tables built and uploaded once
    preds, first_wrong = pf.run(ptrs, tokens)       # one chunk; state updated in place

``Fast`` is a drop-in for ``lx.fast.Fast`` (lx/lx/fast.py:172-550) where the reference's verified
mode uses it: ``Session(c, model, machine, fast=Fast(model, n_chip, rows))`` calls
``fast.forward(e, cache)`` and ``fast.head_argmax(h)`` per chunk (lx/lx/session.py:94-98), and
``Linux.__init__`` builds it (lx/lx/linux.py:109). Both run on liblxb.so (include/lxb.h); the
cache's conv and recurrent tensors are updated in place, as the reference's are. There is no CPU
fallback: without a CUDA device or the built library the constructors raise.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import chip as C
from . import prefill_tables
from ._lib import S_ERRORS, Err, LxbError, check, lib


class Prefill:
    """A chip's prefill plan on one device."""

    def __init__(self, chip: C.Chip, device=None, embed: torch.Tensor | None = None) -> None:
        self.dev = torch.device(device or "cuda")
        if self.dev.type != "cuda":
            raise LxbError("the chip prefill runs on a CUDA device only")
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        torch.cuda.set_device(self.dev)
        self.chip = chip
        self.image, self.stats = prefill_tables.build_image(chip)
        self._img = np.frombuffer(self.image, np.uint8)
        p = ctypes.c_void_p()
        check(lib().lxb_prefill_plan_create(self._img.ctypes.data, len(self.image),
                                            ctypes.byref(p)), "lxb_prefill_plan_create")
        self.plan = p
        if embed is None:
            embed = torch.from_numpy(np.ascontiguousarray(chip.embed).view(np.int16)).to(self.dev)
        self.embed = embed
        self._scratch = None

    def __del__(self):
        p = getattr(self, "plan", None)
        if p is not None and p.value:
            try:
                lib().lxb_prefill_plan_destroy(p)
            except TypeError:  # interpreter shutdown
                pass
            self.plan = None

    def scratch(self, T: int) -> torch.Tensor:
        """Scratch for chunks of up to T tokens (kept and grown as needed)."""
        nb = lib().lxb_prefill_scratch_bytes(self.plan, T)
        if self._scratch is None or self._scratch.numel() < nb:
            self._scratch = None
            self._scratch = torch.empty(nb, dtype=torch.uint8, device=self.dev)
        return self._scratch

    def _stream(self, stream):
        return (stream or torch.cuda.current_stream(self.dev)).cuda_stream

    def launch(self, ptrs: torch.Tensor, tokens: torch.Tensor, preds: torch.Tensor,
               first_wrong: torch.Tensor | None = None, stream=None,
               scratch: torch.Tensor | None = None) -> None:
        """Raw launch on device tensors (no host sync): ptrs int64 [n_layers, 2] (or [1, L, 2]),
        tokens int32 [T], preds int32 [T], first_wrong int32 [1] or None."""
        T = tokens.numel()
        assert tokens.dtype == torch.int32 and tokens.is_contiguous()
        assert preds.dtype == torch.int32 and preds.numel() >= T and preds.is_contiguous()
        assert ptrs.dtype == torch.int64 and ptrs.numel() == 2 * self.chip.n_layers
        sc = scratch if scratch is not None else self.scratch(T)
        check(lib().lxb_prefill(self.plan, ptrs.data_ptr(), self.embed.data_ptr(),
                                tokens.data_ptr(), T, preds.data_ptr(),
                                first_wrong.data_ptr() if first_wrong is not None else None,
                                sc.data_ptr(), self._stream(stream)), "lxb_prefill")

    def set_timing(self, on: bool) -> None:
        """Record a CUDA event pair around every later kernel launch (per-stage timing)."""
        check(lib().lxb_prefill_set_timing(self.plan, int(on)), "lxb_prefill_set_timing")

    def timing(self) -> dict:
        """{stage: (milliseconds, launches)} since the last read (waits for the events)."""
        n = 15
        ms = (ctypes.c_double * n)()
        cnt = (ctypes.c_longlong * n)()
        check(lib().lxb_prefill_timing(self.plan, ms, cnt, n), "lxb_prefill_timing")
        return {lib().lxb_prefill_stage_name(k).decode(): (ms[k], cnt[k]) for k in range(n)
                if cnt[k]}

    def status(self) -> Err:
        e = Err()
        check(lib().lxb_prefill_status(self.plan, ctypes.byref(e)), "lxb_prefill_status")
        return e

    def _raise_status(self) -> None:
        e = self.status()
        if e.status & S_ERRORS:
            check(lib().lxb_prefill_status_clear(self.plan), "lxb_prefill_status_clear")
            raise LxbError(f"device status {e.status:#x} (token {e.first_step})")

    def run(self, ptrs: torch.Tensor, tokens, chunk: int | None = None):
        """Verify tokens in chunks of `chunk` (default: all at once): returns (preds int32
        device tensor [T], the first position i whose prediction is not tokens[i + 1], or -1).
        Raises on a device error (a token id outside the embedding)."""
        tok = torch.as_tensor(np.asarray(tokens, np.int32), device=self.dev)
        T = tok.numel()
        chunk = chunk or T
        preds = torch.empty(T, dtype=torch.int32, device=self.dev)
        first = -1
        fws = []
        for a in range(0, T, chunk):
            part = tok[a:a + chunk]
            f = torch.empty(1, dtype=torch.int32, device=self.dev)
            self.launch(ptrs, part, preds[a:a + chunk], f)
            fws.append((a, f))
        torch.cuda.synchronize(self.dev)
        self._raise_status()
        for a, f in fws:  # within chunks, then across each chunk boundary
            v = int(f.item())
            if v >= 0:
                first = a + v
                break
            b = a + chunk
            if b < T and int(preds[b - 1]) != int(tok[b]):
                first = b - 1
                break
        return preds, first

    def run_host(self, ptrs: torch.Tensor, tokens: np.ndarray, chunk: int) -> tuple:
        """The host-buffer call: token ids from (pinned) host memory in, chunk by chunk, the
        predictions back in host memory; returns (preds int32 [T], the first mismatch or -1)."""
        tok = np.ascontiguousarray(tokens, np.int32)
        T = tok.size
        pin = getattr(self, "_pin", None)
        if pin is None or pin[0].numel() < T:
            pin = (torch.empty(T, dtype=torch.int32).pin_memory(),
                   torch.empty(T, dtype=torch.int32).pin_memory())
            self._pin = pin
        th, ph = pin[0][:T], pin[1][:T]
        th.numpy()[...] = tok
        st = torch.cuda.current_stream(self.dev)
        dtok = torch.empty(T, dtype=torch.int32, device=self.dev)
        dpred = torch.empty(T, dtype=torch.int32, device=self.dev)
        fws = torch.empty(-(-T // chunk), dtype=torch.int32, device=self.dev)
        sc = self.scratch(min(chunk, T))
        for k, a in enumerate(range(0, T, chunk)):
            dtok[a:a + chunk].copy_(th[a:a + chunk], non_blocking=True)
            self.launch(ptrs, dtok[a:a + chunk], dpred[a:a + chunk], fws[k:k + 1], scratch=sc)
        ph.copy_(dpred, non_blocking=True)
        fh = fws.cpu()  # syncs the stream
        st.synchronize()
        self._raise_status()
        preds = ph.numpy().copy()
        first = -1
        for k, a in enumerate(range(0, T, chunk)):
            if int(fh[k]) >= 0:
                first = a + int(fh[k])
                break
            b = a + chunk
            if b < T and preds[b - 1] != tok[b]:
                first = b - 1
                break
        return preds, first

    def layers(self, ptrs: torch.Tensor, h: torch.Tensor, out: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
        """The chip layers on rows h (bf16 [T, 2560] on the device), state updated in place."""
        assert h.dtype == torch.bfloat16 and h.is_contiguous() and h.shape[-1] == C.H
        T = h.numel() // C.H
        out = torch.empty_like(h) if out is None else out
        check(lib().lxb_prefill_layers(self.plan, ptrs.data_ptr(), h.data_ptr(), out.data_ptr(),
                                       T, self.scratch(T).data_ptr(), self._stream(stream)),
              "lxb_prefill_layers")
        return out

    def head(self, h: torch.Tensor, stream=None) -> torch.Tensor:
        """The head's first argmax for rows h (bf16 [T, 2560]): int32 [T]."""
        assert h.dtype == torch.bfloat16 and h.is_contiguous() and h.shape[-1] == C.H
        T = h.numel() // C.H
        preds = torch.empty(T, dtype=torch.int32, device=self.dev)
        check(lib().lxb_prefill_head(self.plan, h.data_ptr(), T, preds.data_ptr(),
                                     self.scratch(T).data_ptr(), self._stream(stream)),
              "lxb_prefill_head")
        return preds


def cache_pointers(cache, n_chip: int, dev) -> torch.Tensor:
    """[n_chip, 2] device pointers (recurrent, conv) of an HF DynamicCache's chip layers."""
    rows = []
    for L in range(n_chip):
        cl = cache.layers[L]
        r, c = cl.recurrent_states[0], cl.conv_states[0]
        assert r.is_contiguous() and c.is_contiguous() and r.dtype == torch.float32
        assert c.dtype == torch.bfloat16 and c.shape[-1] == C.TAPS
        rows.append((r.data_ptr(), c.data_ptr()))
    return torch.tensor(rows, dtype=torch.int64, device=dev)


class Fast:
    """lx.fast.Fast's interface (lx/lx/fast.py:172-550) on liblxb.so: the chip layers' forward
    over a chunk (``forward``), the head's argmax (``head_argmax``) and the single-token step
    (``decode``, a chunk of one token).

    A circuit the prefill kernels do not take (a key head with more live query/key rows than
    their register-resident recurrence holds: the real circuit's memory heads have 256) runs
    through the decode kernel instead, every input forced: the same bits as the stock per-token
    forward, at the decode's speed. The decode kernel keeps no hidden states, so ``forward`` and
    ``decode`` then return NaN rows whose only use is ``head_argmax`` of that same tensor (the
    predictions the kernel made); any other use of them shows up as NaN."""

    FALLBACK_ROWS = 1 << 20  # the largest chunk the decode-kernel path takes

    compile = False     # the reference's flags, kept for its callers; nothing to compile here
    lean = False
    head_block = 8192
    stats = None
    idle_skip = False

    def __init__(self, model, n_chip: int, rows: slice | None = None) -> None:
        from .mega import chip_from_model

        self.model, self.n_chip, self.rows = model, n_chip, rows
        self.dev = next(model.parameters()).device
        offset = rows.start if rows is not None else 0
        chip = chip_from_model(model, n_chip, rows, offset)
        emb = model.model.embed_tokens.weight
        chip.embed = chip.embed[:, :0]  # the kernels read the model's own embedding
        self.dec, self._last = None, None
        try:
            self.pf = Prefill(chip, device=self.dev, embed=emb.view(torch.int16))
        except prefill_tables.PrefillUnsupported as e:
            import dataclasses

            from .runtime import Decoder

            # the decode kernel over the chunk's own rows: its "embedding" is the chunk (row t
            # is input t, offset 0), every input forced
            self.pf, self.unsupported = None, str(e)
            fc = dataclasses.replace(chip, embed=np.zeros((self.FALLBACK_ROWS, 0), np.uint16),
                                     offset=0)
            self.dec = Decoder(fc, cluster=16, device=self.dev,
                               embed=torch.zeros((1, C.H), dtype=torch.int16, device=self.dev))
            self._bm = torch.zeros((1, n_chip, C.NV, 8), dtype=torch.int32, device=self.dev)
            self._scratch = self.dec.scratch(1)
        w = model.lm_head.weight if rows is None else model.lm_head.weight[rows]
        self.head_cols = (w != 0).any(0).nonzero()[:, 0]
        self.w_head = w[:, self.head_cols]

    @torch.no_grad()
    def forward(self, h: torch.Tensor, cache) -> torch.Tensor:
        """h (1, T, hidden) -> (1, T, hidden), updating the cache's conv and recurrent states."""
        x = h[0].contiguous()
        if self.pf is None:
            return self._through_decode(x, cache)[None]
        out = self.pf.layers(cache_pointers(cache, self.n_chip, self.dev), x)
        return out[None]

    @torch.no_grad()
    def decode(self, h: torch.Tensor, cache) -> torch.Tensor:
        """One token: h (1, hidden) -> (1, hidden)."""
        if self.pf is None:
            return self._through_decode(h.contiguous(), cache)
        return self.pf.layers(cache_pointers(cache, self.n_chip, self.dev), h.contiguous())

    @torch.no_grad()
    def head_argmax(self, h: torch.Tensor, block: int | None = None) -> torch.Tensor:
        """The output head's argmax over the rows given at construction, for h (T, hidden)."""
        if self.pf is None:
            if self._last is None or h.untyped_storage().data_ptr() != self._last[0] \
                    or h.shape[0] != self._last[1].shape[0]:
                raise LxbError("this circuit runs through the decode kernel (" + self.unsupported
                               + "): head_argmax takes only the rows forward/decode returned")
            return self._last[1].long()
        return self.pf.head(h.contiguous()).long()

    def _through_decode(self, x: torch.Tensor, cache) -> torch.Tensor:
        """The chunk x (T, hidden) bf16 through the decode kernel, inputs forced; the
        predictions are kept for head_argmax of the NaN rows returned."""
        T = x.shape[0]
        if not 0 < T <= self.FALLBACK_ROWS or x.dtype != torch.bfloat16:
            raise LxbError(f"a chunk of 1..{self.FALLBACK_ROWS} bf16 rows, not {T} {x.dtype}")
        self.dec.embed = x.view(torch.int16)
        forced = torch.arange(T, dtype=torch.int32, device=self.dev).view(1, T)
        preds = torch.empty((1, T), dtype=torch.int32, device=self.dev)
        ptrs = cache_pointers(cache, self.n_chip, self.dev).view(1, self.n_chip, 2)
        self.dec.launch(ptrs, self._bm, forced, T, preds, None, sync_bitmaps=True,
                        scratch=self._scratch)
        e = self.dec.status()
        if e.status & S_ERRORS:
            raise LxbError(f"decode kernel: device status {e.status:#x} at step {e.first_step}")
        out = torch.full_like(x, float("nan"))
        self._last = (out.untyped_storage().data_ptr(), preds[0])
        return out

    def to(self, dev) -> "Fast":
        if torch.device(dev) != self.dev:
            raise LxbError("a Fast plan lives on the device it was built on")
        return self

    def init_cache(self, cache, dev) -> None:
        """The chip layers' states as the stock forward of one zero token leaves them: all zero
        (conv windows bf16, recurrent states fp32), as the reference's (lx/lx/fast.py:420-430)."""
        conv = 2 * C.NK * C.KD + C.NV * C.VD
        for L in range(self.n_chip):
            cache.update_conv_state(torch.zeros(1, conv, 1, dtype=torch.bfloat16, device=dev), L,
                                    conv_kernel_size=C.TAPS)
            cache.layers[L].update_recurrent_state(
                torch.zeros(1, C.NV, C.KD, C.VD, dtype=torch.float32, device=dev))


def _main(argv) -> None:
    """python -m linuxformer_b200.prefill [T] [chunks]: config 1's stack from its seeded state,
    `chunks` chunks of T token ids (uniform over the vocabulary, seed 2) through lxb_prefill, and
    the time of the last chunk (CUDA events). A self-check and the profiling entry."""
    T = int(argv[1]) if len(argv) > 1 else 65536
    n = int(argv[2]) if len(argv) > 2 else 2
    chip = C.c1(0)
    st = C.c1_state(chip, 0)
    pf = Prefill(chip)
    dev = pf.dev
    rec = torch.from_numpy(st.recurrent.copy()).to(dev)
    conv = torch.from_numpy(st.conv.view(np.int16).copy()).to(dev)
    ptrs = torch.tensor([[rec[L].data_ptr(), conv[L].data_ptr()] for L in range(chip.n_layers)],
                        dtype=torch.int64, device=dev)
    ids = torch.from_numpy(np.random.default_rng(2).integers(0, chip.n_vocab, n * T)
                           .astype(np.int32)).to(dev)
    preds = torch.empty(n * T, dtype=torch.int32, device=dev)
    fw = torch.empty(n, dtype=torch.int32, device=dev)
    sc = pf.scratch(T)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for k in range(n):
        if k == n - 1:
            e0.record()
        pf.launch(ptrs, ids[k * T:(k + 1) * T], preds[k * T:(k + 1) * T], fw[k:k + 1], scratch=sc)
    e1.record()
    torch.cuda.synchronize(dev)
    pf._raise_status()
    ms = e0.elapsed_time(e1)
    print(f"{n} chunks of {T} tokens; the last: {ms:.2f} ms, {T / ms * 1e3:.0f} tok/s")


if __name__ == "__main__":
    import sys

    _main(sys.argv)
