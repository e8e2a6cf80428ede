"""Self-drafting verify: a greedy chip decode whose rounds guess tokens from the stream's own past
and check the guess with one chunked-prefill call.

The reference proposes this and simulates how far it would go (lx/tools/draft_sim.py:1-7: drafts
from the stream's own past tokens only, each round checked by one prefill call that keeps the
drafted prefix the model agrees with, plus the model's own next token) but does not build it.
Here it runs on the prefill kernels (csrc/prefill.cu, ``lxb_prefill``):

- the draft ("copy", tools/draft_sim.py:36-66): find the latest earlier occurrence of the last n
  tokens and continue after it with that period (the draft may run past the stream's end into
  its own tokens, so a short cycle fills a long draft);
- the check: the current token and the draft as one chunk through ``lxb_prefill`` from the
  current state; its first-mismatch index (computed on the device) is the number of draft tokens
  the model agrees with, and the prediction there is the model's own next token;
- the state: the prefill advanced it through the whole chunk; when a draft token was wrong it is
  put back (a device copy taken before the round) and advanced through the accepted tokens only.
The prefill is bit-identical to the per-token decode with every input forced, so the stream and
the final state are the plain greedy decode's, bit for bit.

    sd = SelfDraft(Prefill(chip), draft=255)      # chunks of up to 256 tokens
    preds, stats = sd.run(ptrs, [rec, conv], first=0, n=4096)

A chunk is padded to a multiple of 256 tokens inside the prefill, so drafts of 255 (chunks of 256)
cost no more than shorter ones.
"""

from __future__ import annotations

import numpy as np
import torch

from .prefill import Prefill


class CopyDrafter:
    """The n-gram copy drafter over a growing stream (tools/draft_sim.py's "copy")."""

    def __init__(self, ngram: int = 6) -> None:
        self.n = ngram
        self.hist: list[int] = []
        self.seen: dict[tuple, int] = {}  # n-gram ending at q -> q + 1 (the position after it)
        self.q = 0                        # positions < q are indexed

    def extend(self, toks) -> None:
        self.hist.extend(int(t) for t in toks)

    def propose(self, D: int) -> list[int]:
        h, n = self.hist, self.n
        i = len(h)
        # index every n-gram that ends before the current suffix's last token
        while self.q < i - 1:
            q = self.q
            if q + 1 >= n:
                self.seen[tuple(h[q + 1 - n:q + 1])] = q + 1
            self.q += 1
        if D <= 0 or i < n:
            return []
        j = self.seen.get(tuple(h[i - n:i]))
        if j is None:
            return []
        p = i - j
        out: list[int] = []
        for a in range(D):
            b = i + a - p
            out.append(h[b] if b < i else out[b - i])
        return out


class SelfDraft:
    """Greedy decode by draft-and-verify rounds on a Prefill plan (one stream)."""

    def __init__(self, prefill: Prefill, draft: int = 64, ngram: int = 6, drafter=None,
                 decoder=None, burst: int = 16) -> None:
        """drafter: a factory of drafters (objects with extend(tokens) and propose(D)); the
        default is CopyDrafter(ngram). decoder (a runtime.Decoder of the same chip, optional):
        where the drafter has nothing to propose, the decode kernel runs ``burst`` tokens
        instead of one-token prefill calls (its nonzero-row bitmaps rebuilt from the state
        first, since the prefill does not keep them)."""
        self.pf = prefill
        self.dec = decoder
        self.burst = int(burst)
        self.make_drafter = drafter or (lambda: CopyDrafter(self.ngram))
        self.D = int(draft)
        self.ngram = int(ngram)
        dev = prefill.dev
        self.sc = prefill.scratch(self.D + 1)
        self.tokens = torch.empty(self.D + 1, dtype=torch.int32, device=dev)
        self.preds = torch.empty(self.D + 1, dtype=torch.int32, device=dev)
        self.fw = torch.empty(1, dtype=torch.int32, device=dev)
        self.h_tok = torch.empty(self.D + 1, dtype=torch.int32).pin_memory()
        self.h_out = torch.empty(self.D + 2, dtype=torch.int32).pin_memory()

    @torch.no_grad()
    def run(self, ptrs: torch.Tensor, state: list[torch.Tensor], first: int, n: int,
            stream=None):
        """n greedy predictions from the state behind ptrs (updated in place; ``state`` lists
        the tensors it lives in, for the round's copy) with ``first`` as the first input:
        returns (preds int32 [n], stats)."""
        dev = self.pf.dev
        st = torch.cuda.current_stream(dev) if stream is None else stream
        snap = [torch.empty_like(t) for t in state]
        dr = self.make_drafter()
        dr.extend([first])
        out: list[int] = []
        cur = int(first)
        rounds = rollbacks = drafted = bursts = burst_tokens = 0
        if self.dec is not None:
            L = self.pf.chip.n_layers
            ptrs3 = ptrs.view(1, L, 2)
            bitmaps = torch.zeros((1, L, 128, 8), dtype=torch.int32, device=dev)
            dscratch = self.dec.scratch(1)
            bf = torch.empty((1, 1), dtype=torch.int32, device=dev)
            bp = torch.empty((1, max(1, self.burst)), dtype=torch.int32, device=dev)
        with torch.cuda.stream(st):
            while len(out) < n:
                draft = dr.propose(min(self.D, n - len(out) - 1))
                if not draft and self.dec is not None and n - len(out) > 1:
                    k = min(self.burst, n - len(out))
                    bf.fill_(cur)
                    self.dec.launch(ptrs3, bitmaps, bf, k, bp[:, :k], None, sync_bitmaps=True,
                                    stream=st, scratch=dscratch)
                    new = bp[0, :k].tolist()  # syncs
                    out.extend(new)
                    dr.extend(new)
                    cur = new[-1]
                    bursts += 1
                    burst_tokens += k
                    continue
                T = 1 + len(draft)
                self.h_tok[0] = cur
                if draft:
                    self.h_tok[1:T] = torch.tensor(draft, dtype=torch.int32)
                    for s, t in zip(snap, state):
                        s.copy_(t, non_blocking=True)
                self.tokens[:T].copy_(self.h_tok[:T], non_blocking=True)
                self.pf.launch(ptrs, self.tokens[:T], self.preds, self.fw if draft else None,
                               stream=st, scratch=self.sc)
                self.h_out[:T].copy_(self.preds[:T], non_blocking=True)
                if draft:
                    self.h_out[self.D + 1:].copy_(self.fw, non_blocking=True)
                st.synchronize()
                fw = int(self.h_out[self.D + 1]) if draft else -1
                a = len(draft) if fw < 0 else fw
                if a < len(draft):  # put the state back, then advance through cur + draft[:a]
                    for s, t in zip(snap, state):
                        t.copy_(s, non_blocking=True)
                    self.pf.launch(ptrs, self.tokens[:a + 1], self.preds, None, stream=st,
                                   scratch=self.sc)
                    rollbacks += 1
                new = draft[:a] + [int(self.h_out[a])]
                out.extend(new)
                dr.extend(new)
                cur = new[-1]
                rounds += 1
                drafted += len(draft)
        self.pf._raise_status()
        stats = {"rounds": rounds, "decode_bursts": bursts,
                 "decoded_in_bursts": burst_tokens,
                 "tokens_per_round": round((len(out) - burst_tokens) / max(rounds, 1), 2),
                 "rollbacks": rollbacks, "drafted": drafted}
        return np.asarray(out[:n], dtype=np.int32), stats
