"""The reference's verified mode on the B200 decode kernel.

``Session.verify`` (lx/lx/session.py:86-116) runs proposed tokens through the chip model as a
chunked prefill (``Fast.forward`` then ``head_argmax``, lx/lx/fast.py:252-257) and checks that at
every position the output head's argmax is the next token. Here a chunk is one decode launch
with every input forced (``Mega.run(toks, len(toks))``): the kernel embeds each given token, runs
every chip layer and the head, and takes the next input from the list instead of the argmax.
The recurrent step over a chunk computes the stock chunked prefill's function; the tests hold
it to the reference's own chunked forward on its golden fixture (predictions and conv windows
bit for bit, recurrent states within 1e-9).

    mg = Mega(fast, model, cache, offset)          # linuxformer_b200.mega
    v = Verifier(mg, typed=session_typed, go=tok_go)
    r = v.verify(toks)   # {"wrong", "first_wrong", "predicted"[, "out"]}
"""

from __future__ import annotations

from typing import Callable, Sequence

import numpy as np


class Verifier:
    """Session.verify's bookkeeping over a Mega (or anything with ``run(forced, n) -> list``).

    typed: tokens the user types (the reference's ``_typed``: their predictions are not
    checked), as a function of an int64 array returning a bool array; go: the token a stream
    starts with (prepended to the first call when missing, as the reference does with GO);
    console: optional, the reference's ``console`` (bytes of the untyped predictions)."""

    def __init__(self, mega, chunk: int = 65536,
                 typed: Callable[[np.ndarray], np.ndarray] | None = None,
                 go: int | None = None, console: Callable | None = None) -> None:
        if chunk < 1:
            raise ValueError("chunk must be positive")
        self.mega, self.chunk, self.typed, self.go, self.console = mega, chunk, typed, go, console
        self.next: int | None = None  # the prediction for the token after the last one checked
        self.last: int | None = None
        self.n = 0

    def verify(self, toks: Sequence[int]) -> dict:
        """Run toks as chunked prefill; position i's prediction is for token i + 1 (the one for
        toks[0] came from the previous call). Returns {"wrong": count of positions whose
        prediction is not the token there (typed tokens excepted), "first_wrong": up to 8
        (index, want, got), "predicted": the predictions (int64 array)[, "out": console bytes]}."""
        toks = [int(t) for t in toks]
        if self.n == 0 and self.go is not None and toks[:1] != [self.go]:
            toks = [self.go] + toks
        if not toks:
            raise ValueError("no tokens to verify")
        preds: list[int] = []
        for a in range(0, len(toks), self.chunk):
            part = toks[a:a + self.chunk]
            preds += list(self.mega.run(part, len(part)))
        pred = np.asarray(preds, np.int64)
        target = np.asarray(toks, np.int64)
        prev = -1 if self.next is None else self.next
        want_pred = np.concatenate([[prev], pred[:-1]])
        typed = (np.asarray(self.typed(target), bool) if self.typed is not None
                 else np.zeros(len(target), bool))
        bad = (want_pred != target) & ~typed
        if self.next is None:
            bad[0] = False
        idx = np.nonzero(bad)[0].tolist()
        self.next, self.last = int(pred[-1]), toks[-1]
        self.n += len(toks)
        got = want_pred.tolist()
        out = {"wrong": len(idx), "first_wrong": [(i, toks[i], got[i]) for i in idx[:8]],
               "predicted": pred}
        if self.console is not None:
            out["out"] = self.console(got[i] for i in range(len(toks)) if not typed[i])
        return out
