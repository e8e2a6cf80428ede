"""Self-drafting verify on the GPU (linuxformer_b200.draft.SelfDraft over lxb_prefill): the
stream and the final state equal the plain greedy decode's bit for bit (the CPU restatement's,
and the decode kernel's), whatever the drafts; rounds accept many tokens once the stream cycles."""

import numpy as np
import pytest
import torch

from linuxformer_b200 import chip as C
from linuxformer_b200.draft import CopyDrafter, SelfDraft
from linuxformer_b200.prefill import Prefill
from linuxformer_b200.runtime import Decoder
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu


def _state(chip, st):
    rec = torch.from_numpy(st.recurrent.copy()).cuda()
    conv = torch.from_numpy(st.conv.view(np.int16).copy()).cuda()
    ptrs = torch.tensor([[rec[L].data_ptr(), conv[L].data_ptr()] for L in range(chip.n_layers)],
                        dtype=torch.int64, device="cuda")
    return rec, conv, ptrs


@pytest.mark.parametrize("draft", [1, 16, 256])
def test_self_draft_is_the_greedy_stream(c1_chip, draft):
    chip = c1_chip
    st0 = C.c1_state(chip, 0)
    n = 800
    rec, conv, ptrs = _state(chip, st0)
    got, stats = SelfDraft(Prefill(chip), draft=draft).run(ptrs, [rec, conv], 0, n)
    host = st0.copy()
    want, _, _ = Oracle(chip).decode(host, [0], n)
    assert (got == want).all()
    assert np.array_equal(conv.cpu().numpy().view(np.uint16), host.conv)
    assert not (rec.cpu().numpy() != host.recurrent).any()
    if draft >= 16:
        assert stats["tokens_per_round"] > 8


class _Spoiler(CopyDrafter):
    """Drafts with a wrong token in the middle every other round: the rollback path."""

    k = 0

    def propose(self, D):
        d = super().propose(D)
        self.k += 1
        if d and self.k % 2:
            d[len(d) // 2] = (d[len(d) // 2] + 1) % 4096
        return d


def test_rejected_drafts_roll_the_state_back(c1_chip):
    chip = c1_chip
    st0 = C.c1_state(chip, 0)
    n = 600
    rec, conv, ptrs = _state(chip, st0)
    got, stats = SelfDraft(Prefill(chip), draft=32, drafter=lambda: _Spoiler(6)).run(
        ptrs, [rec, conv], 0, n)
    host = st0.copy()
    want, _, _ = Oracle(chip).decode(host, [0], n)
    assert (got == want).all()
    assert stats["rollbacks"] > 10
    assert np.array_equal(conv.cpu().numpy().view(np.uint16), host.conv)
    assert not (rec.cpu().numpy() != host.recurrent).any()


def test_decode_bursts_where_nothing_is_drafted(c1_chip):
    """With a Decoder, undrafted stretches run on the decode kernel: the stream and the state
    stay the plain greedy decode's."""
    chip = c1_chip
    st0 = C.c1_state(chip, 0)
    n = 900
    rec, conv, ptrs = _state(chip, st0)
    sd = SelfDraft(Prefill(chip), draft=64, decoder=Decoder(chip, cluster=16), burst=8)
    got, stats = sd.run(ptrs, [rec, conv], 0, n)
    host = st0.copy()
    want, _, _ = Oracle(chip).decode(host, [0], n)
    assert (got == want).all()
    assert stats["decode_bursts"] > 0 and stats["rounds"] > 0
    assert np.array_equal(conv.cpu().numpy().view(np.uint16), host.conv)
    assert not (rec.cpu().numpy() != host.recurrent).any()


def test_self_draft_matches_the_decode_kernel(c1_chip):
    chip = c1_chip
    st = C.c1_state(chip, 7)
    n = 1500
    dec = Decoder(chip, cluster=16)
    ds = dec.states([st])
    want, _ = dec.run(ds, [[3]], n)
    rec, conv, ptrs = _state(chip, st)
    got, stats = SelfDraft(Prefill(chip), draft=64).run(ptrs, [rec, conv], 3, n)
    assert (got == want[0].cpu().numpy()).all()
    h = ds.host(0)
    assert np.array_equal(conv.cpu().numpy().view(np.uint16), h.conv)
    assert not (rec.cpu().numpy() != h.recurrent).any()
