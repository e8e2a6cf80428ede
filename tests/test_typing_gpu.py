"""The device typing queue (lxb_plan_set_typing) against the same typing rule applied by the
host to the CPU restatement one token at a time: the stream the machine sees, with every key
where the rule puts it, is identical, in one launch and over several chained launches. The rule
is the reference's host loop (Linux.run_alone, lx/lx/linux.py:254-289) at one-token granularity:
a batch of at most RX_SLOTS bytes (KEY0 then KEY) replaces the model's prediction once the
current input is a record boundary and every byte typed so far has been read."""

import numpy as np
import pytest

from linuxformer_b200 import chip as C
from linuxformer_b200.runtime import Decoder
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu

KEY0, KEY, SLOTS = 3000, 3256, 4


def _classes(chip, stream_tokens):
    """Token classes for config 1 (which has no machine semantics of its own): even ids are
    record boundaries, KEY0 / KEY ids are typed keys, and two ids the stream visits often are RX
    reads, so the FIFO drains and several batches go in."""
    tc = np.zeros(chip.n_vocab, np.uint8)
    tc[0::2] |= Decoder.T_FINAL
    tc[KEY0:KEY + 256] |= Decoder.T_TYPED
    for t in stream_tokens:
        tc[t] |= Decoder.T_RX
    return tc


def host_typed(chip, st, first, n, keys, tc):
    """The rule on the host over the CPU restatement, one token at a time."""
    o = Oracle(chip)
    k = wait = left = 0
    cur = first
    wait += int(bool(tc[cur] & Decoder.T_TYPED)) - int(bool(tc[cur] & Decoder.T_RX))
    inputs, preds = [cur], []
    for i in range(n):
        p, _, _ = o.decode(st, [cur], 1)
        bi = int(p[0])
        preds.append(bi)
        if i + 1 == n:
            break
        if left == 0 and k < len(keys) and wait == 0 and tc[cur] & Decoder.T_FINAL:
            left = min(SLOTS, len(keys) - k) - 1
            nt = KEY0 + keys[k]
            k += 1
        elif left > 0 and k < len(keys):
            left -= 1
            nt = KEY + keys[k]
            k += 1
        else:
            nt = bi
        wait += int(bool(tc[nt] & Decoder.T_TYPED)) - int(bool(tc[nt] & Decoder.T_RX))
        cur = nt
        inputs.append(cur)
    return np.array(preds), np.array(inputs), k


def test_device_typing_matches_the_host_rule(c1_chip):
    chip = c1_chip
    st0 = C.c1_state(chip, 0)
    keys = list(b"ls -la /proc\n")
    plain, _, _ = Oracle(chip).decode(st0.copy(), [0], 64)
    tc = _classes(chip, [int(plain[40]), int(plain[41])])
    n = 160
    want_p, want_i, typed = host_typed(chip, st0.copy(), 0, n, keys, tc)
    assert typed == len(keys)  # every byte went in
    dec = Decoder(chip, cluster=16)
    dec.set_typing([keys], KEY0, KEY, SLOTS, tc)
    ds = dec.states([st0])
    preds, inputs = dec.run(ds, [[0]], n)
    assert (inputs[0].cpu().numpy() == want_i).all()
    assert (preds[0].cpu().numpy() == want_p).all()
    assert dec.typing_state()[0, 0] == len(keys)
    # the same over three launches: each takes the previous one's next input
    dec.set_typing([keys], KEY0, KEY, SLOTS, tc)
    ds = dec.states([st0])
    got_i, got_p, first = [], [], [[0]]
    for m in (50, 37, n - 87):
        p, i = dec.run(ds, first, m)
        got_p.append(p[0].cpu().numpy())
        got_i.append(i[0].cpu().numpy())
        first = dec.next_inputs().cpu().numpy().tolist()
    assert (np.concatenate(got_i) == want_i).all()
    assert (np.concatenate(got_p) == want_p).all()
    dec.set_typing(None, 0, 0, 1, None)
