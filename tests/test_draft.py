"""The self-drafting verify's drafter (linuxformer_b200.draft.CopyDrafter), CPU only: the copy
rule of the reference's simulator (lx/tools/draft_sim.py:36-66) on small streams."""

from linuxformer_b200.draft import CopyDrafter


def _sim_rounds(stream, D, n):
    """Rounds the draft-and-verify loop takes to produce `stream` (a perfect model)."""
    dr = CopyDrafter(n)
    dr.extend(stream[:1])
    i, rounds = 1, 0
    while i < len(stream):
        d = dr.propose(min(D, len(stream) - i - 1))
        a = 0
        while a < len(d) and d[a] == stream[i + a]:
            a += 1
        new = stream[i:i + a + 1]
        dr.extend(new)
        i += len(new)
        rounds += 1
    return rounds


def test_no_match_no_draft():
    dr = CopyDrafter(3)
    dr.extend([5, 6, 7, 8])
    assert dr.propose(10) == []


def test_copies_the_continuation_with_its_period():
    dr = CopyDrafter(2)
    dr.extend([1, 2, 3, 9, 1, 2])
    # the last 2 tokens (1, 2) occurred at 0..1; the continuation after them, period 4
    assert dr.propose(6) == [3, 9, 1, 2, 3, 9]


def test_a_cycle_fills_a_long_draft():
    dr = CopyDrafter(4)
    dr.extend([7, 1, 2, 3, 4, 1, 2, 3, 4])
    assert dr.propose(9) == [1, 2, 3, 4, 1, 2, 3, 4, 1]


def test_rounds_on_a_periodic_stream():
    stream = [0, 5, 6] + [1, 2, 3, 4] * 100
    r16 = _sim_rounds(stream, 16, 6)
    r64 = _sim_rounds(stream, 64, 6)
    assert r64 < r16 < len(stream) // 8
