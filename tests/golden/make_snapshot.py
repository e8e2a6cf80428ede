"""A snapshot file written by the reference's own writer, for the snapshot reader's test.

The reference saves a session with ``lx.session.save_safe`` (lx/lx/session.py:259-278): tensors
``conv.L`` / ``recurrent.L``, the proposer machine's byte fields as ``ref.<name>`` uint8 tensors,
the other fields as JSON under the metadata key ``lx.session``. This script imports that writer
from the reference's checkout and saves a small two-layer state (the layout does not depend on
the tensor shapes, so small tensors keep the fixture at a few KB) with host fields of every kind.
tests/test_snapshot.py rebuilds the same values with ``fixture()`` below and reads the file.

Run where the reference's checkout is (its directory in LXB_REFERENCE); the tests only read
the .safetensors file:

    python tests/golden/make_snapshot.py
"""

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

OUT = Path(__file__).resolve().parent / "snapshot_ref.safetensors"


def fixture():
    """The values saved: (state, host fields, machine fields)."""
    g = torch.Generator().manual_seed(11)
    state = []
    for L in range(2):
        conv = (torch.randn(6, 4, generator=g) * (L + 1)).to(torch.bfloat16)
        rec = torch.randn(3, 4, 5, generator=g)
        rec[0, 1, 2] = -0.0
        state.append((conv, rec))
    host = {"next": 1234, "last": 77, "n": 4096, "waiting": True}
    ref = {"pc": 0x80000000, "cycle": 123456789, "regs": [0, 1, 2, 3], "ram": bytearray(b"\x00\x01ram"),
           "out": b"console\n", "empty": b""}
    return state, host, ref


def main():
    ref = os.environ.get("LXB_REFERENCE")
    if not ref:
        sys.exit("set LXB_REFERENCE to the reference checkout's directory")
    sys.path.insert(0, ref + "/lx")
    from lx.session import save_safe

    state, host, ref = fixture()
    save_safe(dict(host, state=state, ref=SimpleNamespace(**ref)), OUT)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
