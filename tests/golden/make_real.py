"""The real compiled circuit as a fixture: the reference's own compiler, run on CPU in the build
container, then stored compactly so that the GPU box (which has no reference checkout) can load it.

What it builds, with the reference's own code:

- the circuit, ``lx.core.build(lx.merge.config())`` (the merged model's circuit, whose exit leaves
  the output code at +-1), and its chip layers at the merged model's width (hidden 2560, the
  residual slots shared), as ``lx.merge.build`` emits them (lx/lx/merge.py:123-157:
  ``emit.allocate``, ``hf.pick_layout``, ``emit.emit_layers``);
- the chip vocabulary's embedding rows, ``lx.hf.embedding_matrix`` (lx/lx/hf.py:63-93); the
  merged model ties its head to them (its chip rows are the head's rows, lx/lx/merge.py:283);
- a machine: 4.5 MiB of seeded random RAM bytes with a small RV32IM program of this script's own
  at the reset address (a hashing walk over the random data: loads, stores, a multiply, branches,
  a UART byte every 64 iterations), loaded into the circuit's tables by ``lx.core.snapshot``
  (lx/lx/core.py:1374-1414) and placed in the GDN states as ``lx.hf.inject`` places them
  (lx/lx/hf.py:154-166);
- the token trace of that machine from the reference's own machine model (``lx.ref.Machine.step``,
  lx/lx/ref.py:177), GO first: the stream the model alone must reproduce (the reference's
  ``tools/mega_boot.py`` checks its megakernel the same way).

The merged model's final norm is Qwen's own weight, which is not part of the chip; here the
chip's final norm weight is 0 (a gain of 1 on every column): at the exit only the 21 code columns
are nonzero, so any positive gain selects the same row.

Stored in ``real_chip.npz`` (about 6 MB): every projection's nonzeros, the conv taps, the per-head
parameters and norms, the embedding's 222 nonzero columns, the machine's program and RAM seed,
the layout of RAM and ROM in the states (which (layer, key head) holds which RAM block or ROM
head), the other tables' initial rows verbatim, a digest of the whole initial state, and the
trace. ``linuxformer_b200.chip.real`` / ``real_state`` rebuild the chip and the state from it.

    LXB_REFERENCE=<checkout> python tests/golden/make_real.py
"""

import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
REF = os.environ.get("LXB_REFERENCE")
OUT = HERE / "real_chip.npz"
RAM_SEED = 11
N_TRACE = 524_288

from linuxformer_b200 import chip as C  # noqa: E402


# --- the machine's program: RV32IM, assembled here ---------------------------------------------
def _r(f7, rs2, rs1, f3, rd, op=0x33):
    return f7 << 25 | rs2 << 20 | rs1 << 15 | f3 << 12 | rd << 7 | op


def _i(imm, rs1, f3, rd, op=0x13):
    return (imm & 0xFFF) << 20 | rs1 << 15 | f3 << 12 | rd << 7 | op


def _s(imm, rs2, rs1, f3):
    return ((imm >> 5) & 0x7F) << 25 | rs2 << 20 | rs1 << 15 | f3 << 12 | (imm & 0x1F) << 7 | 0x23


def _b(off, rs2, rs1, f3):
    o = off & 0x1FFF
    return (((o >> 12) & 1) << 31 | ((o >> 5) & 0x3F) << 25 | rs2 << 20 | rs1 << 15 | f3 << 12
            | ((o >> 1) & 0xF) << 8 | ((o >> 11) & 1) << 7 | 0x63)


def _u(imm20, rd):
    return (imm20 & 0xFFFFF) << 12 | rd << 7 | 0x37


def _j(off, rd):
    o = off & 0x1FFFFF
    return (((o >> 20) & 1) << 31 | ((o >> 1) & 0x3FF) << 21 | ((o >> 11) & 1) << 20
            | ((o >> 12) & 0xFF) << 12 | rd << 7 | 0x6F)


def program() -> bytes:
    """s0 walks RAM from 0x80100000 by 8 + a byte it loads (so the addresses depend on the data);
    each step hashes two loaded words into s2 (xor, rotate by 5, add their product) and stores
    it back; every 64 steps a byte of the hash goes to the UART; s0 wraps at 0x80400000."""
    p = [_u(0x80100, 8), _u(0x10000, 9), _i(0x5A5, 0, 0, 18)]
    outer = len(p)
    p += [_i(64, 0, 0, 19)]
    inner = len(p)
    p += [_i(0, 8, 2, 5, 0x03), _i(4, 8, 2, 6, 0x03),      # lw t0, 0(s0); lw t1, 4(s0)
          _r(0, 6, 5, 0, 7), _r(0, 7, 18, 4, 18),          # add t2, t0, t1; xor s2, s2, t2
          _i(5, 18, 1, 28), _i(27, 18, 5, 29),             # slli t3, s2, 5; srli t4, s2, 27
          _r(0, 29, 28, 6, 18), _r(1, 6, 5, 0, 30),        # or s2, t3, t4; mul t5, t0, t1
          _r(0, 30, 18, 0, 18), _s(0, 18, 8, 2),           # add s2, s2, t5; sw s2, 0(s0)
          _i(9, 8, 4, 31, 0x03), _r(0, 31, 8, 0, 8),       # lbu t6, 9(s0); add s0, s0, t6
          _i(8, 8, 0, 8), _i(-4, 8, 7, 8),                 # addi s0, s0, 8; andi s0, s0, -4
          _i(-1, 19, 0, 19)]                               # addi s3, s3, -1
    p += [_b((inner - len(p)) * 4, 0, 19, 1)]              # bne s3, zero, inner
    p += [_i(63, 18, 7, 10), _i(48, 10, 0, 10), _s(0, 10, 9, 0),  # a0 = '0' + (s2 & 63) -> UART
          _u(0x80400, 7)]
    p += [_b((outer - len(p)) * 4, 7, 8, 6)]               # bltu s0, t2, outer
    p += [_u(0x80100, 8)]
    p += [_j((outer - len(p)) * 4, 0)]                     # j outer
    return np.array(p, dtype="<u4").tobytes()


def machine_ram(ram_size: int, seed: int = RAM_SEED) -> bytearray:
    ram = bytearray(np.random.default_rng(seed).integers(0, 256, ram_size, dtype=np.uint8)
                    .tobytes())
    prog = program()
    ram[:len(prog)] = prog
    return ram


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    if not REF:
        sys.exit("set LXB_REFERENCE to the reference checkout's directory")
    sys.path.insert(0, str(Path(REF) / "lx"))
    from lx import core, hf, merge
    from lx import ref as R
    from lx import spec as S
    from lx.emit import allocate, emit_layers

    t0 = time.time()
    cfg = merge.config()
    c = core.build(cfg)
    keep = set(c.keep)
    alloc = allocate(c, None, keep, c.target.intermediate)
    lay = hf.pick_layout(alloc.n_slots + 1, C.H)
    lay.slots = alloc.slots
    assert (c.target.key_heads, c.target.value_heads, c.target.intermediate) == \
        (C.NK, C.NV, C.INTER)
    tc = dict(hf.BASE, hidden_size=C.H, linear_key_head_dim=hf.KD, linear_value_head_dim=hf.VD,
              linear_num_key_heads=C.NK, linear_num_value_heads=C.NV,
              intermediate_size=C.INTER)
    # the merged model's eps (Qwen's 1e-6, scaled for the wider key dim): lx/lx/merge.py:151
    eps = 1e-6 * 128 / hf.KD
    sd = emit_layers(c, lay, tc, 0, "model.", alloc, keep, dtype=torch.bfloat16)
    print(f"circuit and layers: {time.time() - t0:.0f} s", flush=True)
    arrs = {}
    for L in range(c.n_layers()):
        p = f"model.layers.{L}."
        for f, k in C.REAL_MATS:
            w = sd.pop(p + k)
            nz = (w != 0).nonzero()
            arrs[f"L{L}.{f}.cnt"] = torch.bincount(nz[:, 0], minlength=w.shape[0]).numpy() \
                .astype(np.int32)
            arrs[f"L{L}.{f}.idx"] = nz[:, 1].numpy().astype(np.int32)
            arrs[f"L{L}.{f}.val"] = _bits(w[nz[:, 0], nz[:, 1]])
        arrs[f"L{L}.conv"] = _bits(sd.pop(p + "linear_attn.conv1d.weight")[:, 0, :])
        for f, k in C.REAL_VECS:
            arrs[f"L{L}.{f}"] = _bits(sd.pop(p + k))
    assert not sd, list(sd)[:4]
    emb = hf.embedding_matrix(c, lay).to(torch.bfloat16)
    cols = (emb != 0).any(0).nonzero()[:, 0]
    arrs["emb_cols"] = cols.numpy().astype(np.int32)
    arrs["emb_vals"] = _bits(emb[:, cols])
    del emb
    # the machine and its state
    ram = machine_ram(cfg.ram_size)
    m = R.Machine(ram, cfg.text_end, {})
    core.snapshot(c, m)
    name_of = {id(node): name for name, node in c.tables.items()}
    ram_map, rom_map, init_idx, init_rows = [], [], [], []
    for i, (L, j) in hf.head_slots(c).items():
        node = c.nodes[i]
        if not node.init:
            continue
        name = name_of.get(id(node), "")
        if name.startswith("ram") and name[3:].isdigit():
            ram_map.append((int(name[3:]), L, j))
            continue
        if name.startswith("rom") and name[3:].isdigit():
            rom_map.append((int(name[3:]), L, j))
            continue
        for x, rows in enumerate(node.init):
            for r, v in (rows or {}).items():
                init_idx.append((L, j * C.R + x, r))
                init_rows.append(np.asarray(v, np.float32))
    arrs["ram_map"] = np.array(sorted(ram_map), np.int32).reshape(-1, 3)
    arrs["rom_map"] = np.array(sorted(rom_map), np.int32).reshape(-1, 3)
    arrs["init_idx"] = np.array(init_idx, np.int32).reshape(-1, 3)
    arrs["init_rows"] = np.array(init_rows, np.float32).reshape(-1, C.VD)
    arrs["program"] = np.frombuffer(program(), np.uint8)
    # the reference's own state, as hf.inject writes it, to pin the rebuild below
    rec = np.zeros((c.n_layers(), C.NV, C.KD, C.VD), np.float32)
    for i, (L, j) in hf.head_slots(c).items():
        for x, rows in enumerate(c.nodes[i].init or []):
            for r, v in (rows or {}).items():
                rec[L, j * C.R + x, r] = v
    from lx.core import RAM_HEAD_WORDS, ROM_HEAD_WORDS
    from lx.ir import A_BIT, A_REF, REF_COLS
    meta = dict(eps=eps, vocab=S.VOCAB, n_embed=int(arrs["emb_vals"].shape[0]),
                ram_size=cfg.ram_size, text_end=cfg.text_end, text_words=cfg.text_words,
                ram_seed=RAM_SEED,
                ram_sha256=hashlib.sha256(bytes(ram)).hexdigest(),
                ram_head_words=RAM_HEAD_WORDS, rom_head_words=ROM_HEAD_WORDS, a_ref=A_REF,
                a_bit=A_BIT, ref_cols=list(REF_COLS), code_cols=[lay.dim(d) for d in c.keep],
                n_layers=c.n_layers(), go=S.tok("GO"),
                state_sha256=hashlib.sha256(rec.tobytes()).hexdigest())
    # the trace, by the reference's machine model
    m2 = R.Machine(machine_ram(cfg.ram_size), cfg.text_end, {})
    toks = [S.tok("GO")]
    while len(toks) < N_TRACE and not m2.halted:
        toks += m2.step()
    arrs["trace"] = np.array(toks[:N_TRACE], np.int32)
    arrs["meta"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(OUT, **arrs)
    print(f"{OUT.name}: {OUT.stat().st_size / 1e6:.1f} MB", flush=True)
    # the rebuild from the file must give the reference's state bit for bit
    chip = C.real(OUT)
    st = C.real_state(chip)
    assert np.array_equal(st.recurrent.view(np.uint32), rec.view(np.uint32)), "state rebuild"
    assert not st.conv.any()
    print(f"state rebuilt bit for bit; {time.time() - t0:.0f} s", flush=True)


if __name__ == "__main__":
    main()
