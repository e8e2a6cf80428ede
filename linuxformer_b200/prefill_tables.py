"""Host-side table builder for the chunked prefill: a chip (linuxformer_b200.chip.Chip) -> one
prefill plan image for the C ABI (layout in csrc/lxb_prefill.h; lxb_prefill_plan_create validates
every offset and index in it).

This is the B200 counterpart of what the reference's sparse prefill finds per layer
(``Fast._gdn`` / ``Fast._mlp``, lx/lx/fast.py:187-248): the live channels, key heads, value dims,
out_proj rows and MLP units, and the head's columns. The layout is for token-parallel stages:
every table row is applied to a whole chunk of tokens at once.

- Tap channels: in_proj_qkv channels with a nonzero conv tap. Only their conv output can be
  nonzero (with no tap, the conv sum is +0 and silu(+0) = +0), whatever their window holds.
- Live key heads: those with a query or key tap channel. Their live rows (the rows of those
  channels) are the only state rows a query reads or a key writes; the recurrence keeps them in
  registers (at most MAXLIVE per key head), every other row only decays.
- out_proj rows over the live value heads' dims: any other head's output is exactly 0, and the
  stock sums skip a zero term exactly (from +0).
- MLP units whose gate and up rows are nonzero and whose down column is not empty.
- The head: the columns nonzero in every row (at most 32, at most 4 distinct values) as 2-bit
  codes, the rest as CSR rows (the decode plan's rule, lx/lx/mega.py:354-395).
"""

from __future__ import annotations

import numpy as np

from . import chip as C
from .chip import _ranges
from .tables import _Pool, _f32, _pack

MAGIC = 0x46505A4C
VERSION = 1
MAXLIVE = 31
MAXDENSE = 32
SEC = ("layers", "ent", "i32", "u16", "taps", "vhs", "units", "hcodes")

LAYER = np.dtype([(n, "<i4") for n in (
    "ln_in", "ln_post", "gnorm", "tap0", "n_tap", "chan", "khs", "n_kh", "slots", "n_slot",
    "livemask", "vtap", "zrow", "out_ptr", "unit0", "n_units", "down_ptr", "nl", "p0", "p1")])
TAP = np.dtype([("ent", "<u4"), ("n", "<u4"), ("conv_ch", "<u4"), ("t01", "<u4"), ("t23", "<u4"),
                ("pad", "<u4", (3,))])
VH = np.dtype([("a_ent", "<u4"), ("a_n", "<u4"), ("b_ent", "<u4"), ("b_n", "<u4"),
               ("A_log", "<u2"), ("dt_bias", "<u2"), ("pad", "<u4", (3,))])
UNIT = np.dtype([("g", "<u4"), ("u", "<u4"), ("ng", "<u4"), ("nu", "<u4")])
HEADER = np.dtype([("magic", "<u4"), ("version", "<u4"), ("n_layers", "<i4"), ("n_vocab", "<i4"),
                   ("hidden", "<i4"), ("n_dense", "<i4"), ("n_embed_rows", "<i8"),
                   ("offset", "<i4"), ("eps", "<f4"), ("final_norm", "<i4"), ("head_ptr", "<i4"),
                   ("htab", "<f4", (4,)), ("dense_cols", "<i4", (MAXDENSE,)),
                   ("max_tap", "<i4"), ("max_lvh", "<i4"), ("max_slot", "<i4"),
                   ("max_units", "<i4"), ("sec", "<i8", (len(SEC), 2))])
assert LAYER.itemsize == 80 and TAP.itemsize == 32 and VH.itemsize == 32
assert UNIT.itemsize == 16 and HEADER.itemsize == 336


class PrefillUnsupported(ValueError):
    """The chip has a shape the register-resident recurrence does not cover."""


def _row_ent(m: C.Sparse, ent: _Pool, cols_map=None):
    """Every row of m appended to the entry pool: (offsets, counts) per row."""
    idx = m.indices if cols_map is None else cols_map[m.indices]
    base = ent.add(_pack(idx, m.data))
    return (m.indptr[:-1] + base).astype(np.int64), np.diff(m.indptr).astype(np.int64)


def build_image(chip: C.Chip) -> tuple[bytes, dict]:
    ent, i32, u16 = _Pool(np.uint32), _Pool(np.int32), _Pool(np.uint16)
    layers = np.zeros(chip.n_layers, LAYER)
    taps, vhs, units = [], [], []
    stats = {"taps": 0, "live_kh": 0, "live_rows": 0, "units": 0, "out_nnz": 0, "z_nnz": 0}
    max_tap = max_lvh = max_slot = max_units = 0
    n_tap_total = 0
    for L, ly in enumerate(chip.layers):
        rec = layers[L]
        rec["ln_in"], rec["ln_post"] = u16.add(ly.ln_in), u16.add(ly.ln_post)
        rec["gnorm"] = u16.add(ly.gnorm)
        # --- tap channels and the per-channel table -------------------------------------------
        tapm = (ly.conv & 0x7FFF) != 0                       # [CONV, 4]
        tap_ch = np.nonzero(tapm.any(1))[0]
        q_off, q_cnt = _row_ent(ly.qkv, ent)
        tap_of = np.full(C.CONV, -1, np.int64)
        tap_of[tap_ch] = np.arange(len(tap_ch))
        t = np.zeros(len(tap_ch), TAP)
        t["ent"], t["n"], t["conv_ch"] = q_off[tap_ch], q_cnt[tap_ch], tap_ch
        cv = ly.conv.astype(np.uint32)
        t["t01"] = cv[tap_ch, 0] | (cv[tap_ch, 1] << 16)
        t["t23"] = cv[tap_ch, 2] | (cv[tap_ch, 3] << 16)
        rec["tap0"], rec["n_tap"] = n_tap_total, len(tap_ch)
        n_tap_total += len(tap_ch)
        taps.append(t)
        rec["chan"] = i32.add(np.stack([tap_of, q_off, q_cnt], 1).astype(np.int32))
        # --- live key heads and their slots ------------------------------------------------------
        khs, slots = [], []
        livemask = np.zeros((C.NK, 8), np.uint32)
        nl_max = 0
        for kh in range(C.NK):
            qt = tap_of[kh * C.KD:(kh + 1) * C.KD]
            kt = tap_of[C.NK * C.KD + kh * C.KD:C.NK * C.KD + (kh + 1) * C.KD]
            rows = np.nonzero((qt >= 0) | (kt >= 0))[0]
            if not len(rows):
                continue
            if len(rows) > MAXLIVE:
                raise PrefillUnsupported(
                    f"layer {L} key head {kh}: {len(rows)} live rows (at most {MAXLIVE})")
            khs.append((kh, len(slots), len(rows)))
            nl_max = max(nl_max, len(rows))
            for r in rows:
                slots.append((r, qt[r], kt[r]))
                livemask[kh, r // 32] |= np.uint32(1 << (r % 32))
        rec["khs"], rec["n_kh"] = i32.add(np.array(khs, np.int32).reshape(-1, 3)), len(khs)
        rec["slots"], rec["n_slot"] = i32.add(np.array(slots, np.int32).reshape(-1, 3)), len(slots)
        rec["livemask"] = i32.add(livemask.view(np.int32))
        rec["nl"] = nl_max
        stats["live_kh"] += len(khs)
        stats["live_rows"] += len(slots)
        live_kh = np.array([k[0] for k in khs], np.int64)
        n_lvh = len(live_kh) * C.R
        # live value dims, in (live key head, value head, column) order
        vh_of_lvh = (live_kh[:, None] * C.R + np.arange(C.R)).reshape(-1)
        dims = (vh_of_lvh[:, None] * C.VD + np.arange(C.VD)).reshape(-1)
        vch = 2 * C.NK * C.KD + dims
        rec["vtap"] = i32.add(tap_of[vch].astype(np.int32))
        z_off, z_cnt = _row_ent(ly.z, ent)
        rec["zrow"] = i32.add(np.stack([z_off[dims], z_cnt[dims]], 1).astype(np.int32))
        stats["z_nnz"] += int(z_cnt[dims].sum())
        # out_proj rows over the live dims only, indexed by live dim
        live_of = np.full(C.ZD, -1, np.int64)
        live_of[dims] = np.arange(len(dims))
        o = ly.out
        keep = live_of[o.indices] >= 0
        rows_of = np.repeat(np.arange(C.H), o.row_nnz())[keep]
        ptr = np.zeros(C.H + 1, np.int64)
        np.cumsum(np.bincount(rows_of, minlength=C.H), out=ptr[1:])
        base = ent.add(_pack(live_of[o.indices[keep]], o.data[keep]))
        rec["out_ptr"] = i32.add((ptr + base).astype(np.int32))
        stats["out_nnz"] += int(keep.sum())
        # per value head: in_proj_a / in_proj_b rows and the decay parameters (all 128 heads:
        # every state decays, live or not)
        a_off, a_cnt = _row_ent(ly.a, ent)
        b_off, b_cnt = _row_ent(ly.b, ent)
        v = np.zeros(C.NV, VH)
        v["a_ent"], v["a_n"], v["b_ent"], v["b_n"] = a_off, a_cnt, b_off, b_cnt
        v["A_log"], v["dt_bias"] = ly.A_log, ly.dt_bias
        vhs.append(v)
        # --- the MLP ---------------------------------------------------------------------------
        g_n, u_n = ly.gate.row_nnz(), ly.up.row_nnz()
        d_col = np.bincount(ly.down.indices, minlength=C.INTER) if ly.down.nnz else \
            np.zeros(C.INTER, np.int64)
        live_u = np.nonzero((g_n > 0) & (u_n > 0) & (d_col > 0))[0]
        # each live unit's gate entries, then its up entries, contiguous (one list per unit)
        gs, us = ly.gate.rows_subset(live_u), ly.up.rows_subset(live_u)
        gu_cnt = gs.row_nnz() + us.row_nnz()
        gu_ptr = np.zeros(len(live_u) + 1, np.int64)
        np.cumsum(gu_cnt, out=gu_ptr[1:])
        gu_idx = np.zeros(int(gu_ptr[-1]), np.int64)
        gu_bits = np.zeros(int(gu_ptr[-1]), np.uint16)
        g_pos = _ranges(gu_ptr[:-1], gs.row_nnz())
        u_pos = _ranges(gu_ptr[:-1] + gs.row_nnz(), us.row_nnz())
        gu_idx[g_pos], gu_bits[g_pos] = gs.indices, gs.data
        gu_idx[u_pos], gu_bits[u_pos] = us.indices, us.data
        base = ent.add(_pack(gu_idx, gu_bits))
        un = np.zeros(len(live_u), UNIT)
        un["g"], un["ng"] = base + gu_ptr[:-1], gs.row_nnz()
        un["u"], un["nu"] = base + gu_ptr[:-1] + gs.row_nnz(), us.row_nnz()
        rec["unit0"], rec["n_units"] = sum(len(x) for x in units), len(live_u)
        units.append(un)
        unit_of = np.full(C.INTER, -1, np.int64)
        unit_of[live_u] = np.arange(len(live_u))
        d = ly.down
        keep = unit_of[d.indices] >= 0 if d.nnz else np.zeros(0, bool)
        rows_of = np.repeat(np.arange(C.H), d.row_nnz())[keep]
        ptr = np.zeros(C.H + 1, np.int64)
        np.cumsum(np.bincount(rows_of, minlength=C.H), out=ptr[1:])
        base = ent.add(_pack(unit_of[d.indices[keep]], d.data[keep]))
        rec["down_ptr"] = i32.add((ptr + base).astype(np.int32))
        stats["taps"] += len(tap_ch)
        stats["units"] += len(live_u)
        max_tap, max_lvh = max(max_tap, len(tap_ch)), max(max_lvh, n_lvh)
        max_slot, max_units = max(max_slot, len(slots)), max(max_units, len(live_u))
    # --- the head --------------------------------------------------------------------------------
    hd = chip.head
    V = hd.shape[0]
    col_cnt = np.bincount(hd.indices, minlength=C.H)
    dense = np.nonzero(col_cnt == V)[0] if V else np.zeros(0, np.int64)
    htab = np.zeros(4, np.float32)
    ok = 0 < len(dense) <= MAXDENSE
    if ok:
        isd = np.isin(hd.indices, dense)
        vals = np.unique(_f32(hd.data[isd]))
        ok = len(vals) <= 4
    if not ok:
        dense = dense[:0]
    rows_of = np.repeat(np.arange(V), hd.row_nnz())
    hcodes = np.zeros(V if len(dense) else 0, np.uint64)
    if len(dense):
        htab[:len(vals)] = vals
        isd = np.isin(hd.indices, dense)
        code = np.searchsorted(vals, _f32(hd.data[isd])).astype(np.uint64)
        j = np.searchsorted(dense, hd.indices[isd]).astype(np.uint64)
        np.bitwise_or.at(hcodes, rows_of[isd], code << (np.uint64(2) * j))
        sp = ~isd
    else:
        sp = np.ones(hd.nnz, bool)
    sp_ptr = np.zeros(V + 1, np.int64)
    np.cumsum(np.bincount(rows_of[sp], minlength=V), out=sp_ptr[1:])
    sp_base = ent.add(_pack(hd.indices[sp], hd.data[sp]))
    head_ptr = i32.add((sp_ptr + sp_base).astype(np.int32))
    final_norm = u16.add(chip.final_norm)
    assert ent.n < 1 << 31 and i32.n < 1 << 31 and u16.n < 1 << 31
    stats.update(head_dense=len(dense), head_sparse_nnz=int(sp.sum()), ent=ent.n,
                 max_tap=max_tap, max_lvh=max_lvh, max_slot=max_slot, max_units=max_units)
    # --- the image -------------------------------------------------------------------------------
    cat = lambda parts, dt: np.concatenate(parts) if parts else np.zeros(0, dt)  # noqa: E731
    secs = [layers, ent.array(), i32.array(), u16.array(), cat(taps, TAP), cat(vhs, VH),
            cat(units, UNIT), hcodes]
    hdr = np.zeros(1, HEADER)[0]
    hdr["magic"], hdr["version"] = MAGIC, VERSION
    hdr["n_layers"], hdr["n_vocab"], hdr["hidden"], hdr["n_dense"] = chip.n_layers, V, C.H, \
        len(dense)
    hdr["n_embed_rows"], hdr["offset"], hdr["eps"] = chip.embed.shape[0], chip.offset, chip.eps
    hdr["final_norm"], hdr["head_ptr"] = final_norm, head_ptr
    hdr["htab"] = htab
    hdr["dense_cols"][:len(dense)] = dense
    hdr["max_tap"], hdr["max_lvh"], hdr["max_slot"], hdr["max_units"] = \
        max_tap, max_lvh, max_slot, max_units
    blobs, pos = [], HEADER.itemsize
    for k, a in enumerate(secs):
        pos = -(-pos // 16) * 16
        b = np.ascontiguousarray(a).tobytes()
        hdr["sec"][k] = (pos, len(a))
        blobs.append((pos, b))
        pos += len(b)
    image = bytearray(-(-pos // 16) * 16)
    image[:HEADER.itemsize] = np.array([hdr], HEADER).tobytes()
    for p, b in blobs:
        image[p:p + len(b)] = b
    stats["image_bytes"] = len(image)
    return bytes(image), stats
