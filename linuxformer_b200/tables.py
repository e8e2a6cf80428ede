"""Host-side table builder: a chip (linuxformer_b200.chip.Chip) -> one plan image for the C ABI
(layout in csrc/lxb_plan.h; lxb_plan_create validates every offset and index in it).

This is the B200 counterpart of the reference's Fast._gdn/_mlp/_dec (which find the nonzero rows
and columns, lx/lx/fast.py:187-248, 432-469) and Mega.__init__ (which packs them into CSR/CSC
tables, per-CTA blobs and a phase schedule, lx/lx/mega.py:199-504). What is kept:

- live channels: rows of in_proj_qkv with any weight (their conv windows are state);
- items: key heads with a live channel, or whose value heads can decay;
- live MLP units: gate, up and down all nonzero (fast.py:240-245);
- the head: the columns nonzero in every row (at most 32, at most 4 distinct values) as 2-bit
  codes, the rest as sparse rows (mega.py:354-395).

What differs: the layout is for a cluster of C CTAs per stream. Each owner gets the down_proj and
out_proj entries of its residual rows in CSR order (so every sum is taken by one thread, in
column order) and the list of MLP units those rows need. The out_proj rows are owned in blocks
of 2560 / C; an MLP layer's rows are split per layer in contiguous ranges balanced by their work
(only the rows the MLP can change, around the CTAs' items). Items are spread over the CTAs, at
most LXB_ITEMSLOTS per CTA per layer.
"""

from __future__ import annotations

import numpy as np

from . import chip as C
from .chip import _ranges

MAGIC = 0x50425A4C
VERSION = 10
NSLOT, NOSLOT = 1536, 0xFFFF
ITEMSLOTS, MAXDENSE, MAXUNITS, MAXWIN = 4, 32, 2048, 1024
MINC = 4  # the smallest cluster: an owner holds at most H / MINC rows
# the MLP row split's cost model, in gate/up products: an item on the CTA (the step's average),
# and each owned row (its down sum and its push)
ITEM_COST, ROW_COST = 1000, 2
HEADSLICES = 32
IT_DECAYS, IT_OUT, IT_NONRES = 1, 2, 4
SEC = ("layers", "items", "chans", "ent", "units", "owners", "i32", "u16", "headcta", "hcodes",
       "blobs", "blobidx", "winmap", "winidx")

LAYER = np.dtype([(n, "<i4") for n in ("has_gdn", "has_mlp", "ln_in", "ln_post", "item0",
                                       "n_items", "owner0", "itemof", "decays", "mrow0",
                                       "mrow1", "p2")])
ITEM = np.dtype([(n, "<i4") for n in ("layer", "kh", "cta", "slot", "ch0", "n_ch", "rows",
                                      "params", "flags", "n_eager", "n_vneed", "tapu")])
CHAN = np.dtype([("ent", "<u4"), ("n", "<u2"), ("slot", "<u2"), ("conv_ch", "<u4"),
                 ("t01", "<u4"), ("t23", "<u4"), ("tapmask", "<u4"), ("win", "<u4"),
                 ("p2", "<u4")])
UNIT = np.dtype([("g", "<u4"), ("u", "<u4"), ("ng", "<u2"), ("nu", "<u2"), ("pad", "<u4")])
OWNER = np.dtype([("mr0", "<i4"), ("mr1", "<i4"), ("nlong", "<i4"), ("orow", "<i4")])
HEADCTA = np.dtype([("r0", "<i4"), ("r1", "<i4"), ("rowptr", "<i4"), ("pad", "<i4")])
HEADER = np.dtype([("magic", "<u4"), ("version", "<u4"), ("n_layers", "<i4"), ("cluster", "<i4"),
                   ("n_vocab", "<i4"), ("hidden", "<i4"), ("n_items", "<i4"), ("n_dense", "<i4"),
                   ("n_embed_rows", "<i8"), ("offset", "<i4"), ("eps", "<f4"),
                   ("final_norm", "<i4"), ("pad0", "<i4"), ("htab", "<f4", (4,)),
                   ("dense_cols", "<i4", (MAXDENSE,)), ("blob_max", "<i4"), ("hsp_mask", "<i4"),
                   ("pad1", "<i4", (2,)),
                   ("sec", "<i8", (len(SEC), 2))])
LONG = 32  # rows with more entries are summed by a warp each (LXB_LONG)
BLOBREF = np.dtype([("off", "<i8"), ("bytes", "<i4"), ("pad", "<i4")])
BHDR = np.dtype([("bytes", "<i4"), ("n_items", "<i4"), ("item", "<i4", (ITEMSLOTS,)),
                 ("ln_in", "<i4"), ("ln_post", "<i4"), ("mlp", "<i4"), ("pad", "<i4", (7,))])
BITEM = np.dtype([(n, "<i4") for n in ("item", "n_eager", "eager", "rows", "prm", "kh", "slot",
                                       "flags", "z")] + [("pad", "<i4", (7,))])
BCHAN = np.dtype([("ent", "<i4"), ("n", "<u2"), ("slot", "<u2"), ("conv_ch", "<u4"),
                  ("t01", "<u4"), ("t23", "<u4"), ("win", "<u4"), ("p1", "<u4"), ("p2", "<u4")])
BMLP = np.dtype([(n, "<i4") for n in ("n_units", "units", "down_ptr", "down_ent", "r0", "nr",
                                      "nlong", "p1")])
BUNIT = np.dtype([("g", "<i4"), ("u", "<i4"), ("ng", "<u2"), ("nu", "<u2"), ("pad", "<i4")])
assert LAYER.itemsize == 48 and ITEM.itemsize == 48 and CHAN.itemsize == 32
assert UNIT.itemsize == 16 and OWNER.itemsize == 16 and HEADCTA.itemsize == 16
assert HEADER.itemsize == 440 and BLOBREF.itemsize == 16 and BHDR.itemsize == 64
assert BITEM.itemsize == 64 and BCHAN.itemsize == 32 and BMLP.itemsize == 32
assert BUNIT.itemsize == 16


class _Blob:
    """One step blob: 16-aligned pieces appended to a bytearray."""

    def __init__(self):
        self.b = bytearray(BHDR.itemsize)

    def add(self, a) -> int:
        off = -(-len(self.b) // 16) * 16
        self.b.extend(bytes(off - len(self.b)))
        self.b.extend(np.ascontiguousarray(a).tobytes())
        return off

    def done(self, hdr) -> bytes:
        self.b.extend(bytes(-len(self.b) % 16))
        hdr["bytes"] = len(self.b)
        self.b[:BHDR.itemsize] = np.array([hdr], BHDR).tobytes()
        return bytes(self.b)


class _Pool:
    """A growing flat array (entries, int32, uint16)."""

    def __init__(self, dtype):
        self.dtype, self.parts, self.n = dtype, [], 0

    def add(self, a) -> int:
        a = np.ascontiguousarray(a, self.dtype).reshape(-1)
        off = self.n
        if a.size:
            self.parts.append(a)
            self.n += a.size
        return off

    def array(self) -> np.ndarray:
        return np.concatenate(self.parts) if self.parts else np.zeros(0, self.dtype)


def _pack(idx, bits) -> np.ndarray:
    """(index < 2^16, bf16 bits) -> uint32 entries."""
    idx = np.asarray(idx, np.int64)
    assert idx.size == 0 or (idx.min() >= 0 and idx.max() < 1 << 16)
    return (idx.astype(np.uint32) | (np.asarray(bits, np.uint32) << 16)).astype(np.uint32)


def _f32(bits) -> np.ndarray:
    return C.bf16_float(bits)


def _may_decay(layer: C.Layer, vh: np.ndarray) -> np.ndarray:
    """Whether g = -exp(A_log) * softplus(a + dt_bias) can ever be nonzero, per value head:
    with an empty in_proj_a row a is always 0, and exp(x) is 0 in fp32 below -103.97, so
    softplus(dt_bias) (and -exp(A_log)) is then exactly zero."""
    a_nnz = layer.a.row_nnz()[vh]
    return ((a_nnz > 0) | (_f32(layer.dt_bias[vh]) >= -103.98)) & \
        (_f32(layer.A_log[vh]) >= -103.98)


def _cta_order(Cn: int, L: int) -> np.ndarray:
    """The CTAs a layer's items go to, in order: a rotation by the layer index, so that the
    ranks without an item change from layer to layer."""
    return np.argsort((np.arange(Cn) - 3 * L) % Cn, kind="stable")


def _mlp_split(layer: C.Layer, live: np.ndarray, base: np.ndarray) -> np.ndarray:
    """The owners' MLP rows: bounds R[0..Cn] (multiples of 8) with owner c holding [R[c], R[c+1]),
    the ranges tiling the rows the MLP can change (those with a live unit's down weight, rounded
    out to 8) in rank order, and the largest of base[c] + the range's cost as small as it can be
    (cost: the gate/up entries of the rows' units and ROW_COST a row; base: the owner's items).
    Without an MLP every range is empty."""
    Cn = len(base)
    d = layer.down
    rowid = np.repeat(np.arange(C.H), d.row_nnz())
    keep = live[d.indices]
    R = np.zeros(Cn + 1, np.int64)
    if not keep.any():
        return R
    g_cnt, u_cnt = layer.gate.row_nnz(), layer.up.row_nnz()
    u = d.indices[keep]
    rc = np.bincount(rowid[keep], weights=(g_cnt[u] + u_cnt[u]).astype(np.float64),
                     minlength=C.H).astype(np.int64) + ROW_COST
    act = np.nonzero(np.bincount(rowid[keep], minlength=C.H))[0]
    a, b = int(act[0]) & ~7, (int(act[-1]) + 8) & ~7
    ck = rc[a:b].reshape(-1, 8).sum(1)
    cap = C.H // MINC // 8  # chunks of 8 rows an owner may hold

    def fit(T):
        out = np.full(Cn + 1, b, np.int64)
        out[0], c, cur, n = a, 0, int(base[0]), 0
        for j, w in enumerate(ck.tolist()):
            while cur + w > T or n == cap:
                c += 1
                if c == Cn:
                    return None
                out[c], cur, n = a + 8 * j, int(base[c]), 0
            cur += w
            n += 1
        return out

    lo, hi = 0, int(ck.sum() + base.max())
    while fit(hi) is None:  # (the row cap alone can leave no split: only if Cn * cap < chunks)
        hi *= 2
    while lo < hi:
        mid = (lo + hi) // 2
        if fit(mid) is None:
            lo = mid + 1
        else:
            hi = mid
    return fit(lo)


def build_image(chip: C.Chip, cluster: int = 16) -> tuple[bytes, dict]:
    """The plan image for `chip` on clusters of `cluster` CTAs, and build statistics."""
    Cn = cluster
    assert Cn in (4, 8, 16) and C.H % Cn == 0
    blk = C.H // Cn
    ent, i32, u16 = _Pool(np.uint32), _Pool(np.int32), _Pool(np.uint16)
    layers = np.zeros(chip.n_layers, LAYER)
    items, chans, units, owners = [], [], [], []
    parts, blobs = {}, []
    winmap = [[] for _ in range(Cn)]  # per CTA: its resident (layer, conv channel) windows
    stats = {"cluster": Cn, "items": 0, "chans": 0, "csr_nnz": 0, "units": 0, "unit_evals": 0,
             "down_nnz": 0, "out_nnz": 0}
    for L, ly in enumerate(chip.layers):
        rec = layers[L]
        rec["ln_in"] = u16.add(ly.ln_in)
        rec["ln_post"] = u16.add(ly.ln_post)
        rec["owner0"] = L * Cn
        # --- GDN items ---------------------------------------------------------------------
        qkv = ly.qkv
        cnt = qkv.row_nnz()
        live = np.nonzero(cnt > 0)[0]
        if len(live):
            assert cnt.max() < 1 << 16
        kh_of = np.where(live < C.NK * C.KD, live // C.KD,
                         np.where(live < 2 * C.NK * C.KD, (live - C.NK * C.KD) // C.KD,
                                  (live - 2 * C.NK * C.KD) // C.VD // C.R))
        slot_of = np.where(live < C.NK * C.KD, live % C.KD,
                           np.where(live < 2 * C.NK * C.KD, C.KD + (live - C.NK * C.KD) % C.KD,
                                    2 * C.KD + (live - 2 * C.NK * C.KD) % (C.R * C.VD)))
        decays_vh = _may_decay(ly, np.arange(C.NV))
        heads = sorted(set(kh_of.tolist()) |
                       set(np.nonzero(decays_vh.reshape(C.NK, C.R).any(1))[0].tolist()))
        assert len(heads) <= ITEMSLOTS * Cn, "more key heads in a layer than the cluster holds"
        rec["item0"] = len(items)
        rec["n_items"] = len(heads)
        itemof = np.full(C.NK, -1, np.int32)
        out_cols = ly.out.transpose()  # CSC by value dim
        out_has = out_cols.row_nnz().reshape(C.NK, C.R * C.VD).any(1)
        # the row entries of the whole in_proj_qkv, packed once
        qkv_ent0 = ent.add(_pack(qkv.indices, qkv.data))
        stats["csr_nnz"] += qkv.nnz
        # the items over the CTAs (the MLP rows are split around them below)
        cta_order = _cta_order(Cn, L)
        for k, kh in enumerate(heads):
            cta_k, slot_k = int(cta_order[k % Cn]), k // Cn
            sel = np.nonzero(kh_of == kh)[0]
            # order: eager (query/key with a tap) | value with a tap | the rest (window only)
            tapped = (ly.conv[live[sel]] & 0x7FFF).any(1)
            isqk = slot_of[sel] < 2 * C.KD
            cls = np.where(tapped & isqk, 0, np.where(tapped, 1, 2))
            order = np.argsort(cls, kind="stable")
            sel, cls = sel[order], cls[order]
            chs = live[sel]
            ch = np.zeros(len(chs), CHAN)
            ch["ent"] = qkv_ent0 + qkv.indptr[chs]
            ch["n"] = cnt[chs]
            ch["slot"] = slot_of[sel]
            ch["conv_ch"] = chs
            taps = ly.conv[chs].astype(np.uint32)
            ch["t01"] = taps[:, 0] | (taps[:, 1] << 16)
            ch["t23"] = taps[:, 2] | (taps[:, 3] << 16)
            ch["tapmask"] = ((taps & 0x7FFF) != 0).astype(np.uint32) @ (1 << np.arange(4))
            ch["win"] = 0xFFFFFFFF
            assert len(chs) <= 2 * NSLOT
            ch0 = sum(len(c) for c in chans)
            chans.append(ch)
            vh = kh * C.R + np.arange(C.R)
            refs = np.zeros((2 * C.R + C.R * C.VD, 2), np.int32)
            zrows = (vh[:, None] * C.VD + np.arange(C.VD)).reshape(-1)
            for q0, m, rr in ((0, ly.b, vh), (C.R, ly.a, vh), (2 * C.R, ly.z, zrows)):
                sub = m.rows_subset(rr)
                n = sub.row_nnz()
                base = ent.add(_pack(sub.indices, sub.data))
                refs[q0:q0 + len(rr), 0] = np.where(n > 0, base + sub.indptr[:-1], 0)
                refs[q0:q0 + len(rr), 1] = n
            it = np.zeros(1, ITEM)[0]
            it["layer"], it["kh"], it["cta"], it["slot"] = L, kh, cta_k, slot_k
            it["ch0"], it["n_ch"] = ch0, len(chs)
            it["n_eager"], it["n_vneed"] = int((cls == 0).sum()), int((cls == 1).sum())
            it["tapu"] = int(np.bitwise_or.reduce(ch["tapmask"][cls == 1], initial=0))
            it["rows"] = i32.add(refs)
            it["params"] = u16.add(np.concatenate([ly.A_log[vh], ly.dt_bias[vh], ly.gnorm]))
            it["flags"] = (IT_DECAYS if decays_vh[vh].any() else 0) | \
                (IT_OUT if out_has[kh] else 0)
            # the item's part of its CTA's step blob: query/key channels with their entries,
            # the beta / a rows, the head's parameters
            ne = int((cls == 0).sum())
            e_ch = chs[:ne]
            e_ent = [_pack(qkv.indices[qkv.indptr[c]:qkv.indptr[c + 1]],
                           qkv.data[qkv.indptr[c]:qkv.indptr[c + 1]]) for c in e_ch]
            ba = [(m.indices[m.indptr[v]:m.indptr[v + 1]], m.data[m.indptr[v]:m.indptr[v + 1]])
                  for m in (ly.b, ly.a) for v in vh]
            zsub = ly.z.rows_subset(zrows) if out_has[kh] else None
            parts[len(items)] = dict(chan=ch[:ne].copy(), ent=e_ent,
                                     ba=[_pack(i_, d_) for i_, d_ in ba],
                                     prm=np.concatenate([ly.A_log[vh], ly.dt_bias[vh], ly.gnorm]),
                                     z=zsub)
            itemof[kh] = len(items)
            items.append(it)
            stats["chans"] += len(chs)
        stats["items"] += len(heads)
        rec["itemof"] = i32.add(itemof)
        rec["has_gdn"] = int(len(heads) > 0)
        rec["decays"] = int(any(items[i]["flags"] & IT_DECAYS for i in
                                range(rec["item0"], rec["item0"] + len(heads))))
        # --- owners: MLP units and the rows' down_proj / out_proj entries --------------------
        g_cnt, u_cnt = ly.gate.row_nnz(), ly.up.row_nnz()
        d_cols = ly.down.transpose()
        unit_live = (g_cnt > 0) & (u_cnt > 0) & (d_cols.row_nnz() > 0)
        assert g_cnt.max(initial=0) < 1 << 16 and u_cnt.max(initial=0) < 1 << 16
        rec["has_mlp"] = int(unit_live.any())
        stats["units"] += int(unit_live.sum())
        item_heads = np.zeros(C.NK, bool)
        item_heads[heads] = True
        n_it = np.bincount([int(items[i]["cta"]) for i in range(rec["item0"], len(items))],
                           minlength=Cn)
        R = _mlp_split(ly, unit_live, ITEM_COST * n_it)
        rec["mrow0"], rec["mrow1"] = R[0], R[Cn]
        for c in range(Cn):
            ow = np.zeros(1, OWNER)[0]
            ow["mr0"], ow["mr1"], ow["orow"] = R[c], R[c + 1], -1
            rows = np.arange(c * blk, (c + 1) * blk)  # out_proj rows
            mrows = np.arange(R[c], R[c + 1])
            nr = len(mrows)
            blob = _Blob()
            bh = np.zeros(1, BHDR)[0]
            bh["ln_in"] = blob.add(ly.ln_in) if rec["has_gdn"] else -1
            bh["ln_post"] = blob.add(ly.ln_post) if rec["has_mlp"] else -1
            bh["mlp"] = -1
            mine = sorted((int(items[i]["slot"]), i) for i in range(rec["item0"], len(items))
                          if items[i]["cta"] == c)
            bh["n_items"] = len(mine)
            for q, (_, i) in enumerate(mine):
                pt = parts[i]
                bi = np.zeros(1, BITEM)[0]
                bi["item"], bi["n_eager"] = i, len(pt["chan"])
                bi["kh"], bi["slot"], bi["flags"] = items[i]["kh"], items[i]["slot"], items[i]["flags"]
                bc = np.zeros(len(pt["chan"]), BCHAN)
                for f in ("n", "slot", "conv_ch", "t01", "t23"):
                    bc[f] = pt["chan"][f]
                if len(winmap[c]) + len(bc) <= MAXWIN:  # windows kept in shared memory
                    bc["win"] = len(winmap[c]) + np.arange(len(bc))
                    winmap[c] += [(L, int(x)) for x in bc["conv_ch"]]
                    chans[i]["win"][:len(bc)] = bc["win"]  # (the item's first channels)
                else:
                    bc["win"] = 0xFFFFFFFF
                    if len(bc):
                        items[i]["flags"] |= IT_NONRES
                        bi["flags"] |= IT_NONRES
                bi["z"] = -1
                if pt["z"] is not None:
                    zs = pt["z"]
                    bi["z"] = blob.add(zs.indptr.astype(np.int32))
                    blob.add(_pack(zs.indices, zs.data))  # follows zptr (16-aligned)
                e_off = blob.add(np.concatenate(pt["ent"]) if pt["ent"] else np.zeros(0, np.uint32))
                bc["ent"] = e_off + 4 * np.concatenate([[0], np.cumsum([len(e) for e in pt["ent"]])[:-1]]).astype(np.int64) if len(bc) else 0
                bi["eager"] = blob.add(bc)
                pairs = np.zeros((2 * C.R, 2), np.int32)
                for r_, e_ in enumerate(pt["ba"]):
                    pairs[r_] = (blob.add(e_) if len(e_) else 0, len(e_))
                bi["rows"] = blob.add(pairs)
                bi["prm"] = blob.add(pt["prm"])
                bh["item"][q] = blob.add(np.array([bi], BITEM))
            if rec["has_mlp"]:
                sub = ly.down.rows_subset(mrows)
                keep = unit_live[sub.indices]
                rowid = np.repeat(np.arange(nr), sub.row_nnz())[keep]
                uidx, w = sub.indices[keep], sub.data[keep]
                need = np.unique(uidx)
                assert len(need) <= MAXUNITS, "too many MLP units for one CTA: use a larger cluster"
                loc = np.searchsorted(need, uidx)
                gi = _ranges(ly.gate.indptr[need], g_cnt[need])
                ui = _ranges(ly.up.indptr[need], u_cnt[need])
                g_off = blob.add(_pack(ly.gate.indices[gi], ly.gate.data[gi]))
                u_off = blob.add(_pack(ly.up.indices[ui], ly.up.data[ui]))
                un = np.zeros(len(need), BUNIT)
                un["g"] = g_off + 4 * (np.cumsum(g_cnt[need]) - g_cnt[need])
                un["u"] = u_off + 4 * (np.cumsum(u_cnt[need]) - u_cnt[need])
                un["ng"], un["nu"] = g_cnt[need], u_cnt[need]
                ptr = np.zeros(nr + 1, np.int64)
                np.cumsum(np.bincount(rowid, minlength=nr), out=ptr[1:])
                bm = np.zeros(1, BMLP)[0]
                bm["n_units"] = len(need)
                bm["r0"], bm["nr"] = R[c], nr
                bm["units"] = blob.add(un)
                bm["down_ptr"] = blob.add(ptr.astype(np.int32))
                bm["down_ent"] = blob.add(_pack(loc, w))
                bm["nlong"] = int((np.diff(ptr) > LONG).sum())  # rows the kernel sums by warps
                bh["mlp"] = blob.add(np.array([bm], BMLP))
                stats["unit_evals"] += len(need)
                stats["down_nnz"] += int(keep.sum())
            blobs.append(blob.done(bh))
            if rec["has_gdn"] and out_has[item_heads].any():
                sub = ly.out.rows_subset(rows)
                keep = item_heads[sub.indices // (C.R * C.VD)]
                rowid = np.repeat(np.arange(blk), sub.row_nnz())[keep]
                ptr = np.zeros(blk + 1, np.int64)
                np.cumsum(np.bincount(rowid, minlength=blk), out=ptr[1:])
                base = ent.add(_pack(sub.indices[keep], sub.data[keep]))
                ow["orow"] = i32.add((ptr + base).astype(np.int32))
                ow["nlong"] = int((np.diff(ptr) > LONG).sum())
                stats["out_nnz"] += int(keep.sum())
            owners.append(ow)
    # --- the head ----------------------------------------------------------------------------
    hd = chip.head
    V = hd.shape[0]
    col_cnt = np.bincount(hd.indices, minlength=C.H)
    dense = np.nonzero(col_cnt == V)[0] if V else np.zeros(0, np.int64)
    htab = np.zeros(4, np.float32)
    dense_ok = 0 < len(dense) <= MAXDENSE
    if dense_ok:
        isd = np.isin(hd.indices, dense)
        vals = np.unique(_f32(hd.data[isd]))
        dense_ok = len(vals) <= 4
    if not dense_ok:
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
    sp_rows, sp_cols, sp_bits = rows_of[sp], hd.indices[sp], hd.data[sp]
    sp_ptr = np.zeros(V + 1, np.int64)
    np.cumsum(np.bincount(sp_rows, minlength=V), out=sp_ptr[1:])
    sp_base = ent.add(_pack(sp_cols, sp_bits))
    # the columns with sparse entries, as a bitmask: a token whose normed residual is zero in all
    # of them adds only zeros there, and the kernel skips the rows' sparse entries
    hsp = np.zeros(C.H // 32, np.uint32)
    for c in np.unique(sp_cols):
        hsp[c >> 5] |= np.uint32(1) << np.uint32(c & 31)
    hsp_mask = i32.add(hsp.view(np.int32)) if len(sp_cols) else -1
    # the head rows: CTA rank c owns rows [V c / C, V (c + 1) / C) (entry C * HEADSLICES + c),
    # cut in HEADSLICES slices (entry c * HEADSLICES + k) for a launch with helper clusters: the
    # decoding cluster takes the first slices of its ranges, the helpers the others
    n_parts = Cn * HEADSLICES
    headcta = np.zeros(n_parts + Cn, HEADCTA)
    for c in range(n_parts):
        r0, r1 = V * c // n_parts, V * (c + 1) // n_parts
        headcta[c]["r0"], headcta[c]["r1"] = r0, r1
        headcta[c]["rowptr"] = i32.add((sp_ptr[r0:r1 + 1] + sp_base).astype(np.int32))
    for c in range(Cn):
        r0, r1 = V * c // Cn, V * (c + 1) // Cn
        e = headcta[n_parts + c]
        e["r0"], e["r1"] = r0, r1
        e["rowptr"] = i32.add((sp_ptr[r0:r1 + 1] + sp_base).astype(np.int32))
    final_norm = u16.add(chip.final_norm)
    for c in range(Cn):  # the head's blobs: the final norm
        blob = _Blob()
        bh = np.zeros(1, BHDR)[0]
        bh["ln_in"], bh["ln_post"], bh["mlp"] = blob.add(chip.final_norm), -1, -1
        blobs.append(blob.done(bh))
    widx = np.zeros((Cn, 2), np.int32)
    widx[:, 1] = [len(w) for w in winmap]
    widx[1:, 0] = np.cumsum(widx[:-1, 1])
    wmap = np.array([p for w in winmap for p in w], np.int32).reshape(-1, 2)
    bref = np.zeros(len(blobs), BLOBREF)
    bref["bytes"] = [len(b) for b in blobs]
    bref["off"] = np.concatenate([[0], np.cumsum(bref["bytes"])[:-1]])
    blob_bytes = np.frombuffer(b"".join(blobs), np.uint8)
    stats["blob_max"] = int(bref["bytes"].max())
    stats["blob_bytes"] = int(bref["bytes"].sum())
    assert ent.n < 1 << 31 and i32.n < 1 << 31 and u16.n < 1 << 31
    stats.update(head_dense=len(dense), head_sparse_nnz=int(sp.sum()), ent=ent.n)
    # --- the image ---------------------------------------------------------------------------
    secs = [layers, np.array(items, ITEM) if items else np.zeros(0, ITEM),
            np.concatenate(chans) if chans else np.zeros(0, CHAN), ent.array(),
            np.concatenate(units) if units else np.zeros(0, UNIT),
            np.array(owners, OWNER), i32.array(), u16.array(), headcta, hcodes, blob_bytes,
            bref, wmap, widx]
    hdr = np.zeros(1, HEADER)[0]
    hdr["magic"], hdr["version"] = MAGIC, VERSION
    hdr["n_layers"], hdr["cluster"], hdr["n_vocab"], hdr["hidden"] = chip.n_layers, Cn, V, C.H
    hdr["n_items"], hdr["n_dense"] = len(items), len(dense)
    hdr["n_embed_rows"], hdr["offset"], hdr["eps"] = chip.embed.shape[0], chip.offset, chip.eps
    hdr["final_norm"] = final_norm
    hdr["htab"] = htab
    hdr["dense_cols"][:len(dense)] = dense
    hdr["blob_max"] = stats["blob_max"]
    hdr["hsp_mask"] = hsp_mask
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
