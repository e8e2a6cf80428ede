"""The table builder's layouts (CPU): the MLP row ranges of the owners, the staged blobs' MLP
parts, and the channel table's resident windows that the quiet pass reads. lxb_plan_create
checks the same invariants (tests/test_abi.py feeds it images that break them)."""

import numpy as np
import pytest

from linuxformer_b200 import chip as C
from linuxformer_b200 import tables


class Image:
    def __init__(self, img: bytes):
        self.b = img
        self.h = np.frombuffer(img[:tables.HEADER.itemsize], tables.HEADER)[0]

    def sec(self, name, dt):
        k = tables.SEC.index(name)
        off, cnt = int(self.h["sec"][k][0]), int(self.h["sec"][k][1])
        return np.frombuffer(self.b[off:off + cnt * dt.itemsize], dt)

    def blob(self, L, c, cluster):
        ref = self.sec("blobidx", tables.BLOBREF)[L * cluster + c]
        k = tables.SEC.index("blobs")
        off = int(self.h["sec"][k][0]) + int(ref["off"])
        return self.b[off:off + int(ref["bytes"])]


@pytest.fixture(scope="module", params=["c1", "c2"])
def built(request, c1_chip):
    """Config 1 (two dense-ish layers) and config 2 (the bench's 37 layers, GDN-only runs)."""
    chip = c1_chip if request.param == "c1" else C.c2(1)
    img, _ = tables.build_image(chip, 16)
    return chip, 16, Image(img)


def test_mlp_row_ranges_tile_the_changing_rows(built):
    chip, Cn, im = built
    layers = im.sec("layers", tables.LAYER)
    owners = im.sec("owners", tables.OWNER).reshape(chip.n_layers, Cn)
    for L, ly in enumerate(chip.layers):
        rec, ow = layers[L], owners[L]
        if not rec["has_mlp"]:
            assert rec["mrow0"] == rec["mrow1"] == 0 and (ow["mr0"] == ow["mr1"]).all()
            continue
        bounds = np.concatenate([ow["mr0"], ow["mr1"][-1:]])
        assert bounds[0] == rec["mrow0"] and bounds[-1] == rec["mrow1"]
        assert (ow["mr0"][1:] == ow["mr1"][:-1]).all() and (np.diff(bounds) >= 0).all()
        assert (bounds % 8 == 0).all() and (np.diff(bounds) <= C.H // tables.MINC).all()
        # every row a live unit writes is inside the changing range
        g, u = ly.gate.row_nnz(), ly.up.row_nnz()
        live = (g > 0) & (u > 0) & (ly.down.transpose().row_nnz() > 0)
        rows = np.repeat(np.arange(C.H), ly.down.row_nnz())[live[ly.down.indices]]
        assert rows.min() >= rec["mrow0"] and rows.max() < rec["mrow1"]


def test_blob_mlp_parts_match_their_owner(built):
    chip, Cn, im = built
    layers = im.sec("layers", tables.LAYER)
    owners = im.sec("owners", tables.OWNER).reshape(chip.n_layers, Cn)
    for L in range(chip.n_layers):
        if not layers[L]["has_mlp"]:
            continue
        for c in range(Cn):
            B = im.blob(L, c, Cn)
            bh = np.frombuffer(B[:tables.BHDR.itemsize], tables.BHDR)[0]
            m = np.frombuffer(B[bh["mlp"]:bh["mlp"] + tables.BMLP.itemsize], tables.BMLP)[0]
            assert m["r0"] == owners[L, c]["mr0"] and m["nr"] == owners[L, c]["mr1"] - m["r0"]
            ptr = np.frombuffer(B[m["down_ptr"]:m["down_ptr"] + 4 * (m["nr"] + 1)], np.int32)
            assert ptr[0] == 0 and (np.diff(ptr) >= 0).all()


def test_quiet_pass_windows_match_the_blobs(built):
    """The quiet pass reads a channel's resident window slot from the global channel table; the
    staged path reads it from the blob. Both must name the same slot."""
    chip, Cn, im = built
    items = im.sec("items", tables.ITEM)
    chans = im.sec("chans", tables.CHAN)
    seen = 0
    for L in range(chip.n_layers):
        for c in range(Cn):
            B = im.blob(L, c, Cn)
            bh = np.frombuffer(B[:tables.BHDR.itemsize], tables.BHDR)[0]
            for k in range(bh["n_items"]):
                o = int(bh["item"][k])
                bi = np.frombuffer(B[o:o + tables.BITEM.itemsize], tables.BITEM)[0]
                it = items[bi["item"]]
                bc = np.frombuffer(B[bi["eager"]:bi["eager"] + bi["n_eager"] * tables.BCHAN.itemsize],
                                   tables.BCHAN)
                gc = chans[it["ch0"]:it["ch0"] + bi["n_eager"]]
                assert (gc["win"] == bc["win"]).all() and (gc["n"] == bc["n"]).all()
                assert (gc["t01"] == bc["t01"]).all() and (gc["t23"] == bc["t23"]).all()
                seen += len(bc)
    assert seen > 0
    # every other channel keeps no resident window
    rest = np.ones(len(chans), bool)
    for it in items:
        rest[it["ch0"]:it["ch0"] + it["n_eager"]] = False
    assert (chans["win"][rest] == 0xFFFFFFFF).all()


def test_mlp_split_balances_the_work():
    """_mlp_split on config 1's first layer with random item base costs: the largest owner cost
    is within one 8-row chunk of the lower bound no contiguous split can beat."""
    rng = np.random.default_rng(5)
    chip = C.c1(0)
    ly = chip.layers[0]
    g, u = ly.gate.row_nnz(), ly.up.row_nnz()
    live = (g > 0) & (u > 0) & (ly.down.transpose().row_nnz() > 0)
    for Cn in (16, 8):  # (the per-owner row cap, H / MINC rows, does not bind here)
        base = tables.ITEM_COST * rng.integers(0, 2, Cn)
        R = tables._mlp_split(ly, live, base)
        assert R[0] % 8 == 0 and R[-1] % 8 == 0 and (np.diff(R) >= 0).all()
        rowid = np.repeat(np.arange(C.H), ly.down.row_nnz())
        keep = live[ly.down.indices]
        rc = np.bincount(rowid[keep], weights=(g + u)[ly.down.indices[keep]].astype(float),
                         minlength=C.H) + tables.ROW_COST
        cost = np.array([base[c] + rc[R[c]:R[c + 1]].sum() for c in range(Cn)])
        chunk = rc[R[0]:R[-1]].reshape(-1, 8).sum(1).max()
        # no contiguous split beats (total + bases) / Cn; a greedy one is within a chunk of it
        lower = max((rc[R[0]:R[-1]].sum() + base.sum()) / Cn, base.max())
        assert cost.max() <= lower + chunk + 1e-6, (Cn, cost.max(), lower, chunk)


def test_real_circuit_head_mask_and_long_rows(real_chip):
    """The real circuit's plan: the head's sparse-column mask holds exactly the 191 columns with
    sparse entries (the kernel skips the rows' sparse entries when the normed residual is zero in
    all of them), and every owner's and MLP blob's long-row count is the number of its rows with
    more than LONG entries (the rows the kernel sums by warps)."""
    Cn = 16
    img, st = tables.build_image(real_chip, Cn)
    im = Image(img)
    i32 = im.sec("i32", np.dtype("<i4"))
    mask = i32[int(im.h["hsp_mask"]):int(im.h["hsp_mask"]) + C.H // 32].view(np.uint32)
    cols = np.nonzero((mask[np.arange(C.H) >> 5] >> (np.arange(C.H) & 31)) & 1)[0]
    dense = set(int(c) for c in im.h["dense_cols"][:int(im.h["n_dense"])])
    hd = real_chip.head
    want = sorted(set(np.unique(hd.indices).tolist()) - dense)
    assert cols.tolist() == want and len(want) == 191
    owners = im.sec("owners", tables.OWNER).reshape(real_chip.n_layers, Cn)
    layers = im.sec("layers", tables.LAYER)
    n_long = 0
    for L in range(real_chip.n_layers):
        for c in range(Cn):
            ow = owners[L, c]
            if ow["orow"] >= 0:
                ptr = i32[int(ow["orow"]):int(ow["orow"]) + C.H // Cn + 1]
                assert ow["nlong"] == int((np.diff(ptr) > tables.LONG).sum())
                n_long += int(ow["nlong"])
            else:
                assert ow["nlong"] == 0
            if layers[L]["has_mlp"]:
                b = im.blob(L, c, Cn)
                bh = np.frombuffer(b[:tables.BHDR.itemsize], tables.BHDR)[0]
                if bh["mlp"] >= 0:
                    m = np.frombuffer(b[bh["mlp"]:bh["mlp"] + tables.BMLP.itemsize], tables.BMLP)[0]
                    dp = np.frombuffer(b[m["down_ptr"]:m["down_ptr"] + 4 * (m["nr"] + 1)], "<i4")
                    assert m["nlong"] == int((np.diff(dp) > tables.LONG).sum())
    assert n_long > 0  # layer 2's memory-read rows (1,024 entries) among them
