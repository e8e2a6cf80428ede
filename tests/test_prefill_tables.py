"""The prefill plan image (linuxformer_b200.prefill_tables, csrc/lxb_prefill.h): what it keeps, and
that lxb_prefill_check_image (the validation lxb_prefill_plan_create runs before any upload)
accepts it and rejects corrupt ones. CPU only: no kernel runs here."""

import numpy as np
import pytest

from linuxformer_b200 import chip as C
from linuxformer_b200 import prefill_tables as PT
from linuxformer_b200._lib import lib


@pytest.fixture(scope="module")
def built(c1_chip):
    return PT.build_image(c1_chip)


def _check(img) -> int:
    a = np.frombuffer(bytes(img), np.uint8).copy()
    return lib().lxb_prefill_check_image(a.ctypes.data, len(a))


def _sections(img):
    hdr = np.frombuffer(img[:PT.HEADER.itemsize], PT.HEADER)[0]
    return hdr, {name: (int(hdr["sec"][k][0]), int(hdr["sec"][k][1]))
                 for k, name in enumerate(PT.SEC)}


def _layers(img, hdr, secs):
    off, n = secs["layers"]
    return np.frombuffer(img, PT.LAYER, count=n, offset=off)


def _i32(img, secs):
    off, n = secs["i32"]
    return np.frombuffer(img, np.int32, count=n, offset=off)


def test_valid_images_pass(built):
    assert _check(built[0]) == 0
    img, _ = PT.build_image(C.c2(1, vocab=20000))
    assert _check(img) == 0


def test_live_rows_are_the_tapped_query_and_key_rows(c1_chip, built):
    img, _ = built
    hdr, secs = _sections(img)
    i32 = _i32(img, secs)
    for L, ly in enumerate(_layers(img, hdr, secs)):
        layer = c1_chip.layers[L]
        tapped = ((layer.conv & 0x7FFF) != 0).any(1)
        khs = i32[ly["khs"]:ly["khs"] + 3 * ly["n_kh"]].reshape(-1, 3)
        slots = i32[ly["slots"]:ly["slots"] + 3 * ly["n_slot"]].reshape(-1, 3)
        want = {}
        for kh in range(C.NK):
            rows = np.nonzero(tapped[kh * C.KD:(kh + 1) * C.KD] |
                              tapped[C.NK * C.KD + kh * C.KD:C.NK * C.KD + (kh + 1) * C.KD])[0]
            if len(rows):
                want[kh] = rows.tolist()
        assert [int(k) for k in khs[:, 0]] == sorted(want)
        for kh, s0, nl in khs:
            assert slots[s0:s0 + nl, 0].tolist() == want[kh]  # ascending rows
        assert ly["nl"] == max(len(v) for v in want.values())


def test_out_proj_keeps_exactly_the_live_heads_entries(c1_chip, built):
    img, _ = built
    hdr, secs = _sections(img)
    i32 = _i32(img, secs)
    for L, ly in enumerate(_layers(img, hdr, secs)):
        khs = i32[ly["khs"]:ly["khs"] + 3 * ly["n_kh"]].reshape(-1, 3)[:, 0]
        live_vh = (khs[:, None] * C.R + np.arange(C.R)).reshape(-1)
        o = c1_chip.layers[L].out
        want = int(np.isin(o.indices // C.VD, live_vh).sum())
        ptr = i32[ly["out_ptr"]:ly["out_ptr"] + C.H + 1]
        assert int(ptr[-1] - ptr[0]) == want


def test_corrupt_images_are_rejected(built):
    img, _ = built
    hdr, secs = _sections(img)
    lay_off = secs["layers"][0]
    bad = []
    b = bytearray(img); b[0] ^= 1; bad.append(b)                                   # magic
    bad.append(bytearray(img[:len(img) - 64]))                                      # truncated
    b = bytearray(img)                                                               # n_tap
    f = np.frombuffer(b, PT.LAYER, count=1, offset=lay_off).copy()
    f["n_tap"] = hdr["max_tap"] + 1
    b[lay_off:lay_off + PT.LAYER.itemsize] = f.tobytes(); bad.append(b)
    b = bytearray(img)                                                               # nl > 31
    f = np.frombuffer(b, PT.LAYER, count=1, offset=lay_off).copy()
    f["nl"] = PT.MAXLIVE + 1
    b[lay_off:lay_off + PT.LAYER.itemsize] = f.tobytes(); bad.append(b)
    # an out_proj entry whose index is past the live dims
    ly = _layers(img, hdr, secs)[0]
    i32 = _i32(img, secs)
    e0 = int(i32[ly["out_ptr"]])
    ent_off = secs["ent"][0] + 4 * e0
    b = bytearray(img)
    v = np.frombuffer(b, np.uint32, count=1, offset=ent_off).copy()
    v[0] = (v[0] & 0xFFFF0000) | 0xFFFF
    b[ent_off:ent_off + 4] = v.tobytes(); bad.append(b)
    # a slot's key tap past the layer's taps
    so = secs["i32"][0] + 4 * (int(ly["slots"]) + 2)
    b = bytearray(img)
    b[so:so + 4] = np.array([ly["n_tap"]], np.int32).tobytes(); bad.append(b)
    for k, b in enumerate(bad):
        assert _check(b) == -2, k


def test_too_many_live_rows_is_reported():
    chip = C.c1(0)
    ly = chip.layers[0]
    ly.conv = ly.conv.copy()
    ly.conv[:40, 3] = C.bf16_bits(np.float32(0.5))  # 40 tapped query rows in key head 0
    with pytest.raises(PT.PrefillUnsupported, match="live rows"):
        PT.build_image(chip)
