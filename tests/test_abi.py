"""The C ABI library (CPU-side checks: no kernel runs here)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from linuxformer_b200 import chip as C
from linuxformer_b200 import tables
from linuxformer_b200._lib import lib

ROOT = Path(__file__).resolve().parents[1]


def test_exports_every_declared_symbol():
    decl = set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(lxb_\w+)\s*\(", (ROOT / "include" / "lxb.h").read_text(),
                          re.M))
    assert decl, "no declarations found"
    L = lib()
    for name in decl:
        assert hasattr(L, name), name
    assert L.lxb_abi_version() == 1


@pytest.fixture(scope="module")
def image(c1_chip):
    img, _ = tables.build_image(c1_chip, 16)
    return img


def _create(img, cluster=16):
    a = np.frombuffer(bytes(img), np.uint8)
    p = ctypes.c_void_p()
    rc = lib().lxb_plan_create(a.ctypes.data, len(a), cluster, ctypes.byref(p))
    if rc == 0:
        lib().lxb_plan_destroy(p)
    return rc


def test_valid_image_passes_validation(image):
    rc = _create(image)
    assert rc != -2, "a valid image was rejected"  # here (no GPU) the CUDA call then fails


def test_corrupt_images_are_rejected(image):
    hdr = np.frombuffer(image[:tables.HEADER.itemsize], tables.HEADER)[0]
    bad = []
    b = bytearray(image); b[0] ^= 1; bad.append(b)                       # magic
    b = bytearray(image); b[8:12] = np.int32(1000).tobytes(); bad.append(b)  # n_layers
    # an entry column out of range
    ent_off = int(hdr["sec"][3][0])
    b = bytearray(image); b[ent_off:ent_off + 4] = np.uint32(0xffff).tobytes(); bad.append(b)
    # a channel's conv index out of range
    ch_off = int(hdr["sec"][2][0])
    b = bytearray(image); b[ch_off + 8:ch_off + 12] = np.uint32(1 << 20).tobytes(); bad.append(b)
    # a truncated image
    bad.append(bytearray(image[:len(image) // 2]))
    # an owner's MLP row range not 8-aligned; a layer's MLP rows not the owners' ranges
    ow_off = int(hdr["sec"][tables.SEC.index("owners")][0])
    mr1 = np.frombuffer(image[ow_off + 4:ow_off + 8], np.int32)[0]
    b = bytearray(image); b[ow_off + 4:ow_off + 8] = np.int32(mr1 + 1).tobytes(); bad.append(b)
    ly_off = int(hdr["sec"][tables.SEC.index("layers")][0])
    f = tables.LAYER.fields["mrow1"][1]
    v = np.frombuffer(image[ly_off + f:ly_off + f + 4], np.int32)[0]
    b = bytearray(image); b[ly_off + f:ly_off + f + 4] = np.int32(v + 8).tobytes(); bad.append(b)
    # the channel table naming another resident window than the blob (first item's first channel)
    it_off = int(hdr["sec"][tables.SEC.index("items")][0])
    it0 = np.frombuffer(image[it_off:it_off + tables.ITEM.itemsize], tables.ITEM)[0]
    assert it0["n_eager"] > 0 and not (it0["flags"] & tables.IT_NONRES)
    ch0 = int(it0["ch0"])
    w = ch_off + ch0 * tables.CHAN.itemsize + tables.CHAN.fields["win"][1]
    win = np.frombuffer(image[w:w + 4], np.uint32)[0]
    b = bytearray(image); b[w:w + 4] = np.uint32(win ^ 1).tobytes(); bad.append(b)
    for k, img in enumerate(bad):
        assert _create(img) == -2, k
    assert _create(image, cluster=8) == -2  # built for 16


def test_invalid_arguments():
    L = lib()
    p = ctypes.c_void_p()
    assert L.lxb_plan_create(None, 0, 16, ctypes.byref(p)) == -1
    assert L.lxb_decode(None, None, None, 0, None, None, 1, None, 1, 1, None, None, None) == -1
    assert L.lxb_error_string(-2) == b"malformed plan image"
