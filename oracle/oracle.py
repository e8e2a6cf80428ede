"""TEST INFRASTRUCTURE ONLY: ctypes access to the CPU restatement in oracle.c.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg import this module, and
only as the checker; the product path (linuxformer_b200) never does.

    o = Oracle(chip)                       # a linuxformer_b200.chip.Chip
    preds, inputs, margins = o.decode(state, forced=[0], n=512)   # state updated in place
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"

P = ctypes.c_void_p
I64 = ctypes.c_int64


class _Csr(ctypes.Structure):
    _fields_ = [("rows", I64), ("cols", I64), ("indptr", P), ("indices", P), ("data", P)]


class _Layer(ctypes.Structure):
    _fields_ = [(n, _Csr) for n in ("qkv", "z", "b", "a", "out", "gate", "up", "down")] + \
        [(n, P) for n in ("conv", "A_log", "dt_bias", "gnorm", "ln_in", "ln_post")]


class _Chip(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("layers", P), ("embed", P), ("n_embed", I64),
                ("offset", ctypes.c_int), ("head", _Csr), ("final_norm", P),
                ("eps", ctypes.c_float)]


def build() -> Path:
    """Compile oracle.c into oracle/_build/liboracle.so (make, no reference sources)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        _lib.lxo_decode.restype = ctypes.c_int
        _lib.lxo_decode.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, P, P, P, P, P, P, P]
        for f in ("lxo_exp", "lxo_log1p", "lxo_silu", "lxo_sigmoid", "lxo_softplus"):
            getattr(_lib, f).restype = ctypes.c_float
            getattr(_lib, f).argtypes = [ctypes.c_float]
        _lib.lxo_ssq2560.restype = ctypes.c_float
        _lib.lxo_ssq2560.argtypes = [P]
        _lib.lxo_sumsq128.restype = ctypes.c_float
        _lib.lxo_sumsq128.argtypes = [P]
        assert _lib.lxo_n_counters() == len(Oracle.COUNTERS)
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return a.ctypes.data


class Oracle:
    def __init__(self, chip) -> None:
        self.chip = chip
        self._keep = []
        layers = (_Layer * chip.n_layers)()
        for i, L in enumerate(chip.layers):
            ly = layers[i]
            for name in ("qkv", "z", "b", "a", "out", "gate", "up", "down"):
                setattr(ly, name, self._csr(getattr(L, name)))
            for name in ("conv", "A_log", "dt_bias", "gnorm", "ln_in", "ln_post"):
                a = np.ascontiguousarray(getattr(L, name), np.uint16)
                self._keep.append(a)
                setattr(ly, name, _ptr(a))
        self._layers = layers
        emb = np.ascontiguousarray(chip.embed, np.uint16)
        fn = np.ascontiguousarray(chip.final_norm, np.uint16)
        self._keep += [emb, fn]
        self._chip = _Chip(n_layers=chip.n_layers, layers=ctypes.addressof(layers),
                           embed=_ptr(emb), n_embed=emb.shape[0], offset=chip.offset,
                           head=self._csr(chip.head), final_norm=_ptr(fn), eps=chip.eps)

    def _csr(self, m) -> _Csr:
        ip = np.ascontiguousarray(m.indptr, np.int64)
        ix = np.ascontiguousarray(m.indices, np.int32)
        da = np.ascontiguousarray(m.data, np.uint16)
        self._keep += [ip, ix, da]
        return _Csr(rows=m.shape[0], cols=m.shape[1], indptr=_ptr(ip), indices=_ptr(ix),
                    data=_ptr(da))

    COUNTERS = ("chans", "qkv_ent", "ba_ent", "z_ent", "rows", "out_ent", "gu_ent", "down_ent",
                "head_bytes", "vh_active", "vh_write", "vh_out", "gdn_write")

    def decode(self, state, forced, n: int, resid: bool = False, counts: bool = False,
               xin: bool = False, act: bool = False):
        """n steps of the model alone from `state` (a chip.State, updated in place). Returns
        (preds, inputs, margins[, resid][, counts][, xin]); counts: int64 [n, len(COUNTERS)];
        xin: each step's GDN input rows, float32 [n, n_layers, 2560]; act: per (step, layer,
        key head) bits: 1 query, 2 key, 4 decay, value heads with output << 8."""
        assert state.recurrent.dtype == np.float32 and state.conv.dtype == np.uint16
        assert state.recurrent.flags["C_CONTIGUOUS"] and state.conv.flags["C_CONTIGUOUS"]
        f = np.ascontiguousarray(forced, np.int32)
        preds = np.zeros(n, np.int32)
        inputs = np.zeros(n, np.int32)
        margins = np.zeros(n, np.float32)
        rs = np.zeros((n, 2560), np.float32) if resid else None
        cn = np.zeros((n, len(self.COUNTERS)), np.int64) if counts else None
        xi = np.zeros((n, self.chip.n_layers, 2560), np.float32) if xin else None
        ac = np.zeros((n, self.chip.n_layers, 16), np.int32) if act else None
        rc = lib().lxo_decode(ctypes.addressof(self._chip), _ptr(state.recurrent),
                              _ptr(state.conv), _ptr(f), len(f), n, _ptr(preds), _ptr(inputs),
                              _ptr(margins), _ptr(rs) if resid else None,
                              _ptr(cn) if counts else None, _ptr(xi) if xin else None,
                              _ptr(ac) if act else None)
        if rc:
            raise ValueError("oracle: token id out of the embedding's range")
        out = (preds, inputs, margins)
        if resid:
            out += (rs,)
        if counts:
            out += (cn,)
        if xin:
            out += (xi,)
        if act:
            out += (ac,)
        return out
