"""The device-side runtime: a chip's plan on the GPU, machine states in device memory, and the
decode launch through the C ABI.

    dec = Decoder(chip, cluster=16)               # tables built and uploaded once
    st = dec.states([state0, state1])             # device copies of chip.State (HF cache layout)
    preds, inputs = dec.run(st, forced=[[0], [7]], n=4096)   # [streams, n] int32, on the device

PyTorch is used for device memory and streams only; all compute is in liblxb.so.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import chip as C
from . import tables
from ._lib import S_ERRORS, Caps, Err, LxbError, Typing, check, lib


def _u16(t: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(t).view(np.int16)).to(dev)


@dataclass
class DeviceStates:
    """n_streams machines: recurrent [S, L, 128, 256, 128] fp32, conv [S, L, 24576, 4] bf16 bits
    (int16 storage), the per-(stream, layer) pointer table and the nonzero-row bitmaps."""
    recurrent: torch.Tensor
    conv: torch.Tensor
    ptrs: torch.Tensor      # int64 [S, L, 2]
    bitmaps: torch.Tensor   # int32 [S, L, 128, 8]
    scratch: torch.Tensor   # uint8, lxb_scratch_bytes(plan, S)

    @property
    def n_streams(self) -> int:
        return self.recurrent.shape[0]

    def host(self, s: int) -> C.State:
        return C.State(self.recurrent[s].cpu().numpy().copy(),
                       self.conv[s].cpu().numpy().view(np.uint16).copy())


def state_pointers(rec_list, conv_list, dev) -> torch.Tensor:
    """[S][L][2] device pointers from per-(stream, layer) tensors (lists of lists)."""
    rows = [[(r.data_ptr(), c.data_ptr()) for r, c in zip(rs, cs)]
            for rs, cs in zip(rec_list, conv_list)]
    return torch.tensor(rows, dtype=torch.int64, device=dev)


class Decoder:
    def __init__(self, chip: C.Chip, cluster: int = 16, device=None, embed=None) -> None:
        self.dev = torch.device(device or "cuda")
        if self.dev.type != "cuda":
            raise LxbError("the chip decode runs on a CUDA device only")
        if self.dev.index is None:
            self.dev = torch.device("cuda", torch.cuda.current_device())
        torch.cuda.set_device(self.dev)
        self.chip, self.cluster = chip, cluster
        self.image, self.stats = tables.build_image(chip, cluster)
        self._img = np.frombuffer(self.image, np.uint8)
        p = ctypes.c_void_p()
        check(lib().lxb_plan_create(self._img.ctypes.data, len(self.image), cluster,
                                    ctypes.byref(p)), "lxb_plan_create")
        self.plan = p
        self.max_clusters = lib().lxb_plan_max_clusters(p)
        self.embed = embed if embed is not None else _u16(chip.embed, self.dev)
        assert self.embed.is_contiguous() and self.embed.shape[1] == C.H

    def __del__(self):
        p = getattr(self, "plan", None)
        if p is not None and p.value:
            try:
                lib().lxb_plan_destroy(p)
            except TypeError:  # interpreter shutdown: the module's globals are gone already
                pass
            self.plan = None

    def caps(self) -> Caps:
        c = Caps()
        check(lib().lxb_query(self.dev.index or 0, ctypes.byref(c)), "lxb_query")
        c.max_clusters = self.max_clusters
        return c

    def states(self, init) -> DeviceStates:
        """Device copies of chip.State objects (or an int: that many zero states)."""
        nl = self.chip.n_layers
        if isinstance(init, int):
            S = init
            rec = torch.zeros((S, nl, C.NV, C.KD, C.VD), dtype=torch.float32, device=self.dev)
            conv = torch.zeros((S, nl, C.CONV, C.TAPS), dtype=torch.int16, device=self.dev)
        else:
            S = len(init)
            rec = torch.empty((S, nl, C.NV, C.KD, C.VD), dtype=torch.float32, device=self.dev)
            conv = torch.empty((S, nl, C.CONV, C.TAPS), dtype=torch.int16, device=self.dev)
            for s, st in enumerate(init):
                rec[s].copy_(torch.from_numpy(st.recurrent))
                conv[s].copy_(torch.from_numpy(st.conv.view(np.int16)))
        ptrs = state_pointers([[rec[s, L] for L in range(nl)] for s in range(S)],
                              [[conv[s, L] for L in range(nl)] for s in range(S)], self.dev)
        bm = torch.zeros((S, nl, C.NV, 8), dtype=torch.int32, device=self.dev)
        return DeviceStates(rec, conv, ptrs, bm, self.scratch(S))

    def scratch(self, n_streams: int) -> torch.Tensor:
        """The device scratch one launch of n_streams streams needs."""
        nb = lib().lxb_scratch_bytes(self.plan, n_streams)
        return torch.empty(nb, dtype=torch.uint8, device=self.dev)

    def launch(self, ptrs: torch.Tensor, bitmaps: torch.Tensor, forced: torch.Tensor, n: int,
               preds: torch.Tensor, inputs: torch.Tensor | None, sync_bitmaps: bool = True,
               stream=None, scratch: torch.Tensor | None = None) -> None:
        """Raw launch on device tensors (no host sync): forced int32 [S, nf], preds [S, n]."""
        S = forced.shape[0]
        assert forced.dtype == torch.int32 and forced.is_contiguous() and forced.dim() == 2
        assert preds.dtype == torch.int32 and preds.shape == (S, n) and preds.is_contiguous()
        assert ptrs.shape == (S, self.chip.n_layers, 2) and bitmaps.shape[0] == S
        if scratch is None:
            scratch = self.scratch(S)
        assert scratch.numel() >= lib().lxb_scratch_bytes(self.plan, S)
        st = (stream or torch.cuda.current_stream(self.dev)).cuda_stream
        check(lib().lxb_decode(self.plan, ptrs.data_ptr(), bitmaps.data_ptr(), int(sync_bitmaps),
                               scratch.data_ptr(), self.embed.data_ptr(), S, forced.data_ptr(),
                               forced.shape[1], n,
                               preds.data_ptr(),
                               inputs.data_ptr() if inputs is not None else None, st),
              "lxb_decode")

    T_FINAL, T_TYPED, T_RX = 1, 2, 4  # lxb_typing token classes

    def set_typing(self, keys, key0_base: int, key_base: int, rx_slots: int,
                   tclass: np.ndarray | None) -> None:
        """The device typing queue (lxb_plan_set_typing): keys, one byte sequence per stream;
        tclass, T_* bits per token id (record boundary, typed key, RX read); None turns it off.
        The queue state starts cleared; ``typing_state()`` reads it back and ``next_inputs()``
        is the forced first input of each stream's next launch."""
        if tclass is None:
            check(lib().lxb_plan_set_typing(self.plan, None), "lxb_plan_set_typing")
            self._typing = None
            return
        S = len(keys)
        mk = max(1, max(len(k) for k in keys))
        kt = torch.zeros((S, mk), dtype=torch.int32, device=self.dev)
        for i, k in enumerate(keys):
            if len(k):
                kt[i, :len(k)] = torch.as_tensor(np.asarray(list(k), np.int32), device=self.dev)
        nk = torch.tensor([len(k) for k in keys], dtype=torch.int32, device=self.dev)
        tc = torch.as_tensor(np.asarray(tclass, np.uint8), device=self.dev)
        ts = torch.zeros((S, 4), dtype=torch.int32, device=self.dev)
        ty = Typing(kt.data_ptr(), nk.data_ptr(), mk, key0_base, key_base, rx_slots,
                    tc.data_ptr(), tc.numel(), ts.data_ptr())
        check(lib().lxb_plan_set_typing(self.plan, ctypes.byref(ty)), "lxb_plan_set_typing")
        self._typing = (kt, nk, tc, ts)

    def typing_state(self) -> np.ndarray:
        """Per stream: bytes typed, the RX FIFO count, bytes left in the batch, next input."""
        return self._typing[3].cpu().numpy()

    def next_inputs(self) -> torch.Tensor:
        """The first input of each stream's next launch (int32 [S, 1] on the device)."""
        return self._typing[3][:, 3:4].contiguous()

    PROFILE = ("norm", "items", "mlp", "sync", "pull", "fixup", "head", "embed", "fixups",
               "tokens", "wait", "polls", "takesync", "barriers", "group_items", "group_sync",
               "group_fixup", "fixup_mlp", "fixup_out")
    COUNTS = ("fixups", "tokens", "polls", "barriers")  # counts; the others are clock cycles

    def barrier_cycles(self, iters: int = 10000) -> float:
        """An empty cluster barrier's latency (SM clock cycles) at this plan's cluster size."""
        v = ctypes.c_double()
        check(lib().lxb_cluster_sync_cycles(self.cluster, iters, ctypes.byref(v)),
              "lxb_cluster_sync_cycles")
        return v.value

    def set_profile(self, buf: torch.Tensor | None) -> None:
        """Accumulate per-section cycle counters into buf (int64 [S, cluster, 13]) on every
        later launch; None stops it."""
        if buf is not None:
            assert buf.dtype == torch.int64 and buf.is_contiguous()
            assert buf.shape[-1] == lib().lxb_profile_sections() == len(self.PROFILE)
        check(lib().lxb_plan_set_profile(self.plan, buf.data_ptr() if buf is not None else None),
              "lxb_plan_set_profile")
        self._prof = buf

    def staging(self) -> dict:
        """The plan's staging: buffers, bytes per buffer, shared memory per CTA."""
        v = [ctypes.c_int() for _ in range(3)]
        check(lib().lxb_plan_staging(self.plan, *(ctypes.byref(x) for x in v)), "lxb_plan_staging")
        return {"buffers": v[0].value, "stage_bytes": v[1].value, "smem_bytes": v[2].value}

    def status(self) -> Err:
        e = Err()
        check(lib().lxb_status(self.plan, ctypes.byref(e)), "lxb_status")
        return e

    def _pinned(self, key, shape) -> torch.Tensor:
        buf = getattr(self, "_pin", {})
        self._pin = buf
        t = buf.get(key)
        if t is None or t.numel() < int(np.prod(shape)):
            t = torch.empty(int(np.prod(shape)), dtype=torch.int32).pin_memory()
            buf[key] = t
        return t[:int(np.prod(shape))].view(shape)

    def run_host(self, states: DeviceStates, forced: np.ndarray, n: int,
                 sync_bitmaps: bool = True) -> np.ndarray:
        """The host-buffer call: forced tokens from host memory in, predictions [S, n] back in
        host memory (copies through pinned buffers on the current stream)."""
        forced = np.ascontiguousarray(forced, np.int32).reshape(states.n_streams, -1)
        S = states.n_streams
        fh = self._pinned("f", forced.shape)
        fh.numpy()[...] = forced
        fd = fh.to(self.dev, non_blocking=True)
        preds = torch.empty((S, n), dtype=torch.int32, device=self.dev)
        self.launch(states.ptrs, states.bitmaps, fd, n, preds, None, sync_bitmaps,
                    scratch=states.scratch)
        ph = self._pinned("p", (S, n))
        ph.copy_(preds, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        e = self.status()
        if e.status & S_ERRORS:
            check(lib().lxb_status_clear(self.plan), "lxb_status_clear")
            raise LxbError(f"device status {e.status:#x} (stream {e.first_stream}, "
                           f"step {e.first_step})")
        return ph.numpy().copy()

    def run(self, states: DeviceStates, forced, n: int):
        """n steps of every stream; forced: one list of ints per stream (equal lengths >= 1).
        Returns (preds, inputs) as int32 device tensors [S, n]; raises on a device error."""
        f = torch.as_tensor(np.asarray(forced, np.int32).reshape(states.n_streams, -1),
                            device=self.dev)
        preds = torch.empty((states.n_streams, n), dtype=torch.int32, device=self.dev)
        inputs = torch.empty_like(preds)
        self.launch(states.ptrs, states.bitmaps, f, n, preds, inputs, scratch=states.scratch)
        torch.cuda.synchronize(self.dev)
        e = self.status()
        if e.status & S_ERRORS:
            check(lib().lxb_status_clear(self.plan), "lxb_status_clear")
            raise LxbError(f"device status {e.status:#x} (stream {e.first_stream}, "
                           f"step {e.first_step})")
        return preds, inputs
