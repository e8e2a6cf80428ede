"""Benchmark: the chip hot path on B200, one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lxb|reference]
                    [--mode all|decode|real|prefill|batched|text]

BASELINE.json's metric has three parts (single-stream decode, verify-prefill, batched decode); the
default line carries all three, the real circuit's decode and config 5's text decode:

- headline (``value``): single-stream chip decode (config 2): the 37-layer chip-shaped stack
  (497 live key heads, 36,716 SwiGLU units, 459,982 head rows, 5.5 MB of RAM/ROM in the GDN
  states), greedy decode in launches of --tokens tokens (a step), each launch continuing its
  stream from the last prediction (as Linux.run_alone chains Mega.run); K steps decode
  K x --tokens tokens of the stream (the reference's published figure runs 262,144 tokens a
  launch: 8 steps are one such chunk). Rank r decodes its own machine (state seed 1 + r): N
  GPUs decode N independent streams, no collective on the path (weak scaling).
- ``real``: the same measurement on the real compiled circuit (tests/golden/real_chip.npz, made by
  the reference's own compiler: the circuit behind the reference's published megakernel figure),
  decoding the model alone from GO on the fixture's machine (a RISC-V program over 4.5 MiB of
  seeded random RAM), --real-steps timed launches of --real-tokens after the warm-up launches
  (--steps of --tokens with --mode real); the whole stream is checked against the reference
  machine's own trace. The default line carries it at N = 1 (the headline covers the scaling
  runs); --mode real runs it on every rank.
- ``prefill``: verify-prefill tok/s (config 3): 1,048,576 token ids uniform over the config-1
  vocabulary (seed 2) through the config-1 stack as chunked prefill (lxb_prefill), chunks of
  65,536 (the headline) and of 8,192; a step is one pass over all of them, continuing the state.
  Also the first mismatch of the random trace, and a self-consistent trace (the decode's own
  greedy stream) that must verify with no mismatch. Every rank runs the whole config (replicas).
- ``batched``: batched tok/s (config 4): 64 machines on the config-1 stack (state seed 3 + i,
  start token 0), sharded 64 / N per GPU (strong scaling over the 64 streams); a step is one
  launch of all of the rank's streams for --batched-tokens tokens each (8 steps are config 4's
  32,768 tokens). Per-stream SHA-256 digests are gathered on the host after the timed region.
- ``text``: config 5's batch-1 decode (the Qwen3.5-4B-shaped model with zero-padded GDN layers,
  seeded random weights): a 4,096-token random-id prompt (seed 4), then a step is 512 greedy
  tokens from the state after the prompt (put back before every step, so every step decodes
  positions 4,096-4,607). Every rank runs the whole config (replicas).

Each part: ``value`` from CUDA events on the launch stream around the K timed steps (L2 flushed
between decode steps; the prefill's and the batched decode's working sets are larger than L2),
the slowest rank's time; ``e2e`` the same metric through the host-buffer API (inputs copied in
from pinned host memory, predictions copied back, inside the timed region); ``roofline`` for the
part's dominant kernel against the measured HBM copy bandwidth; ``cpu_baseline`` on the host
cores of rank 0: the CPU restatement (oracle/) for config 2, the reference's own stock forward
(transformers' torch GDN path through the HF decoder layers, oracle/stock.py) for configs 3
and 4, on bounded samples.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# The CPU baselines run on every host thread this process may use, also under torchrun, which
# sets OMP_NUM_THREADS=1 for its ranks (set before anything loads OpenMP).
HOST_THREADS = len(os.sched_getaffinity(0))
os.environ["OMP_NUM_THREADS"] = str(HOST_THREADS)

BASELINE_TOKS = 6017.4      # the reference's published megakernel figure: single stream, H100
BASELINE_PREFILL = 59236.0  # the reference's published lx.fast compiled verify-prefill, H100
FALLBACK_HBM = 6650.0
C3_TOKENS = 1 << 20
C4_STREAMS = 64
C5_PROMPT, C5_NEW = 4096, 512


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM, "fallback"


class Clocks:
    """nvidia-smi samples (every 200 ms) while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.p = gpu, [], None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.p = None
        return self

    def _read(self):
        for line in self.p.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()
            self.t.join(timeout=2)

    def summary(self):
        rows = [r for r in self.rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def bytes_per_token(counts) -> float:
    """Algorithmic bytes of one decode step from the oracle's counters (per token mean):
    4 B per weight entry used, 16 B per live conv window (read + write), 2 x 512 B per state row
    touched, the head's code/entry bytes, the 5,120-byte embedding row, a 4-byte prediction."""
    from oracle.oracle import Oracle

    k = {n: i for i, n in enumerate(Oracle.COUNTERS)}
    c = counts.mean(0)
    return float(16 * c[k["chans"]] + 4 * (c[k["qkv_ent"]] + c[k["ba_ent"]] + c[k["z_ent"]] +
                                          c[k["out_ent"]] + c[k["gu_ent"]] + c[k["down_ent"]]) +
                 1024 * c[k["rows"]] + c[k["head_bytes"]] + 5120 + 4)


def activity(counts) -> dict:
    from oracle.oracle import Oracle

    k = {n: i for i, n in enumerate(Oracle.COUNTERS)}
    c = counts.mean(0)
    return {"vh_active": round(float(c[k["vh_active"]]), 1),
            "vh_state_write": round(float(c[k["vh_write"]]), 2),
            "vh_output": round(float(c[k["vh_out"]]), 1),
            "gdn_writes": round(float(c[k["gdn_write"]]), 2)}


def profile_value(name: str, key: str):
    """A number recorded in a committed ncu summary (profiles/<name>), if there is one."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith(key + ":"):
            return float(line.split(":")[1])
    return None


def _event_time(fn, stream) -> float:
    import torch

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    fn()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / 1000.0


# --- config 2: single-stream decode (the headline) ---------------------------------------------
def decode_c2(a, rank, world, dev, kw):
    from linuxformer_b200 import chip as C
    from linuxformer_b200.streams import stream_seed

    chip = C.c2(1, **kw)
    st0 = C.c2_state(chip, stream_seed(1, rank))
    workload = (f"c2: 37-layer chip-shaped stack, greedy decode of {a.steps * a.tokens} tokens "
                f"per stream as {a.steps} launches of {a.tokens}, one stream per GPU")
    line = _decode_single(a, rank, world, dev, chip, st0, 0, None, "decode_c2_ncu.md")
    if line is None:
        return None
    line.update(metric="chip decode tok/s (single stream per GPU)",
                data="synthetic (seeded c2 generator)")
    line["config"] = dict({"workload": workload, "seed": 1}, **line["config"])
    return line


def decode_real(a, rank, world, dev):
    """The real compiled circuit (tests/golden/real_chip.npz: the reference's compiler, the
    merged model's circuit at hidden 2560) decoding the model alone from GO on the fixture's
    machine (a RISC-V program walking 4.5 MiB of seeded random RAM): the workload of the
    reference's published megakernel figure (the same circuit, its own kernel image booting).
    Every rank decodes its own copy of the machine (weak scaling); the stream is checked against
    the reference machine's own token trace."""
    from linuxformer_b200 import chip as C

    chip = C.real()
    st0 = C.real_state(chip)
    tr = chip.meta["fixture"]["trace"]
    line = _decode_single(a, rank, world, dev, chip, st0, int(tr[0]), tr, "decode_real_ncu.md")
    if line is None:
        return None
    line.update(metric="chip decode tok/s, real circuit (single stream per GPU)",
                data="the real circuit (reference compiler), seeded random RAM + program")
    line["config"] = dict({"workload": (
        f"real circuit: 37 compiled chip layers, 459,982-row head, greedy decode of "
        f"{a.steps * a.tokens} tokens per stream as {a.steps} launches of {a.tokens} after "
        f"{a.warmup} warm-up launches, from GO")}, **line["config"])
    return line


def _decode_single(a, rank, world, dev, chip, st0, first: int, trace, ncu_summary):
    """One machine per GPU decoding greedily in launches of a.tokens; the line's common keys."""
    import numpy as np
    import torch

    from linuxformer_b200._lib import S_ERRORS
    from linuxformer_b200.runtime import Decoder
    from linuxformer_b200.streams import job_rate, slowest
    from oracle.oracle import Oracle

    dec = Decoder(chip, cluster=a.cluster, device=dev)
    states = dec.states([st0])
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    T = a.tokens
    forced = torch.full((1, 1), first, dtype=torch.int32, device=dev)
    preds = torch.empty((1, T), dtype=torch.int32, device=dev)
    cpu = None
    if rank == 0:  # the CPU restatement on the stream's first tokens; the GPU must agree
        st = st0.copy()
        t0 = time.perf_counter()
        cpu_preds, _, _, counts = Oracle(chip).decode(st, [first], a.cpu_tokens, counts=True)
        cpu_v = a.cpu_tokens / (time.perf_counter() - t0)
        chk = dec.states([st0])
        got, _ = dec.run(chk, [[first]], a.cpu_tokens)
        same = bool((got[0].cpu().numpy() == cpu_preds).all())
        del chk
        cpu = (cpu_v, counts, same)
    stream_all = []  # the stream, launch by launch (checked against the trace, if there is one)
    for w in range(a.warmup):
        dec.launch(states.ptrs, states.bitmaps, forced, T, preds, None, sync_bitmaps=(w == 0),
                   stream=stream, scratch=states.scratch)
        forced = preds[:, -1:].clone()
        if trace is not None:
            stream_all.append(preds[0].clone())
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    times = []
    with Clocks(dev.index) as clk:
        for k in range(a.steps):
            flush.fill_(k & 0xff)  # L2 flush (256 MB written), outside the events
            times.append(_event_time(
                lambda: dec.launch(states.ptrs, states.bitmaps, forced, T, preds, None,
                                   sync_bitmaps=False, stream=stream, scratch=states.scratch),
                stream))
            forced = preds[:, -1:].clone()
            if trace is not None:
                stream_all.append(preds[0].clone())  # outside the events
    torch.cuda.synchronize(dev)
    if dec.status().status & S_ERRORS:
        raise RuntimeError(f"device status {dec.status().status:#x}")
    tot = sum(times)
    e2e_steps = max(2, a.steps // 4)
    last = int(forced[0, 0])
    e2e_t = []
    for k in range(e2e_steps):
        flush.fill_(k & 0xff)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        out = dec.run_host(states, np.array([[last]], np.int32), T, sync_bitmaps=False)
        e2e_t.append(time.perf_counter() - t0)
        last = int(out[0, -1])
        if trace is not None:
            stream_all.append(torch.from_numpy(np.asarray(out[0])))
    tot, e2e_tot = slowest([tot, sum(e2e_t)], dev)
    if rank != 0:
        return None
    trace_check = None
    if trace is not None:
        got = torch.cat([x.cpu() for x in stream_all]).numpy()
        n = min(len(got), len(trace) - 1)
        bad = np.nonzero(got[:n] != trace[1:n + 1])[0]
        trace_check = (f"first {n} tokens (warm-up, timed and e2e launches) "
                       + ("identical to the reference machine's trace" if len(bad) == 0 else
                          f"DIFFER from the reference machine's trace at token {bad[0] + 1}"))
    # outside the timed region: the per-section split of a profiled launch continuing the
    # stream, and the barrier floor (barriers per token x an empty cluster barrier's latency)
    prof = torch.zeros((1, a.cluster, len(dec.PROFILE)), dtype=torch.int64, device=dev)
    dec.set_profile(prof)
    n_prof = 4096
    pp = torch.empty((1, n_prof), dtype=torch.int32, device=dev)
    dec.launch(states.ptrs, states.bitmaps, forced, n_prof, pp, None, sync_bitmaps=False,
               stream=stream, scratch=states.scratch)
    torch.cuda.synchronize(dev)
    dec.set_profile(None)
    pr = prof[0].cpu().numpy().astype(np.float64).mean(0)  # the cluster's CTAs
    mhz = clk.summary().get("sm_mhz") or 1965.0
    split = {n: round(pr[k] / n_prof / mhz, 3) for k, n in enumerate(dec.PROFILE)
             if n not in dec.COUNTS}
    bar_tok = pr[dec.PROFILE.index("barriers")] / n_prof
    bar_ns = dec.barrier_cycles() / mhz * 1e3
    us_tok = 1e6 * tot / (a.steps * T)
    floor = {"barriers_per_token": round(bar_tok, 2), "empty_barrier_ns": round(bar_ns, 1),
             "floor_us_per_token": round(bar_tok * bar_ns / 1e3, 2),
             "floor_frac_of_step": round(bar_tok * bar_ns / 1e3 / us_tok, 4)}
    value = job_rate(a.steps * T, world, tot)
    e2e_value = job_rate(e2e_steps * T, world, e2e_tot)
    peak, peak_kind = _peaks()
    cpu_v, counts, same = cpu
    btok = bytes_per_token(counts)
    achieved = btok * T / (tot / a.steps) / 1e9
    tr = profile_value(ncu_summary, "dram_bytes_per_token") if ncu_summary else None
    line = {
        "metric": "", "value": round(value, 1),
        "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(1000 * tot / a.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / BASELINE_TOKS, 3), "dtype": "fp32",
        "data": "",
        "config": {"tokens_per_step": T, "cluster": a.cluster,
                   "streams_per_gpu": 1, "l2": "flushed between timed launches",
                   "staging": dec.staging()},
        "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * T},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": round(tr * T) if tr else None,
                     "note": f"peak of {peak_kind}; algorithmic {btok / 1e6:.2f} MB/token; "
                             "lxb_decode_kernel is the only kernel of a step"},
        "cpu_baseline": {"value": round(cpu_v, 2), "unit": "tok/s", "cores": HOST_THREADS,
                         "kind": "port",
                         "sample": f"first {a.cpu_tokens} tokens of the rank-0 stream"},
        "clocks": clk.summary(), "gpu_launches": a.steps,
        "parity_sample": f"first {a.cpu_tokens} tokens {'identical' if same else 'DIFFER'} "
                         "to the CPU restatement",
        "activity_per_token": activity(counts),
        "us_per_token": round(1e6 * tot / (a.steps * T), 3),
        "profile_us_per_token": split,
        "barrier_floor": floor,
    }
    if trace_check:
        line["trace_check"] = trace_check
    return line


# --- config 3: verify-prefill ---------------------------------------------------------------
# Algorithmic bytes of one launch of each prefill stage over a chunk of T tokens (per layer): what
# the stage must read and write once (feature-major bf16 activations; the weights, read once per
# launch, are a few hundred KB and left out).
def _prefill_stage_bytes(pf, T: int) -> dict:
    st = pf.stats
    H = 2560
    nl = pf.chip.n_layers
    units = st["units"] / nl                  # live MLP units per layer
    lvh = 8 * st["live_kh"] / nl              # live value heads per layer
    kh = st["live_kh"] / nl
    slots = st["live_rows"] / nl              # live query/key rows per layer
    return {
        "mlp": T * (2 * H + 2 * units),                          # the normed input, h out
        "recur": T * (lvh * (4 + 4 + 2 * 128) + kh * 8 + slots * 8),  # exp(g), beta, o out; masks
        "out": T * (2 * lvh * 128 + 4 * H),                      # on in; residual read + written
        "down": T * (2 * units + 4 * H),
        "gnorm": T * (lvh * (2 * 128 + 2 * 128) + 2 * H),       # o in, on out; the input norm
        "norm": T * 3 * 2 * H,                                   # residual twice, norm out
        "head": T * 2 * H,
    }


def prefill_c3(a, rank, world, dev):
    import numpy as np
    import torch

    from linuxformer_b200 import chip as C
    from linuxformer_b200.prefill import Prefill
    from linuxformer_b200.runtime import Decoder
    from linuxformer_b200.streams import job_rate, slowest
    from oracle.oracle import Oracle

    chip = C.c1(0)
    st0 = C.c1_state(chip, 0)
    pf = Prefill(chip, device=dev)

    def fresh():
        rec = torch.from_numpy(st0.recurrent.copy()).to(dev)
        conv = torch.from_numpy(st0.conv.view(np.int16).copy()).to(dev)
        ptrs = torch.tensor([[rec[L].data_ptr(), conv[L].data_ptr()]
                             for L in range(chip.n_layers)], dtype=torch.int64, device=dev)
        return rec, conv, ptrs

    ids_h = np.random.default_rng(2).integers(0, chip.n_vocab, C3_TOKENS).astype(np.int32)
    ids = torch.from_numpy(ids_h).to(dev)
    preds = torch.empty(C3_TOKENS, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = {}
    rec, conv, ptrs = fresh()
    fw = torch.empty(C3_TOKENS // 8192, dtype=torch.int32, device=dev)
    for chunk in (65536, 8192):
        sc = pf.scratch(chunk)
        n_ch = C3_TOKENS // chunk

        def one_pass():
            for k in range(n_ch):
                pf.launch(ptrs, ids[k * chunk:(k + 1) * chunk], preds[k * chunk:(k + 1) * chunk],
                          fw[k:k + 1], scratch=sc)

        for _ in range(max(1, a.warmup)):
            one_pass()
        torch.cuda.synchronize(dev)
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        steps = max(1, min(a.steps, a.prefill_steps))
        tot = sum(_event_time(one_pass, stream) for _ in range(steps))
        out[chunk] = (steps, tot)
    # the first mismatch of the random trace (the last pass, from the state it found)
    f = fw.cpu().numpy()[:C3_TOKENS // 8192]
    first = -1
    pr = preds.cpu().numpy()
    for k in range(C3_TOKENS // 8192):
        if f[k] >= 0:
            first = k * 8192 + int(f[k])
            break
        b = (k + 1) * 8192
        if b < C3_TOKENS and pr[b - 1] != ids_h[b]:
            first = b - 1
            break
    # e2e through the host-buffer call (token ids in, predictions out, per chunk of 65,536)
    e2e_steps = 1
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        pf.run_host(ptrs, ids_h, 65536)
    e2e_tot = time.perf_counter() - t0
    # the stage split of one pass (per-stage CUDA events; not the timed passes)
    sc = pf.scratch(65536)
    pf.set_timing(True)
    for k in range(C3_TOKENS // 65536):
        pf.launch(ptrs, ids[k * 65536:(k + 1) * 65536], preds[k * 65536:(k + 1) * 65536],
                  fw[k:k + 1], scratch=sc)
    split = pf.timing()
    pf.set_timing(False)
    (s64, t64), (s8, t8) = out[65536], out[8192]
    t64, t8, e2e_tot = slowest([t64, t8, e2e_tot], dev)
    if rank != 0:
        return None
    # parity: the first 2,048 ids from the seeded state against the CPU restatement, and a
    # self-consistent trace (the decode's own greedy stream) that verifies with no mismatch
    n_par = 2048
    _, _, ptrs2 = fresh()
    got, _ = pf.run(ptrs2, ids_h[:n_par])
    want, _, _ = Oracle(chip).decode(st0.copy(), ids_h[:n_par], n_par)
    same = bool((got.cpu().numpy() == want).all())
    dec = Decoder(chip, cluster=16, device=dev)
    ds = dec.states([st0])
    dp, dinp = dec.run(ds, [[0]], 4096)
    _, _, ptrs3 = fresh()
    tp, tfirst = pf.run(ptrs3, dinp[0].cpu().numpy(), chunk=1024)
    trace_ok = tfirst == -1 and bool((tp.cpu().numpy() == dp[0].cpu().numpy()).all())
    draft = self_draft_c1(chip, st0, pf, dev)
    # the CPU baseline: the reference's stock chunked forward on the first ids
    from oracle.stock import StockCPU

    sc_cpu = StockCPU(chip)
    cache = sc_cpu.cache(st0)
    n_cpu = a.cpu_prefill_tokens
    t0 = time.perf_counter()
    sc_cpu.prefill(cache, ids_h[:n_cpu])
    cpu_v = n_cpu / (time.perf_counter() - t0)
    value = job_rate(s64 * C3_TOKENS, world, t64)
    peak, peak_kind = _peaks()
    dom = max((k for k in split if k != "scan"), key=lambda k: split[k][0])
    sb = _prefill_stage_bytes(pf, 65536)
    dom_ms = split[dom][0] / split[dom][1]  # per launch (one layer of one chunk)
    launches_per_pass = sum(v[1] for v in split.values())
    achieved = sb.get(dom, 0.0) / (dom_ms / 1e3) / 1e9
    return {
        "metric": "verify-prefill tok/s (config 3, chunks of 65,536)",
        "value": round(value, 1), "unit": "tok/s", "steps": s64,
        "ms_per_step": round(1000 * t64 / s64, 3),
        "vs_reference_published": round(value / BASELINE_PREFILL, 2),
        "chunk_8192": {"value": round(job_rate(s8 * C3_TOKENS, world, t8), 1), "unit": "tok/s",
                       "steps": s8},
        "config": {"workload": "c3: config-1 stack, 1,048,576 ids uniform over 4,096 (seed 2), "
                               "as chunked prefill, each rank all of it (replicas)",
                   "l2": "working set larger than L2 (activations of a 65,536-token chunk)"},
        "scaling": "weak",
        "first_mismatch": first,
        "self_consistent_trace": ("4,096-token greedy trace: no mismatch, predictions identical "
                                  "to the decode") if trace_ok else "FAILED",
        "parity_sample": f"first {n_par} positions {'identical' if same else 'DIFFER'} to the "
                         "CPU restatement (forced per-token decode)",
        "e2e": {"value": round(job_rate(e2e_steps * C3_TOKENS, world, e2e_tot), 1),
                "unit": "tok/s", "h2d_bytes_per_step": 4 * C3_TOKENS,
                "d2h_bytes_per_step": 4 * C3_TOKENS},
        "stages_ms_per_pass": {k: round(v[0], 3) for k, v in split.items()},
        "roofline": {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": (profile_value("prefill_c3_ncu.md",
                                               "mlp_tile_traffic_per_launch_65536")
                                 if dom == "mlp" else None),
                     "note": f"peak of {peak_kind}; the dominant stage by CUDA events; "
                             "algorithmic bytes: its inputs and outputs once per token"},
        "cpu_baseline": {"value": round(cpu_v, 2), "unit": "tok/s", "cores": HOST_THREADS,
                         "kind": "reference",
                         "sample": f"the reference's stock chunked forward (HF decoder layers, "
                                   f"transformers torch GDN) on the first {n_cpu} ids"},
        "gpu_launches": int(launches_per_pass * s64),
        "self_draft": draft,
    }


def self_draft_c1(chip, st0, pf, dev, n: int = 8192, D: int = 255) -> dict:
    """Self-drafting verify (linuxformer_b200.draft) on config 1's greedy stream from token 0:
    wall time of the whole host-driven loop (each round: draft on the host, one prefill call,
    a device copy of the state, and a rollback when a draft token was wrong; bursts of the decode
    kernel where nothing is drafted), against the decode kernel's single-stream rate on the same
    stream; both streams compared token for token."""
    import numpy as np
    import torch

    from linuxformer_b200.draft import SelfDraft
    from linuxformer_b200.runtime import Decoder

    def fresh():
        rec = torch.from_numpy(st0.recurrent.copy()).to(dev)
        conv = torch.from_numpy(st0.conv.view(np.int16).copy()).to(dev)
        ptrs = torch.tensor([[rec[L].data_ptr(), conv[L].data_ptr()]
                             for L in range(chip.n_layers)], dtype=torch.int64, device=dev)
        return rec, conv, ptrs

    sd = SelfDraft(pf, draft=D, decoder=Decoder(chip, cluster=16, device=dev))
    rec, conv, ptrs = fresh()
    sd.run(ptrs, [rec, conv], 0, 512)  # warm-up
    rec, conv, ptrs = fresh()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    got, stats = sd.run(ptrs, [rec, conv], 0, n)
    torch.cuda.synchronize(dev)
    t_sd = time.perf_counter() - t0
    dec = Decoder(chip, cluster=16, device=dev)
    ds = dec.states([st0])
    dec.run(ds, [[0]], 64)
    ds = dec.states([st0])
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    want, _ = dec.run(ds, [[0]], n)
    torch.cuda.synchronize(dev)
    t_dec = time.perf_counter() - t0
    return {"metric": "self-drafting greedy decode tok/s (config 1, one stream)",
            "value": round(n / t_sd, 1), "unit": "tok/s", "tokens": n, "draft": D,
            "plain_decode": round(n / t_dec, 1), "speedup": round(t_dec / t_sd, 2),
            "identical_to_decode": bool((got == want[0].cpu().numpy()).all()), **stats,
            "timing": "wall clock of the host-driven loop (per-round host sync), both sides"}


# --- config 4: batched independent machines -----------------------------------------------
_STOCK = {}


def stock_c1():
    """The reference's stock forward of the config-1 stack on the CPU (built once)."""
    from linuxformer_b200 import chip as C
    from oracle.stock import StockCPU

    if "c1" not in _STOCK:
        _STOCK["c1"] = StockCPU(C.c1(0))
    return _STOCK["c1"]


def batched_c4(a, rank, world, dev):
    import numpy as np
    import torch

    from linuxformer_b200 import chip as C
    from linuxformer_b200._lib import S_ERRORS
    from linuxformer_b200.runtime import Decoder
    from linuxformer_b200.streams import gather_digests, job_rate, shard, slowest
    from oracle.oracle import Oracle

    chip = C.c1(0)
    mine = shard(C4_STREAMS, rank, world)
    S, T = len(mine), a.batched_tokens
    dec = Decoder(chip, cluster=a.cluster, device=dev)
    states = dec.states([C.c1_state(chip, 3 + i) for i in mine])
    stream = torch.cuda.current_stream(dev)
    forced = torch.zeros((S, 1), dtype=torch.int32, device=dev)
    preds = torch.empty((S, T), dtype=torch.int32, device=dev)
    for w in range(a.warmup):
        dec.launch(states.ptrs, states.bitmaps, forced, T, preds, None, sync_bitmaps=(w == 0),
                   stream=stream, scratch=states.scratch)
        forced = preds[:, -1:].clone()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    steps = max(1, min(a.steps, 8))
    hs = {i: hashlib.sha256() for i in mine}
    times = []
    with Clocks(dev.index) as clk:
        for _ in range(steps):
            times.append(_event_time(
                lambda: dec.launch(states.ptrs, states.bitmaps, forced, T, preds, None,
                                   sync_bitmaps=False, stream=stream, scratch=states.scratch),
                stream))
            forced = preds[:, -1:].clone()
            got = preds.cpu().numpy()  # after the step's events: outside the timed region
            for k, i in enumerate(mine):
                hs[i].update(got[k].tobytes())
    if dec.status().status & S_ERRORS:
        raise RuntimeError(f"device status {dec.status().status:#x}")
    tot = sum(times)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    dec.run_host(states, forced.cpu().numpy(), T, sync_bitmaps=False)
    e2e_tot = time.perf_counter() - t0
    digests = gather_digests({i: h.hexdigest() for i, h in hs.items()})
    tot, e2e_tot = slowest([tot, e2e_tot], dev)
    if rank != 0:
        return None
    # parity: two streams' first 64 tokens from their seeded states against the CPU restatement
    chk = dec.states([C.c1_state(chip, 3), C.c1_state(chip, 3 + C4_STREAMS - 1)])
    got, _ = dec.run(chk, [[0], [0]], 64)
    o = Oracle(chip)
    same = all(bool((got[k].cpu().numpy() == o.decode(C.c1_state(chip, sd), [0], 64)[0]).all())
               for k, sd in ((0, 3), (1, 3 + C4_STREAMS - 1)))
    # algorithmic bytes per token once the seeded states have decayed (oracle counters)
    _, _, _, counts = o.decode(C.c1_state(chip, 3), [0], 600, counts=True)
    btok = bytes_per_token(counts[400:])
    # the CPU baseline: the reference's stock decode, streams one after another
    sc_cpu = stock_c1()
    n_cpu, s_cpu = a.cpu_batched_tokens, 2
    t0 = time.perf_counter()
    for i in range(s_cpu):
        sc_cpu.decode(sc_cpu.cache(C.c1_state(chip, 3 + i)), 0, n_cpu)
    cpu_v = s_cpu * n_cpu / (time.perf_counter() - t0)
    value = job_rate(S * steps * T, world, tot)
    per_gpu = value / world
    peak, peak_kind = _peaks()
    achieved = btok * per_gpu / 1e9
    combined = hashlib.sha256("".join(digests[i] for i in range(C4_STREAMS)).encode()).hexdigest()
    return {
        "metric": "batched tok/s (config 4: 64 streams on the config-1 stack)",
        "value": round(value, 1), "unit": "tok/s", "steps": steps,
        "ms_per_step": round(1000 * tot / steps, 3),
        "config": {"workload": f"c4: 64 machines (state seeds 3..66, start token 0) on the "
                               f"config-1 stack, {C4_STREAMS // world} per GPU, {steps} launches "
                               f"of {T} tokens each (config 4 is 8 x 4,096 = 32,768)",
                   "cluster": a.cluster, "streams_per_gpu": S,
                   "co_resident_clusters": dec.max_clusters,
                   "l2": "working set larger than L2 (64 streams' states, 2.1 GB)"},
        "scaling": "strong",
        "streams_digest": combined,
        "distinct_streams": len(set(digests.values())),
        "parity_sample": f"streams 0 and 63, first 64 tokens "
                         f"{'identical' if same else 'DIFFER'} to the CPU restatement",
        "e2e": {"value": round(job_rate(S * T, world, e2e_tot), 1), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * S, "d2h_bytes_per_step": 4 * S * T},
        "roofline": {"bound": "hbm", "kernel": "lxb_decode_kernel",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None,
                     "note": f"peak of {peak_kind}; algorithmic {btok / 1e6:.3f} MB/token once "
                             "the seeded states have decayed (tokens 400-600 of a stream)"},
        "cpu_baseline": {"value": round(cpu_v, 2), "unit": "tok/s", "cores": HOST_THREADS,
                         "kind": "reference",
                         "sample": f"the reference's stock decode (HF decoder layers, "
                                   f"transformers torch GDN), {s_cpu} streams x {n_cpu} tokens "
                                   "one after another"},
        "clocks": clk.summary(), "gpu_launches": steps,
    }


# --- config 5: the text path's batch-1 decode -------------------------------------------------
def text_bytes_per_token(dec, pos: int) -> float:
    """Algorithmic bytes of one config-5 decode step at position pos: every non-padding weight
    once (the packed tables, the head, the norms), the embedding row, the attention layers' key and
    value rows up to pos plus the new ones, the GDN states' live rows (read and write) and the
    conv windows of the live channels (read and write), a 4-byte prediction."""
    from linuxformer_b200 import text as T

    w = sum(v.numel() * v.element_size() for d in dec.t["layers"] for k, v in d.items()
            if hasattr(v, "numel"))
    w += dec.t["head"].numel() * 2 + dec.t["norm"].numel() * 2
    kv = dec.n_att * T.NKV * (pos + 1) * T.HD * 2 * 2
    gdn = dec.n_gdn * (T.QNV * T.QKD * T.VD * 4 * 2 + (2 * T.QNK * T.QKD + T.QNV * T.QVD) * 8 * 2)
    return float(w + kv + gdn + T.H * 2 + 4)


def text_c5(a, rank, world, dev):
    import numpy as np
    import torch

    from linuxformer_b200 import text as T
    from linuxformer_b200.streams import job_rate, slowest
    from oracle.text_stock import cpu_copy, steps as stock_steps

    model = T.random_model(seed=4, device=str(dev))
    dec = T.TextDecoder(model, max_pos=C5_PROMPT + C5_NEW)
    ids_h = np.random.default_rng(4).integers(0, T.VOCAB, C5_PROMPT).astype(np.int32)
    ids = torch.from_numpy(ids_h).to(dev)
    pp = torch.empty(C5_PROMPT, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    dec.launch(ids, C5_PROMPT, pp)
    torch.cuda.synchronize(dev)
    prompt_s = time.perf_counter() - t0
    snap = (dec.conv.clone(), dec.rec.clone(), dec.kc[:, :, :C5_PROMPT].clone(),
            dec.vc[:, :, :C5_PROMPT].clone())
    first = pp[-1:].clone()
    out = torch.empty(C5_NEW, dtype=torch.int32, device=dev)

    def restore():
        dec.conv.copy_(snap[0])
        dec.rec.copy_(snap[1])
        dec.kc[:, :, :C5_PROMPT].copy_(snap[2])
        dec.vc[:, :, :C5_PROMPT].copy_(snap[3])
        dec.pos = C5_PROMPT

    stream = torch.cuda.current_stream(dev)
    for _ in range(a.warmup):
        restore()
        dec.launch(first, C5_NEW, out)
    ref = out.clone()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    steps = max(1, min(a.steps, a.text_steps))
    times, same = [], True
    with Clocks(dev.index) as clk:
        for _ in range(steps):
            restore()  # outside the timed region
            times.append(_event_time(lambda: dec.launch(first, C5_NEW, out), stream))
            same &= bool(torch.equal(out, ref))
    if dec.status():
        raise RuntimeError(f"device status {dec.status():#x}")
    tot = sum(times)
    # e2e: the first token from pinned host memory, the predictions back into it
    h_in = torch.tensor([int(first)], dtype=torch.int32).pin_memory()
    h_out = torch.empty(C5_NEW, dtype=torch.int32).pin_memory()
    restore()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    dec.launch(h_in.to(dev, non_blocking=True), C5_NEW, out)
    h_out.copy_(out, non_blocking=True)
    torch.cuda.synchronize(dev)
    e2e_tot = time.perf_counter() - t0
    tot, e2e_tot = slowest([tot, e2e_tot], dev)
    if rank != 0:
        return None
    # parity: 16 decode steps after the prompt against the stock forward (prompt as one chunk,
    # then the same inputs token by token), teacher-forced with this stream
    n_chk = 16
    restore()
    hid = torch.empty(n_chk, len(dec.t["layers"]) + 1, T.H, dtype=torch.float32, device=dev)
    chk = torch.empty(n_chk, dtype=torch.int32, device=dev)
    dec.launch(first, n_chk, chk, hid)
    from transformers import DynamicCache

    cache = DynamicCache(config=model.config)
    with torch.no_grad():
        model.model(input_ids=ids.long()[None], past_key_values=cache, use_cache=True)
    inp = torch.cat([first, chk[:-1]]).long()
    hs, lg = stock_steps(model, inp, cache)
    top = lg.max(1)
    gap = float((top.values - lg.gather(1, chk.long()[:, None])[:, 0]).max())
    agree = float((top.indices.int() == chk).float().mean())
    dh = float((hid[:, -1] - hs).abs().max())
    # the CPU baseline: the reference's text path (the stock forward) on the host cores
    cpu = cpu_copy(model)
    del model
    torch.cuda.empty_cache()
    from oracle.text_stock import zero_cache

    cc = zero_cache(cpu)
    stock_steps(cpu, ids_h[:8], cc, logits=False)  # a short prompt, then timed decode steps
    n_cpu = max(2, a.cpu_text_tokens)
    t0 = time.perf_counter()
    stock_steps(cpu, ids_h[8:8 + n_cpu], cc)
    cpu_v = n_cpu / (time.perf_counter() - t0)
    del cpu
    value = job_rate(steps * C5_NEW, world, tot)
    per_gpu = value / world
    peak, peak_kind = _peaks()
    btok = text_bytes_per_token(dec, C5_PROMPT + C5_NEW // 2)
    achieved = btok * per_gpu / 1e9
    return {
        "metric": "text decode tok/s (config 5: batch 1 after a 4,096-token prompt)",
        "value": round(value, 1), "unit": "tok/s", "steps": steps, "dtype": "bf16",
        "data": "synthetic (seeded random-init weights, torch Philox on the device; seeded "
                "random prompt ids)",
        "ms_per_step": round(1000 * tot / steps, 3),
        "config": {"workload": f"c5: Qwen3.5-4B-shaped random-init model (32 layers, GDN padded "
                               f"to 128 value heads x 256 key dims, vocab {T.VOCAB}), "
                               f"{C5_PROMPT}-token prompt (seed 4), {steps} steps of {C5_NEW} "
                               "greedy tokens from the post-prompt state",
                   "prompt_s": round(prompt_s, 2), "grid": dec.grid,
                   "l2": "working set larger than L2 (8.4 GB of weights per token)"},
        "scaling": "weak", "steps_identical": same,
        "parity_sample": {"steps": n_chk, "argmax_agree": round(agree, 3),
                          "max_logit_gap": round(gap, 4), "max_hidden_diff": round(dh, 4),
                          "tolerance": {"logit_gap": 0.25, "hidden": 0.5},
                          "against": "the stock HF forward on the GPU, prompt as one chunk, "
                                     "then token by token"},
        "e2e": {"value": round(job_rate(C5_NEW, world, e2e_tot), 1), "unit": "tok/s",
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4 * C5_NEW},
        "roofline": {"bound": "hbm", "kernel": "lxb_text_kernel", "achieved": round(achieved, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None,
                     "note": f"peak of {peak_kind}; algorithmic {btok / 1e9:.3f} GB/token "
                             "(non-padding weights, attention cache at the mean position, GDN "
                             "live state rows and windows)"},
        "cpu_baseline": {"value": round(cpu_v, 3), "unit": "tok/s", "cores": HOST_THREADS,
                         "kind": "reference",
                         "sample": f"the reference's text path (stock HF forward, transformers "
                                   f"torch GDN) on the host: {n_cpu} decode steps after an "
                                   "8-token prompt"},
        "clocks": clk.summary(), "gpu_launches": steps,
    }


def reference_arm(a, rank, world, kw):
    """The reference's CPU path on the host cores (rank 0; the other ranks exit): config 2 by the
    CPU restatement (the reference's own stock model of config 2 is 16 GB of dense bf16 layers),
    configs 3 and 4 by the reference's stock forward (oracle/stock.py)."""
    if rank != 0:
        return
    import numpy as np

    from linuxformer_b200 import chip as C
    from oracle.oracle import Oracle

    chip = C.c2(1, **kw)
    st = C.c2_state(chip, 1)
    o = Oracle(chip)
    per = max(8, a.cpu_tokens // 4)
    tok, last = 0, 0
    for _ in range(a.warmup):
        p, _, _ = o.decode(st, [last], per)
        last = int(p[-1])
    t0 = time.perf_counter()
    for _ in range(a.steps):
        p, _, _ = o.decode(st, [last], per)
        last = int(p[-1])
        tok += per
    dt = time.perf_counter() - t0
    v = tok / dt
    line = {
        "impl": "reference", "metric": "chip decode tok/s (single stream per GPU)",
        "value": round(v, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(1000 * dt / a.steps, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic",
        "config": {"workload": f"c2 decode, {a.steps} samples of {per} tokens of the stream",
                   "tokens_per_step": per},
        "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": HOST_THREADS,
                         "kind": "port", "sample": f"{a.steps} x {per} tokens of the c2 stream"},
        "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}
    if a.mode in ("all", "prefill", "batched"):
        c1 = C.c1(0)
        sc = stock_c1()
        if a.mode in ("all", "prefill"):
            ids = np.random.default_rng(2).integers(0, c1.n_vocab, a.cpu_prefill_tokens)
            t0 = time.perf_counter()
            sc.prefill(sc.cache(C.c1_state(c1, 0)), ids)
            pv = len(ids) / (time.perf_counter() - t0)
            line["prefill"] = {"metric": "verify-prefill tok/s (config 3)", "value": round(pv, 2),
                               "unit": "tok/s", "kind": "reference", "cores": HOST_THREADS,
                               "sample": f"one chunk of the first {len(ids)} config-3 ids"}
        if a.mode in ("all", "batched"):
            n = a.cpu_batched_tokens
            t0 = time.perf_counter()
            for i in range(2):
                sc.decode(sc.cache(C.c1_state(c1, 3 + i)), 0, n)
            bv = 2 * n / (time.perf_counter() - t0)
            line["batched"] = {"metric": "batched tok/s (config 4)", "value": round(bv, 2),
                               "unit": "tok/s", "kind": "reference", "cores": HOST_THREADS,
                               "sample": f"2 streams x {n} tokens, one after another"}
    if a.mode in ("all", "text"):
        line["text"] = reference_text(a)
    print(json.dumps(line))


def reference_text(a):
    """Config 5 by the reference's text path (the stock HF forward) on the host cores: the seeded
    random-init model (made on the GPU when there is one, then copied to the host), an 8-token
    prompt, then --steps decode steps timed."""
    import numpy as np
    import torch

    from linuxformer_b200 import text as T
    from oracle.text_stock import cpu_copy, steps as stock_steps, zero_cache

    gpu = torch.cuda.is_available()
    model = T.random_model(seed=4, device="cuda" if gpu else "cpu")
    cpu = cpu_copy(model) if gpu else model
    del model
    ids = np.random.default_rng(4).integers(0, T.VOCAB, 8 + max(1, a.steps)).astype(np.int64)
    cache = zero_cache(cpu)
    stock_steps(cpu, ids[:8], cache, logits=False)
    t0 = time.perf_counter()
    stock_steps(cpu, ids[8:], cache)
    v = (len(ids) - 8) / (time.perf_counter() - t0)
    return {"metric": "text decode tok/s (config 5)", "value": round(v, 3), "unit": "tok/s",
            "kind": "reference", "cores": HOST_THREADS,
            "sample": f"{len(ids) - 8} decode steps after an 8-token prompt (the stock HF "
                      "forward, transformers torch GDN)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=32768, help="decode tokens per step (launch)")
    ap.add_argument("--cluster", type=int, default=16)
    ap.add_argument("--impl", default="lxb", choices=["lxb", "reference"])
    ap.add_argument("--mode", default="all",
                    choices=["all", "decode", "real", "prefill", "batched", "text"])
    ap.add_argument("--cpu-tokens", type=int, default=400)
    ap.add_argument("--cpu-prefill-tokens", type=int, default=1024)
    ap.add_argument("--prefill-steps", type=int, default=4)
    ap.add_argument("--batched-tokens", type=int, default=4096)
    ap.add_argument("--cpu-batched-tokens", type=int, default=16)
    ap.add_argument("--text-steps", type=int, default=4)
    ap.add_argument("--real-steps", type=int, default=4, help="timed launches, real circuit")
    ap.add_argument("--real-tokens", type=int, default=8192,
                    help="tokens per launch of the real circuit's part in the default line")
    ap.add_argument("--cpu-text-tokens", type=int, default=4)
    ap.add_argument("--vocab", type=int, default=None, help="(tests) a smaller c2 head")
    a = ap.parse_args()
    assert a.warmup >= 3 or a.impl == "reference", "at least 3 warm-up steps"
    from linuxformer_b200.streams import rank_env

    rank, world, local = rank_env()
    kw = {"vocab": a.vocab} if a.vocab else {}
    if a.impl == "reference":
        return reference_arm(a, rank, world, kw)

    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    line = None
    if a.mode in ("all", "decode"):
        line = decode_c2(a, rank, world, dev, kw)
    parts = {}
    # (the default line carries the real circuit's part on one GPU; with --mode real, on every N)
    if a.mode == "real" or (a.mode == "all" and world == 1):
        import copy

        ar = copy.copy(a)
        if a.mode == "all":
            ar.steps, ar.tokens = a.real_steps, a.real_tokens
        parts["real"] = decode_real(ar, rank, world, dev)
    if a.mode in ("all", "prefill"):
        parts["prefill"] = prefill_c3(a, rank, world, dev)
    if a.mode in ("all", "batched"):
        parts["batched"] = batched_c4(a, rank, world, dev)
    if a.mode in ("all", "text"):
        parts["text"] = text_c5(a, rank, world, dev)
    if rank == 0:
        if line is None:  # a single part as the line itself
            (name, part), = parts.items()
            line = dict({"dtype": "fp32", "data": "synthetic (seeded c1 generator)"}, **part)
            line.update(n_gpus=world, warmup=a.warmup, higher_is_better=True, vs_baseline=None)
        else:
            line.update(parts)
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
