"""Benchmark: single-stream chip decode on B200 (config 2), one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl lxb|reference]

Workload: the 37-layer chip-shaped stack (497 live key heads, 36,716
SwiGLU units, 459,982 head rows, 5.5 MB of RAM/ROM in the GDN states), greedy decode of one
262,144-token chunk per GPU, as steps of --tokens tokens (one launch each, every launch
continuing its stream from the last prediction, as Linux.run_alone chains Mega.run launches).
Synthetic seeded weights (linuxformer_b200.chip.c2); rank r runs its own machine (state seed
1 + r): N GPUs decode N independent streams, no collective on the path (weak scaling).

value: tokens of all ranks / the slowest rank's device time of the K timed launches (CUDA
events on the launch stream; L2 flushed between launches). e2e: the same metric through the
host-buffer API (forced tokens copied in from pinned host memory, predictions copied back,
inside the timed region). roofline: the decode kernel's algorithmic bytes per token (counted
by the CPU restatement on a sample of the same stream) x tokens / kernel time, against the
measured HBM copy bandwidth. cpu_baseline: the CPU restatement (oracle/, all host threads) on
a bounded sample of the same stream, rank 0.
"""

from __future__ import annotations

import argparse
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

# The CPU baseline (the OpenMP restatement) runs on every host thread this process may use, also
# under torchrun, which sets OMP_NUM_THREADS=1 for its ranks (set before anything loads OpenMP).
HOST_THREADS = len(os.sched_getaffinity(0))
os.environ["OMP_NUM_THREADS"] = str(HOST_THREADS)

BASELINE_TOKS = 6017.4  # the reference's published megakernel figure: single stream, H100
FALLBACK_HBM = 6650.0


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


def traffic_per_token():
    """DRAM bytes per decoded token from the committed ncu summary, if there is one."""
    p = ROOT / "profiles" / "decode_c2_ncu.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("dram_bytes_per_token:"):
            return float(line.split(":")[1])
    return None


def cpu_sample(chip, state, n_tokens: int):
    """The oracle on the first n_tokens of the stream: (tok/s, preds, counts, threads)."""
    from oracle.oracle import Oracle

    o = Oracle(chip)
    st = state.copy()
    t0 = time.perf_counter()
    preds, _, _, counts = o.decode(st, [0], n_tokens, counts=True)
    dt = time.perf_counter() - t0
    return n_tokens / dt, preds, counts, HOST_THREADS


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=32768, help="tokens per step (one launch)")
    ap.add_argument("--cluster", type=int, default=16)
    ap.add_argument("--impl", default="lxb", choices=["lxb", "reference"])
    ap.add_argument("--cpu-tokens", type=int, default=400)
    ap.add_argument("--vocab", type=int, default=None, help="(tests) a smaller head")
    a = ap.parse_args()
    assert a.warmup >= 3 or a.impl == "reference", "at least 3 warm-up steps"

    import numpy as np

    from linuxformer_b200 import chip as C
    from linuxformer_b200.streams import job_rate, rank_env, slowest, stream_seed

    rank, world, local = rank_env()

    kw = {"vocab": a.vocab} if a.vocab else {}
    workload = (f"c2: 37-layer chip-shaped stack, greedy decode of {a.steps * a.tokens} tokens "
                f"per stream as {a.steps} launches of {a.tokens}, one stream per GPU")
    config = {"workload": workload, "tokens_per_step": a.tokens, "cluster": a.cluster,
              "streams_per_gpu": 1, "seed": 1, "l2": "flushed between timed launches"}

    if a.impl == "reference":
        # the reference's CPU path for this workload: the CPU restatement (the reference itself
        # is Python + fla/transformers and cannot run on the box), rank 0 only
        if rank != 0:
            return
        chip = C.c2(1, **kw)
        st = C.c2_state(chip, 1)
        from oracle.oracle import Oracle

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
        print(json.dumps({
            "impl": "reference", "metric": "chip decode tok/s (single stream per GPU)",
            "value": round(v, 2), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(1000 * dt / a.steps, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": dict(config, tokens_per_step=per),
            "cpu_baseline": {"value": round(v, 2), "unit": "tok/s", "cores": HOST_THREADS,
                             "kind": "port", "sample": f"{a.steps} x {per} tokens of the c2 stream"},
            "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}))
        return

    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=dev)
    from linuxformer_b200._lib import S_ERRORS
    from linuxformer_b200.runtime import Decoder

    chip = C.c2(1, **kw)
    st0 = C.c2_state(chip, stream_seed(1, rank))
    dec = Decoder(chip, cluster=a.cluster, device=dev)
    states = dec.states([st0])
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    T = a.tokens
    forced = torch.zeros((1, 1), dtype=torch.int32, device=dev)
    preds = torch.empty((1, T), dtype=torch.int32, device=dev)

    # parity spot check (rank 0): the first tokens of the stream against the CPU restatement
    cpu = None
    if rank == 0:
        cpu_v, cpu_preds, counts, cores = cpu_sample(chip, st0, a.cpu_tokens)
        chk = dec.states([st0])
        got, _ = dec.run(chk, [[0]], a.cpu_tokens)
        same = bool((got[0].cpu().numpy() == cpu_preds).all())
        del chk
        cpu = (cpu_v, counts, cores, same)

    # warm-up: W launches, the stream chained
    for w in range(a.warmup):
        dec.launch(states.ptrs, states.bitmaps, forced, T, preds, None, sync_bitmaps=(w == 0),
                   stream=stream, scratch=states.scratch)
        forced = preds[:, -1:].clone()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    times = []
    with Clocks(local) as clk:
        for k in range(a.steps):
            flush.fill_(k & 0xff)  # L2 flush (256 MB written), outside the events
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            dec.launch(states.ptrs, states.bitmaps, forced, T, preds, None, sync_bitmaps=False,
                       stream=stream, scratch=states.scratch)
            e1.record(stream)
            forced = preds[:, -1:].clone()
            e1.synchronize()
            times.append(e0.elapsed_time(e1) / 1000.0)
    torch.cuda.synchronize(dev)
    if dec.status().status & S_ERRORS:
        raise RuntimeError(f"device status {dec.status().status:#x}")
    tot = sum(times)
    # e2e: the host-buffer call (pinned H2D of the forced token, D2H of the predictions)
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
    e2e_tot = sum(e2e_t)
    tot, e2e_tot = slowest([tot, e2e_tot], dev)  # the slowest rank's times
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    value = job_rate(a.steps * T, world, tot)
    e2e_value = job_rate(e2e_steps * T, world, e2e_tot)
    peak, peak_kind = _peaks()
    cpu_v, counts, cores, same = cpu
    btok = bytes_per_token(counts)
    per_launch = tot / a.steps
    achieved = btok * T / per_launch / 1e9
    tr = traffic_per_token()
    line = {
        "metric": "chip decode tok/s (single stream per GPU)", "value": round(value, 1),
        "unit": "tok/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": round(1000 * tot / a.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": round(value / BASELINE_TOKS, 3), "dtype": "fp32",
        "data": "synthetic (seeded c2 generator)", "config": config,
        "e2e": {"value": round(e2e_value, 1), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * T},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": round(tr * T) if tr else None,
                     "note": f"peak of {peak_kind}; algorithmic {btok / 1e6:.2f} MB/token"},
        "cpu_baseline": {"value": round(cpu_v, 2), "unit": "tok/s", "cores": cores,
                         "kind": "port",
                         "sample": f"first {a.cpu_tokens} tokens of the rank-0 stream"},
        "clocks": clk.summary(), "gpu_launches": a.steps,
        "parity_sample": f"first {a.cpu_tokens} tokens {'identical' if same else 'DIFFER'} "
                         "to the CPU restatement",
        "activity_per_token": activity(counts),
        "us_per_token": round(1e6 * tot / (a.steps * T), 3),
    }
    print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
