"""Benchmark of the decoder's per-step attention (32 layers of self-attention with cache append + cross-attention,
plus the slot-table bookkeeping of the step) on B200, in the reference's headline metric.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config3] [--impl ours|reference]
    (N > 1: torchrun --nproc-per-node N bench.py --gpus N ..., one process per GPU)

A step = one replay of a CUDA graph holding, for each of the 32 layers, ``self_attn_step_triton(write_cache=True)``
and ``cross_attn_triton`` of ``whisper_trt_b200.attn_plugin`` (the reference plugin's call surface, through the C
ABI), then the bookkeeping of the step (windows replaced by fresh ones, ``slot_reset``; the new beams' slot tables
from random parent permutations, ``beam_reorder``, which also advances the windows' positions). Inputs are seeded
synthetic tensors of whisper-large-v3's shapes (20 heads x 64, 1500 frames) resident in HBM; every step reads
several GB, far more than the 126 MB L2, so no flush is needed between steps.

value = algorithmic HBM bytes per step (see ``step_bytes``) x steps / time, summed over all GPUs (GB/s, whole job);
ms_per_step = the max over ranks of the device time per step. Prints one JSON line on rank 0, with: ``e2e`` (the
same step through the public API with its inputs copied in from pinned host memory and its result -- the last
layer's outputs -- copied out, and the copy rate each rank gets); ``roofline`` (the dominant kernel's achieved bandwidth); ``also`` (configs 2, 4 and
5 at the same N); at N = 1 ``vs_reference_gpu`` (the reference's own Triton kernels timed beside these on the same
inputs) and ``cpu_baseline``.

``--impl reference``: the reference's CPU implementation of the path on the host cores -- its own PyTorch ops,
imported unmodified from ``baseline/_ref`` (their numpy restatement in ``oracle/`` when it is not staged) -- a
bounded sample per step (one layer of a block of windows), same metric and config.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "whisper-trt_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "decode-step attention µs/step (32 layers) & HBM GB/s vs roofline at 40/160 rows"
L, H, D, T_FRAMES = 32, 20, 64, 1500
HD = H * D
KV_ROW_BYTES = H * D * 2 * 2  # K + V of one (row, cached position), fp16: 5120
SRC_BYTES = 4
FIXED_ROW_BYTES = 7680 + 5120 + 2560 + 2560 + 2560  # qkv read, append write, self out, cross q, cross out
CROSS_WINDOW_BYTES = T_FRAMES * H * D * 2 * 2  # 7,680,000 per window per layer
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    # 8 slots x beam 5, 80 cached positions, random parent permutation every step
    "config2": dict(windows=8, beams=5, capacity=228, off_lo=80, off_hi=80, refill_p=0.0, advance=False,
                    reorder="perm", refill_to=80, episode=0, desc="config 2: 8 slots x beam 5 = 40 rows, 80 cached positions (C = 228), "
                    "random parent permutation each step"),
    # 32 slots x beam 5, ragged U[4, 224], windows replaced (fresh length 4) with p = 0.02 per step
    "config3": dict(windows=32, beams=5, capacity=228, off_lo=4, off_hi=224, refill_p=0.02, advance=True,
                    reorder="perm", refill_to=4, episode=120, desc="config 3: 32 slots x beam 5 = 160 rows, cache lengths U[4, 224] "
                    "(C = 228), random parent reorder + append every step, windows replaced (fresh length 4) with "
                    "p = 0.02 per step"),
    # 16 slots x 5 samples, identity reorder, 224-token prompt prefix, lengths U[224, 447], C = 448
    # (the prompt prefix prefilled once per window in its first row and shared by the window's samples through the
    # slot table, as the reference's prefilled Search lays it out: search.py:440-443)
    "config4": dict(windows=16, beams=5, capacity=448, off_lo=224, off_hi=447, refill_p=0.0, advance=True,
                    reorder="identity", refill_to=224, episode=224, prefix=224, prefilled=True,
                    desc="config 4: 16 slots x 5 samples = 80 rows, identity reorder, 224-token prompt prefix shared "
                    "through the slot table, lengths U[224, 447] (C = 448)"),
    # 64 slots x beam 5 per GPU, U[4, 448], C = 448
    "config5": dict(windows=64, beams=5, capacity=448, off_lo=4, off_hi=447, refill_p=0.0, advance=True,
                    reorder="perm", refill_to=4, episode=200, desc="config 5: 64 slots x beam 5 = 320 rows per GPU, cache lengths U[4, 448] "
                    "(C = 448), random parent reorder every step"),
}


# --- the workload's schedule (host, deterministic) ------------------------------------------------------------
class Schedule:
    """Positions, parents and window replacements for ``n_steps`` steps of a workload (numpy, seeded).

    Windows start with cached lengths U[off_lo, off_hi]; every step each live window advances one position and its
    beams take random parents (a permutation; identity for sampling); a window is replaced by a fresh one (length
    ``refill_to``) with probability refill_p per step or when its cache is full. An episode (``episode`` steps,
    counted from step ``start``, the first timed step) is the workload's run: at each episode start every window is
    replaced by one with a fresh U[off_lo, off_hi] length, so any number of timed steps repeats the workload's
    episode."""

    def __init__(self, wl: dict, n_steps: int, seed: int, start: int = 0):
        rng = np.random.default_rng(seed)
        W, K, C = wl["windows"], wl["beams"], wl["capacity"]
        self.W, self.K, self.C, self.n = W, K, C, n_steps
        self.prefix = wl.get("prefix", 0)  # slots every row of a window reads from the window's first row

        def draw():
            return rng.integers(wl["off_lo"], wl["off_hi"] + 1, W).astype(np.int64)

        pos = draw()
        self.pos = np.zeros((n_steps + 1, W), dtype=np.int64)  # offsets used at step s
        self.refill = np.zeros((n_steps, W), dtype=bool)  # windows replaced after step s
        self.refill_pos = np.zeros((n_steps, W), dtype=np.int64)  # ... with these lengths
        self.parent = np.zeros((n_steps, W, K), dtype=np.int64)
        ep = wl["episode"]
        for s in range(n_steps):
            self.pos[s] = pos
            if wl["reorder"] == "perm":
                self.parent[s] = np.stack([rng.permutation(K) for _ in range(W)])
            else:
                self.parent[s] = np.arange(K)[None, :]
            if ep and s + 1 >= start and (s + 1 - start) % ep == 0:
                self.refill[s], self.refill_pos[s] = True, draw()
            elif wl["advance"]:
                fresh = (rng.random(W) < wl["refill_p"]) | (pos + 1 >= C)
                self.refill[s] = fresh
                self.refill_pos[s] = wl["refill_to"]
            if wl["advance"] or self.refill[s].any():
                pos = np.where(self.refill[s], self.refill_pos[s], pos + (1 if wl["advance"] else 0))
        self.pos[n_steps] = pos

    def kv_positions(self, p: np.ndarray, unique: bool = True) -> int:
        """(row, cached position) pairs whose K/V a layer reads for windows at offsets ``p``: every row's own, or,
        ``unique``, a shared prompt prefix once per window (its rows read it from the window's first row)."""
        if not unique or not self.prefix:
            return int(p.sum()) * self.K
        shared = np.minimum(p, self.prefix)
        return int(shared.sum() + self.K * (p - shared).sum())

    def step_bytes(self, s: int, windows: slice | None = None, unique: bool = True) -> int:
        """Algorithmic HBM bytes of step s (all 32 layers): per layer K/V of the cached positions (5120 B each; a
        shared prefix once per window when ``unique``) + the slot table (4 B per row and position) + rows*20480
        (qkv/append/outputs) + windows*7.68e6 (the cross K/V)."""
        p = self.pos[s] if windows is None else self.pos[s][windows]
        rows = p.size * self.K
        return L * (self.kv_positions(p, unique) * KV_ROW_BYTES + int(p.sum()) * self.K * SRC_BYTES
                    + rows * FIXED_ROW_BYTES + p.size * CROSS_WINDOW_BYTES)

    def cross_launch_bytes(self) -> int:
        return self.W * CROSS_WINDOW_BYTES + self.W * self.K * (2560 + 2560)

    def self_launch_bytes(self, p: np.ndarray, append: bool) -> int:
        """One self-attention launch at offsets ``p``: K/V (unique) + slot table + qkv in + output (+ the append)."""
        return (self.kv_positions(p) * KV_ROW_BYTES + int(p.sum()) * self.K * SRC_BYTES
                + self.W * self.K * (7680 + 2560 + (5120 if append else 0)))


def initial_src(W: int, K: int, C: int, seed: int, wl: dict | None = None) -> np.ndarray:
    """The slot tables at the start. Beam workloads: each slot column of a window a random permutation of its
    beams' rows -- what random parent permutations produce -- so every row reads distinct cache rows (no two rows of
    a window share a (row, slot): the bytes counted are the bytes the kernels must fetch). Identity reorder (sampled
    rows): each row its own. A prompt prefix (``wl["prefix"]`` slots) is read by every row of a window from the
    window's first row, where the reference's prefill writes it (search.py:440-443)."""
    wl = wl or {}
    if wl.get("reorder", "perm") == "perm":
        rng = np.random.default_rng(seed + 7)
        perm = np.argsort(rng.random((W, C, K)), axis=2)  # [W, C, K]: a permutation of the K beams per (window, slot)
        rows = (np.arange(W)[:, None, None] * K + perm).transpose(0, 2, 1).reshape(W * K, C)
    else:
        rows = np.repeat(np.arange(W * K)[:, None], C, axis=1)
    prefix = min(wl.get("prefix", 0), C)
    if prefix:
        rows[:, :prefix] = (np.arange(W * K) // K * K)[:, None]
    return rows.astype(np.int32)


def measured_hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "of measured"
    except Exception:
        return FALLBACK_HBM_GBS, "of fallback"


def profiled_traffic(workload: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary, if there is one
    (profiles/cross_attn_<workload>.md, a line ``traffic_bytes_per_launch: <n>``)."""
    p = ROOT / "profiles" / f"cross_attn_{workload}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# --- clocks during the timed region --------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons of one GPU, sampled from a thread every ~2 ms through NVML (read-only queries;
    a timed region of a few tens of ms still gets samples), else through ``nvidia-smi -lms 100``. ``stop(t0, t1)``
    keeps the samples taken inside [t0, t1] (host wall clock)."""

    QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc, self.thread, self.rows = None, None, []
        try:
            import threading

            import pynvml as nv

            nv.nvmlInit()
            h = nv.nvmlDeviceGetHandleByIndex(gpu_index)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                    nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
            self.stop_flag = threading.Event()

            def poll():
                while not self.stop_flag.is_set():
                    t = time.time()
                    mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.rows.append((t, mhz, self.max_mhz, ["Active" if r & b else "Not Active" for b in bits]))
                    time.sleep(0.002)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            self.source = "nvml, every ~2 ms"
            return
        except Exception:
            self.thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(gpu_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi, every 100 ms"
        except OSError:
            self.proc = None

    def _smi_rows(self) -> list:
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = []
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                ts += float("0." + parts[0].split(".")[1]) if "." in parts[0] else 0.0
                rows.append((ts, float(parts[2]), float(parts[3]), parts[5:9]))
            except (ValueError, IndexError):
                continue
        return rows

    def stop(self, t0: float, t1: float) -> dict:
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
            rows = list(self.rows)
        elif self.proc is not None:
            rows = self._smi_rows()
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "no clock source"}
        inside = [r for r in rows if t0 <= r[0] <= t1]
        note = f"samples inside the timed region ({self.source})"
        if not inside:
            inside = [r for r in rows if t0 - 0.15 <= r[0] <= t1 + 0.15]
            note = f"samples within 150 ms of the timed region ({self.source})"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "no samples"}
        reasons = sorted({n for r in inside for n, v in zip(self.NAMES, r[3]) if v.lower().startswith("active")})
        return {"sm_mhz": float(np.median([r[1] for r in inside])), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": reasons, "samples": len(inside), "note": note}


# --- our arm -----------------------------------------------------------------------------------------------------
def make_config(args, wl: dict, sch: Schedule, world: int) -> dict:
    """The ``config`` of a bench line, from rank 0's schedule (both arms print the same one for the same run)."""
    timed = range(args.warmup, args.warmup + args.steps)
    W, K, C = wl["windows"], wl["beams"], wl["capacity"]
    cfg = {"workload": wl["desc"], "name": args.workload, "rows": W * K, "windows": W, "beams": K, "layers": L,
           "heads": H, "head_dim": D, "frames": T_FRAMES, "capacity": C,
           "mean_cached_positions": round(float(np.mean([sch.pos[s].mean() for s in timed])), 1),
           "bytes_per_step": int(sum(sch.step_bytes(s) for s in timed) / args.steps),
           "parallelism": f"{world} independent shards (windows per GPU), no collective on the hot path",
           "l2": "inputs larger than L2: several GB read per step vs 126 MB L2; no flush",
           "graph": "one CUDA graph replay per step",
           "launch": "programmatic dependent launch" if not args.no_pdl else "plain launches"}
    if sch.prefix:
        cfg["prefix"] = sch.prefix
        cfg["bytes_per_step_logical"] = int(sum(sch.step_bytes(s, unique=False) for s in timed) / args.steps)
        cfg["bytes"] = ("unique: the shared prompt prefix counted once per window (its rows read it from the "
                        "window's first row); bytes_per_step_logical counts it per row")
    if wl.get("prefilled"):
        cfg["self_attn_prefix"] = ("per row" if args.no_shared_prefix else
                                   f"once per window: self_attn_step_triton(shared_prefix_group={K})")
    return cfg


def run_ours(args, rank: int, world: int, local_rank: int, light: bool = False) -> dict | None:
    """The workload on this rank's GPU; ``light``: the step and the per-kernel times only (no e2e leg)."""
    import torch

    from whisper_trt_b200 import attn_plugin as ap
    from whisper_trt_b200 import slots as sl

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    wl = WORKLOADS[args.workload]
    W, K, C = wl["windows"], wl["beams"], wl["capacity"]
    N = W * K
    n_sched = args.warmup + 2 * args.steps + 4
    seed = shard_seed(rank)  # each rank its own windows (independent shards)
    sch = Schedule(wl, n_sched, seed, start=args.warmup)

    g = torch.Generator(device=dev).manual_seed(seed)
    cache = torch.randn(L, 2, N, H, C, D, generator=g, device=dev, dtype=torch.float16)
    cross = torch.randn(L, 2, W, H, T_FRAMES, D, generator=g, device=dev, dtype=torch.float16)
    qkv = torch.randn(L, N, 1, 3 * HD, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(L, W, K, HD, generator=g, device=dev, dtype=torch.float16)
    y_self = torch.empty(L, N, 1, HD, device=dev, dtype=torch.float16)
    y_cross = torch.empty(L, W, K, HD, device=dev, dtype=torch.float16)
    src0 = torch.from_numpy(initial_src(W, K, C, seed, wl)).to(dev)
    src = src0.clone()
    pos = torch.from_numpy(sch.pos[0].copy()).to(dev)
    offset = pos.repeat_interleave(K).contiguous()
    parents_all = torch.from_numpy(sch.parent).to(dev)
    refill_slots_all = torch.from_numpy(np.where(sch.refill, np.arange(W)[None, :], -1).astype(np.int64)).to(dev)
    refill_mask_all = torch.from_numpy(sch.refill).to(dev)
    refill_pos_all = torch.from_numpy(sch.refill_pos).to(dev)
    rpos_cur = torch.empty(1, W, dtype=torch.long, device=dev)
    live_all = ~refill_mask_all
    step_idx = torch.zeros(1, dtype=torch.long, device=dev)
    parent_cur = torch.empty(1, W, K, dtype=torch.long, device=dev)
    slots_cur = torch.empty(1, W, dtype=torch.long, device=dev)
    mask_cur = torch.empty(1, W, dtype=torch.bool, device=dev)
    live_cur = torch.empty(1, W, dtype=torch.bool, device=dev)

    # a window's rows read one prefilled prompt through the slot table: its keys attended once per window
    spg = K if (wl.get("prefilled") and not args.no_shared_prefix) else None

    def layer(i, qkv_i=None, q_i=None):
        """Layer i's attention (its qkv and cross queries, or the given copies of them)."""
        ap.self_attn_step_triton(qkv[i] if qkv_i is None else qkv_i, cache[i, 0], cache[i, 1], offset, src,
                                 write_cache=True, out=y_self[i], shared_prefix_group=spg)
        ap.cross_attn_triton(q[i] if q_i is None else q_i, cross[i, 0], cross[i, 1], out=y_cross[i])

    def tail():
        """The step's bookkeeping from its schedule row (parent_cur .. rpos_cur): window replacements, then the
        parents' slot-table reorder and the offsets' advance."""
        sl.slot_reset(src, slots_cur.view(W), K, prefilled=wl.get("prefilled", False))
        torch.where(mask_cur.view(W), rpos_cur.view(W), pos, out=pos)
        sl.beam_reorder(src, parent_cur.view(W, K), pos, live=live_cur.view(W), offset=offset,
                        advance=wl["advance"])

    def step():
        for i in range(L):
            layer(i)
        torch.index_select(parents_all, 0, step_idx, out=parent_cur)
        torch.index_select(refill_slots_all, 0, step_idx, out=slots_cur)
        torch.index_select(refill_mask_all, 0, step_idx, out=mask_cur)
        torch.index_select(live_all, 0, step_idx, out=live_cur)
        torch.index_select(refill_pos_all, 0, step_idx, out=rpos_cur)
        tail()
        step_idx.add_(1)

    launches_per_step = 2 * L + 2

    def reset_state():
        src.copy_(src0)
        pos.copy_(torch.from_numpy(sch.pos[0].copy()))
        offset.copy_(pos.repeat_interleave(K))
        step_idx.zero_()

    # warm-up outside capture (workspaces), capture, then restart the schedule from step 0
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    reset_state()
    torch.cuda.synchronize(dev)

    dist = None
    if world > 1:
        import torch.distributed as dist_mod

        dist = dist_mod

    sampler = ClockSampler(gpu_index(local_rank))
    for _ in range(args.warmup):
        graph.replay()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0 = time.time()
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize(dev)
    t1 = time.time()
    if dist:
        dist.barrier()
    clocks = sampler.stop(t0, t1)
    elapsed_ms = ev0.elapsed_time(ev1)
    timed = range(args.warmup, args.warmup + args.steps)
    my_bytes = sum(sch.step_bytes(s) for s in timed)
    t_max, total_bytes = combine_ranks(elapsed_ms, my_bytes, dist, dev)
    ms_per_step = t_max / args.steps
    value = total_bytes / (t_max * 1e-3) / 1e9

    # per-kernel device times (roofline), at the schedule's state in the middle of the timed steps (the schedule
    # replayed from its start: the offsets the timed steps saw on average)
    reset_state()
    for _ in range(args.warmup + args.steps // 2):
        graph.replay()
    torch.cuda.synchronize(dev)
    ker = kernel_times(torch, ap, dev, qkv, cache, cross, q, y_self, y_cross, offset, src, sch, spg=spg)

    # end to end through the public API: H2D of the step's inputs from pinned memory, the step, D2H of its outputs
    e2e = None
    if not light:
        cur = {"parent": parent_cur, "slots": slots_cur, "mask": mask_cur, "live": live_cur, "rpos": rpos_cur}
        e2e = run_e2e(torch, dev, layer, tail, qkv, q, y_self, y_cross, cur, args.steps, reset_state, sch,
                      args.warmup, dist)

    peak, peak_kind = measured_hbm_peak()
    cross_bytes = sch.cross_launch_bytes()
    achieved = cross_bytes / (ker["cross_ms"] * 1e-3) / 1e9
    traffic = profiled_traffic(args.workload)
    res = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "us_per_step": round(ms_per_step * 1e3, 1),
        "rows_steps_per_s": round(N * world * args.steps / (t_max * 1e-3), 1), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "accumulate": "f32",
        "data": DATA,
        "config": make_config(args, wl, Schedule(wl, n_sched, shard_seed(0), start=args.warmup), world),
        "frac_of_hbm_peak": round(value / world / peak, 4), "hbm_peak_gbs": peak, "hbm_peak_kind": peak_kind,
        "roofline": {"bound": "hbm", "kernel": "cross_attn (cross_window_kernel: split + combine fused, one CTA per (window, head))",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": cross_bytes, "launch_us": round(ker["cross_ms"] * 1e3, 2),
                     "timing": "launch_us: the kernel's 32 layers' launches back to back in a CUDA graph (programmatic "
                               "dependent launch, as in the step), events around the replays / launches; "
                               "launch_us_isolated: one launch at a time between events",
                     "launch_us_isolated": round(ker["cross_iso_ms"] * 1e3, 2),
                     "frac_isolated": round(cross_bytes / (ker["cross_iso_ms"] * 1e-3) / 1e9 / peak, 4),
                     "traffic": traffic,
                     "self_attn": {"launch_us": round(ker["self_ms"] * 1e3, 2),
                                   "achieved": round(ker["self_bytes"] / (ker["self_ms"] * 1e-3) / 1e9, 1),
                                   "frac": round(ker["self_bytes"] / (ker["self_ms"] * 1e-3) / 1e9 / peak, 4),
                                   "launch_us_isolated": round(ker["self_iso_ms"] * 1e3, 2),
                                   "frac_isolated": round(ker["self_bytes"] / (ker["self_iso_ms"] * 1e-3) / 1e9
                                                          / peak, 4),
                                   "algorithmic_bytes_per_launch": ker["self_bytes"],
                                   "mean_cached_positions": round(ker["mean_cached_positions"], 1)}},
        "clocks": clocks, "gpu_launches": launches_per_step * args.steps,
    }
    if e2e is not None:
        res["e2e"] = e2e
    if L != 32:
        res["note"] = f"profiling case: {L} layers per step instead of the workload's 32 (not a bench value)"
    return res


def shard_seed(rank: int) -> int:
    """Each rank decodes its own windows (an independent shard): its inputs and schedule come from its own seed."""
    return 1234 + 7919 * rank


def combine_ranks(elapsed_ms: float, nbytes: int, dist, device) -> tuple[float, float]:
    """(max over ranks of the timed region, sum over ranks of the bytes) -- after the timed region, every rank in
    the same order; ``dist`` None for one process."""
    if dist is None:
        return float(elapsed_ms), float(nbytes)
    import torch

    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=device)
    b = torch.tensor([float(nbytes)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(b, op=dist.ReduceOp.SUM)
    return float(t.item()), float(b.item())


def gpu_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local_rank])
        except (ValueError, IndexError):
            return local_rank
    return local_rank


def kernel_times(torch, ap, dev, qkv, cache, cross, q, y_self, y_cross, offset, src, sch, reps: int = 3,
                 spg=None) -> dict:
    """Device time per launch of each attention kernel, two ways (CUDA events on the launching stream, warm):

    * chained -- each kernel alone, its 32 layers' launches back to back in a CUDA graph (with programmatic dependent
      launch, as in the step: a launch's start overlaps its predecessor's drain), events around the replays / 32;
    * isolated -- one launch at a time between events, self and cross alternating (no overlap: every launch pays
      its own ramp-up and drain).

    Algorithmic bytes use the offsets as they stand (after the timed steps)."""

    def graph_of(fn):
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def chained(fn) -> float:
        g = graph_of(fn)
        g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        del g
        return e0.elapsed_time(e1) / (reps * L)

    def self_all():
        for i in range(L):
            ap.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], offset, src, out=y_self[i],
                                     shared_prefix_group=spg)

    def cross_all():
        for i in range(L):
            ap.cross_attn_triton(q[i], cross[i, 0], cross[i, 1], out=y_cross[i])

    self_chain, cross_chain = chained(self_all), chained(cross_all)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(reps * L)]
    torch.cuda.synchronize(dev)
    torch.cuda._sleep(200_000_000)
    for r in range(reps):
        for i in range(L):
            e = evs[r * L + i]
            e[0].record()
            ap.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], offset, src, out=y_self[i],
                                     shared_prefix_group=spg)
            e[1].record()
            ap.cross_attn_triton(q[i], cross[i, 0], cross[i, 1], out=y_cross[i])
            e[2].record()
    torch.cuda.synchronize(dev)
    offs = offset.cpu().numpy()[:: sch.K]  # (a window's rows share its offset)
    return {"self_ms": self_chain, "cross_ms": cross_chain,
            "self_iso_ms": float(np.mean([e[0].elapsed_time(e[1]) for e in evs])),
            "cross_iso_ms": float(np.mean([e[1].elapsed_time(e[2]) for e in evs])),
            "self_bytes": sch.self_launch_bytes(offs, append=False),
            "mean_cached_positions": float(offs.mean())}


def run_e2e(torch, dev, layer, tail, qkv, q, y_self, y_cross, cur, steps, reset_state, sch, warmup,
            dist=None) -> dict:
    """The step through the public API with its inputs copied in from pinned host memory and its result copied
    out every step; whole-job GB/s (bytes summed over ranks, time the max).

    The inputs are each layer's qkv and cross queries and the step's schedule row (parents, window replacements),
    which the host writes into pinned staging before each step. The step's result is its last layer's attention
    outputs (self and cross), which the host reads back: the earlier layers' outputs feed the next layer on the
    device in a decoder and never cross PCIe (copying them all out too added 26 MB a step per rank, which 8 ranks
    sharing the host's links could not move in a step's time). One CUDA graph per step, the layers' inputs double-
    buffered on the device: step s computes from buffer s % 2 while its copy stream brings step s + 1's inputs (52.4
    MB at config 3) into the other buffer, so no layer waits for its own step's copy and a step costs the longer of
    its kernels and its copy, not their sum; the step's schedule row goes in first on the same stream, and a copy-out
    stream takes the last layer's outputs back after it. Two steps are in flight, as a serving loop keeps them: the
    host stages step s + 1's schedule row while step s runs (two pinned staging and output buffers, one graph for
    each) and reads each step's result once that step's completion event has fired, one step behind; every timed step
    copies one step's inputs in and one result out."""
    W, K = sch.W, sch.K
    qkv_h = torch.empty(qkv.shape, dtype=qkv.dtype, pin_memory=True)
    q_h = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    qkv_h.copy_(qkv)
    q_h.copy_(q)
    ys_h = [torch.empty(y_self.shape[1:], dtype=y_self.dtype, pin_memory=True) for _ in range(2)]
    yc_h = [torch.empty(y_cross.shape[1:], dtype=y_cross.dtype, pin_memory=True) for _ in range(2)]
    stage = [{k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in cur.items()} for _ in range(2)]
    arange_w = np.arange(W)

    def fill_stage(b: int, s: int) -> None:
        st = stage[b]
        st["parent"].numpy().reshape(W, K)[:] = sch.parent[s]
        st["slots"].numpy().reshape(W)[:] = np.where(sch.refill[s], arange_w, -1)
        st["mask"].numpy().reshape(W)[:] = sch.refill[s]
        st["live"].numpy().reshape(W)[:] = ~sch.refill[s]
        st["rpos"].numpy().reshape(W)[:] = sch.refill_pos[s]

    n = qkv.shape[0]
    qkv_buf, q_buf = (qkv, torch.empty_like(qkv)), (q, torch.empty_like(q))  # (buffer 0 holds step 0's inputs)
    cin, cout = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_out = torch.cuda.Event()
    ev_sched = torch.cuda.Event()

    def piped_step(b: int):
        main = torch.cuda.current_stream(dev)
        cin.wait_stream(main)
        cout.wait_stream(main)
        with torch.cuda.stream(cin):
            for k, v in cur.items():
                v.copy_(stage[b][k], non_blocking=True)
            ev_sched.record(cin)
            for i in range(n):  # the next step's inputs, under this step's kernels
                qkv_buf[1 - b][i].copy_(qkv_h[i], non_blocking=True)
                q_buf[1 - b][i].copy_(q_h[i], non_blocking=True)
        for i in range(n):
            layer(i, qkv_buf[b][i], q_buf[b][i])
        ev_out.record(main)
        cout.wait_event(ev_out)
        with torch.cuda.stream(cout):  # the step's result: the last layer's outputs
            ys_h[b].copy_(y_self[n - 1], non_blocking=True)
            yc_h[b].copy_(y_cross[n - 1], non_blocking=True)
        main.wait_event(ev_sched)
        tail()
        main.wait_stream(cin)
        main.wait_stream(cout)

    torch.cuda.synchronize(dev)
    graphs = []
    for b in range(2):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            piped_step(b)
        graphs.append(g)
    reset_state()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    done = [torch.cuda.Event(), torch.cuda.Event()]
    checksum = [0.0]

    def run(first: int, count: int) -> None:
        for s in range(first, first + count):
            b = s % 2
            if s - 2 >= first:
                done[b].synchronize()  # step s - 2 (this buffer's last user) is complete: read its result
                checksum[0] += float(ys_h[b][0, 0, 0]) + float(yc_h[b][0, 0, 0])
            fill_stage(b, s)
            graphs[b].replay()
            done[b].record(stream)
        for s in range(max(first, first + count - 2), first + count):  # the last two steps' results
            done[s % 2].synchronize()
            checksum[0] += float(ys_h[s % 2][0, 0, 0]) + float(yc_h[s % 2][0, 0, 0])

    run(0, warmup)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    run(warmup, steps)
    ev1.record()
    torch.cuda.synchronize(dev)
    ms, nbytes = combine_ranks(ev0.elapsed_time(ev1), sum(sch.step_bytes(s) for s in range(warmup, warmup + steps)),
                               dist, dev)
    h2d = sum(t.numel() * t.element_size() for t in (qkv, q, *cur.values()))
    d2h = sum(t.numel() * t.element_size() for t in (ys_h[0], yc_h[0]))
    del graphs
    # the copy-in alone (the layers' qkv and queries, 3 steps' worth), every rank at once after a barrier: the
    # pinned host-to-device rate each rank gets when all copy together -- the bound of the step above when the
    # kernels keep HBM busy
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cin):
        c0.record(cin)
        for _ in range(3):
            for i in range(n):
                qkv[i].copy_(qkv_h[i], non_blocking=True)
                q[i].copy_(q_h[i], non_blocking=True)
        c1.record(cin)
    torch.cuda.synchronize(dev)
    in_bytes = qkv.numel() * qkv.element_size() + q.numel() * q.element_size()
    copy_ms = c0.elapsed_time(c1) / 3
    copy_max, _ = combine_ranks(copy_ms, 0, dist, dev)
    return {"value": round(nbytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(ms / steps, 4),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "copy_in": {"bytes_per_step": in_bytes, "ms_per_step_all_ranks_at_once": round(copy_max, 4),
                        "gbs_per_rank": round(in_bytes / (copy_max * 1e-3) / 1e9, 2),
                        "gbs_whole_job": round(in_bytes * (dist.get_world_size() if dist else 1)
                                               / (copy_max * 1e-3) / 1e9, 1),
                        "note": "the layers' inputs copied alone from pinned host memory, every rank at once "
                                "(slowest rank): the bound on the e2e step"},
            "path": "whisper_trt_b200.attn_plugin calls (C ABI) captured in a CUDA graph; every step the host "
                    "stages the step's schedule row; the layers' qkv / queries are copied in from pinned host memory "
                    "one step ahead, into the other of two device buffers on a copy stream under this step's "
                    "kernels, and the step's result (the last layer's self and cross outputs) copied out; two steps "
                    "in flight: the host stages step s + 1 while step s runs and reads each step's result when its "
                    "completion event fires"}


# --- the reference's CPU implementation ---------------------------------------------------------------------------
REF_PKG = ROOT / "baseline" / "_ref"
DATA = ("synthetic: seeded N(0,1) fp16 caches / cross K/V / qkv / queries (random init; no checkpoint or dataset), "
        "seeded schedule of parents and window replacements")


def reference_module():
    """The reference's ``whisper_trt.attn_plugin``, imported unmodified from the package staged under
    ``baseline/_ref`` (None when it is not staged). Its ops' PyTorch bodies are selected (``RUNTIME_TRITON`` off:
    the reference's CPU path); its Triton launchers are called by name where the GPU comparison wants them."""
    if not (REF_PKG / "whisper_trt" / "attn_plugin.py").is_file():
        return None
    if str(REF_PKG) not in sys.path:
        sys.path.insert(0, str(REF_PKG))
    try:
        from whisper_trt import attn_plugin
    except Exception:
        return None
    attn_plugin.RUNTIME_TRITON = False
    return attn_plugin


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return 1


class CpuSample:
    """One layer of the workload's attention for a block of ``sw`` windows on the host cores, fp16 inputs with
    float32 math. With the reference package staged (``kind`` "reference"): the reference's own PyTorch ops on CPU
    tensors, in the order its TritonDecoderBackend calls them (runtime.py:139-145) -- ``self_attn`` through the slot
    table, the cache append its Search then does for that op (search.py:249-250), ``cross_attn_split`` and
    ``cross_attn_combine`` -- on all the host's cores (torch threads = the CPU count, under torchrun too). Without it
    (``kind`` "port"): their numpy restatement, ``oracle/attn.py``."""

    def __init__(self, wl: dict, sw: int, seed: int):
        rng = np.random.default_rng(seed)
        K, C = wl["beams"], wl["capacity"]
        self.sw, self.K, self.C = sw, K, C
        n = sw * K
        qkv = rng.standard_normal((n, 1, 3 * HD), dtype=np.float32).astype(np.float16)
        kc = rng.standard_normal((n, H, C, D), dtype=np.float32).astype(np.float16)
        vc = rng.standard_normal((n, H, C, D), dtype=np.float32).astype(np.float16)
        src = initial_src(sw, K, C, seed, wl)
        q = rng.standard_normal((sw, K, HD), dtype=np.float32).astype(np.float16)
        xk = rng.standard_normal((sw, H, T_FRAMES, D), dtype=np.float32).astype(np.float16)
        xv = rng.standard_normal((sw, H, T_FRAMES, D), dtype=np.float32).astype(np.float16)
        self.ops = reference_module()
        if self.ops is None:
            from oracle import attn as oa

            self.kind, self.oa = "port", oa
            self.np = (qkv, kc, vc, src, q, xk, xv)
            self.cores = cpu_threads()
            return
        import torch

        torch.set_num_threads(os.cpu_count() or 1)
        self.torch, self.kind, self.cores = torch, "reference", torch.get_num_threads()
        self.qkv, self.kc, self.vc = torch.from_numpy(qkv), torch.from_numpy(kc), torch.from_numpy(vc)
        self.src, self.q = torch.from_numpy(src), torch.from_numpy(q)
        self.xk, self.xv = torch.from_numpy(xk), torch.from_numpy(xv)
        self.rows = torch.arange(n)

    def run(self, offsets: np.ndarray) -> None:
        off = np.repeat(offsets[: self.sw], self.K)
        if self.ops is None:
            qkv, kc, vc, src, q, xk, xv = self.np
            self.oa.self_attn_step(qkv, kc, vc, off, src, write_cache=True)
            self.oa.cross_attn(q, xk, xv)
            return
        torch = self.torch
        o = torch.from_numpy(off)
        self.ops.self_attn(self.qkv, self.kc, self.vc, o, self.src)
        ok = o < self.C
        new = self.qkv.view(-1, 3, H, D)
        self.kc[self.rows[ok], :, o[ok]] = new[ok, 1]
        self.vc[self.rows[ok], :, o[ok]] = new[ok, 2]
        self.ops.cross_attn_combine(self.ops.cross_attn_split(self.q, self.xk, self.xv), self.q)

    def describe(self) -> str:
        if self.kind == "reference":
            return ("the reference's own PyTorch ops (whisper_trt.attn_plugin from baseline/_ref, RUNTIME_TRITON "
                    "off: self_attn + the cache append + cross_attn_split + cross_attn_combine) on CPU tensors")
        return "the reference's PyTorch op bodies restated in numpy (oracle/attn.py)"


def cpu_sample_bytes(sch: Schedule, s: int, sw: int) -> int:
    return sch.step_bytes(s, slice(0, sw)) // L  # one layer


def run_cpu_baseline(wl: dict, sch: Schedule, min_seconds: float, sw: int) -> dict:
    smp = CpuSample(wl, sw, seed=99)
    smp.run(sch.pos[0])  # warm-up
    t_total, nbytes, layers, s = 0.0, 0, 0, 0
    while t_total < min_seconds:
        t0 = time.perf_counter()
        smp.run(sch.pos[s % sch.n])
        t_total += time.perf_counter() - t0
        nbytes += cpu_sample_bytes(sch, s % sch.n, sw)
        layers += 1
        s += 1
    return {"value": round(nbytes / t_total / 1e9, 3), "unit": "GB/s", "cores": smp.cores, "kind": smp.kind,
            "host_cpus": os.cpu_count(),
            "sample": f"{layers} layer(s) of the workload's attention for {sw} of its {sch.W} windows "
                      f"({sw * sch.K} rows), {t_total:.1f} s: {smp.describe()}"}


def run_reference(args, world: int) -> dict:
    """``--impl reference``: the reference's CPU implementation of the path on the host cores, a bounded sample per
    step (one layer of the first ``sw`` windows at the step's offsets), same metric; value = the sample's algorithmic
    bytes / its time."""
    wl = WORKLOADS[args.workload]
    n_sched = args.warmup + 2 * args.steps + 4
    sch = Schedule(wl, n_sched, shard_seed(0), start=args.warmup)
    sw = min(wl["windows"], 2)
    smp = CpuSample(wl, sw, seed=99)
    for s in range(args.warmup):
        smp.run(sch.pos[s])
    t_total, nbytes, full = 0.0, 0, 0
    for s in range(args.warmup, args.warmup + args.steps):
        t0 = time.perf_counter()
        smp.run(sch.pos[s])
        t_total += time.perf_counter() - t0
        nbytes += cpu_sample_bytes(sch, s, sw)
        full += sch.step_bytes(s)
    value = nbytes / t_total / 1e9
    base = {"kind": smp.kind, "cores": smp.cores, "host_cpus": os.cpu_count(), "value": round(value, 3),
            "unit": "GB/s", "sample": f"per step one layer of the workload's attention for {sw} of its "
                                      f"{wl['windows']} windows ({sw * wl['beams']} rows): {smp.describe()}"}
    return {"metric": METRIC, "impl": "reference", "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_total / args.steps * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16", "accumulate": "f32",
            "data": DATA, "config": make_config(args, wl, sch, world),
            "extrapolated": {"sampled_layers_per_step": 1, "sampled_windows": sw, "of_layers": L,
                             "of_windows": wl["windows"],
                             "ms_per_full_step": round(t_total * full / nbytes / args.steps * 1e3, 1),
                             "note": "ms_per_step is the timed sample's; the whole step (all layers and windows) "
                                     "scaled by its algorithmic bytes is ms_per_full_step"},
            "cpu_baseline": base,
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_reference_gpu(local_rank: int, reps: int = 10) -> dict:
    """The reference's own GPU kernels beside this package's, on this GPU and the same inputs, at config 3 and
    config 2, each side captured in a CUDA graph (``benchmarks/triton_baseline.py``'s ``step`` and ``decoder_step``
    sections), with the clocks of the run: the decode step's attention of 32 layers as its TritonDecoderBackend
    sequences it (self_attn_step_triton with the append, then cross_attn_split_triton + cross_attn_combine_triton per
    layer), and the whole decode step through that backend itself."""
    R = reference_module()
    if R is None or getattr(R, "triton", None) is None:
        return {"unavailable": "the reference package (baseline/_ref) or Triton is not available"}
    sys.path.insert(0, str(ROOT / "benchmarks"))
    from types import SimpleNamespace

    import triton_baseline as tb
    import torch

    from whisper_trt_b200 import attn_plugin

    sampler = ClockSampler(gpu_index(local_rank))
    t0 = time.time()
    out = {}
    from whisper_trt_b200 import decoder_kernels

    ours = SimpleNamespace(attn_plugin=attn_plugin, decoder_kernels=decoder_kernels)
    for name in ("config3", "config2"):
        r = tb.step(R, ours, name, reps)
        out[name] = {k: r[k] for k in ("rows", "cached_mean", "bytes_per_step", "ref_step_us", "ref_step_unsplit_us",
                                       "ours_step_us", "ref_step_gbs", "ours_step_gbs", "speedup_vs_ref_step",
                                       "speedup_vs_ref_step_unsplit", "max_abs_diff")}
        torch.cuda.empty_cache()
        out[name]["decoder_step"] = {k: v for k, v in tb.decoder_step(R, ours, name, reps).items()
                                     if k not in ("section", "workload")}
        torch.cuda.empty_cache()
    out["clocks"] = sampler.stop(t0, time.time())
    out["how"] = ("device time per step of CUDA-graph replays (10 after 3 warm-up), the same seeded inputs and static "
                  "offsets on both sides; attention alone (no bookkeeping), and decoder_step: the whole 32-layer decode "
                  "step through the reference's own TritonDecoderBackend (random-init whisper-large-v3 decoder), as it "
                  "ships (ref_cublas) and with this package installed (ours_attn: attention + logits32; ours_attn_ln: also its "
                  "LayerNorms, the GEMMs still cuBLAS; ours_whole: "
                  "also the fused linear layers); the reference's Triton 3.6 kernels from baseline/_ref")
    return out


# --- main ----------------------------------------------------------------------------------------------------
def main() -> None:
    ap_ = argparse.ArgumentParser()
    ap_.add_argument("--gpus", type=int, default=1)
    ap_.add_argument("--steps", type=int, default=120)
    ap_.add_argument("--warmup", type=int, default=5)
    ap_.add_argument("--workload", default="config3", choices=sorted(WORKLOADS))
    ap_.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap_.add_argument("--cpu-seconds", type=float, default=10.0, help="cpu_baseline sample length (rank 0, N=1)")
    ap_.add_argument("--no-cpu-baseline", action="store_true")
    ap_.add_argument("--also", default="config2,config4,config5",
                     help="more workloads reported under 'also', at every N (comma-separated; '' = none)")
    ap_.add_argument("--no-ref-gpu", action="store_true",
                     help="skip the reference's Triton kernels timed beside these (N=1, rank 0)")
    ap_.add_argument("--no-shared-prefix", action="store_true",
                     help="config 4: attend each row's prompt prefix per row instead of once per window")
    ap_.add_argument("--no-pdl", action="store_true",
                     help="launch without programmatic dependent launch (default: with, WT_LAUNCH_PDL)")
    ap_.add_argument("--layers", type=int, default=32,
                     help="decoder layers per step (32 = the workload; fewer only for small profiling cases)")
    args = ap_.parse_args()
    global L
    L = args.layers
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:  # (the other ranks of a torchrun launch exit without work)
            print(json.dumps(run_reference(args, world)), flush=True)
        return

    import torch

    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    if not args.no_pdl:
        from whisper_trt_b200 import _lib

        _lib.set_launch_flags(_lib.WT_LAUNCH_PDL)
    res = run_ours(args, rank, world, local_rank)
    also = [w for w in args.also.split(",") if w and w != args.workload]
    if also:
        res["also"] = {}
    for name in also:  # (every rank runs the same workloads in the same order: the same collectives)
        torch.cuda.empty_cache()
        a = run_ours(argparse.Namespace(**{**vars(args), "workload": name}), rank, world, local_rank, light=True)
        res["also"][name] = {k: a[k] for k in ("value", "unit", "ms_per_step", "us_per_step", "rows_steps_per_s",
                                               "frac_of_hbm_peak", "clocks")} | {
            "workload": a["config"]["workload"], "mean_cached_positions": a["config"]["mean_cached_positions"],
            "bytes_per_step": a["config"]["bytes_per_step"], "roofline_frac": a["roofline"]["frac"],
            "self_attn_frac": a["roofline"]["self_attn"]["frac"]}
        if "bytes_per_step_logical" in a["config"]:
            res["also"][name]["bytes_per_step_logical"] = a["config"]["bytes_per_step_logical"]
            res["also"][name]["bytes"] = a["config"]["bytes"]
        if "self_attn_prefix" in a["config"]:
            res["also"][name]["self_attn_prefix"] = a["config"]["self_attn_prefix"]
    torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_ref_gpu:
        res["vs_reference_gpu"] = run_reference_gpu(local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        wl = WORKLOADS[args.workload]
        res["cpu_baseline"] = run_cpu_baseline(wl, Schedule(wl, args.warmup + args.steps + 4, shard_seed(0),
                                                            start=args.warmup), args.cpu_seconds,
                                               min(wl["windows"], 2))
    elif rank == 0:
        res["cpu_baseline"] = {"value": None, "note": "timed on rank 0 at N=1 only"}
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
