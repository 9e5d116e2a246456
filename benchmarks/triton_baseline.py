"""The reference's own Triton kernels, timed on the same GPU as this package's kernels, on the same inputs -- the
GPU baseline beside ``bench.py`` (whose reference arm is the reference's CPU op bodies).

    python benchmarks/triton_baseline.py --ref baseline/_ref [--sections step,logits32,prompt,beam,decoder]

``--ref`` is a directory holding the reference's ``whisper_trt`` package, unmodified (its ``attn_plugin``,
``beam_kernels`` and ``decoder_kernels`` need only torch and Triton). When it is missing the module prints one
``{"unavailable": ...}`` line and exits 0. Each section prints one JSON line: device time per call or per step
(CUDA graphs of the calls, replayed between CUDA events after warm-up; inputs rotate or exceed L2) for the
reference's launchers and for this package's, and the largest difference between the two implementations' outputs
on the same inputs -- the reference's GPU kernels as a second parity anchor.

Sections (whisper-large-v3 shapes: 20 heads x 64, d 1280, 1500 frames, 32 layers, vocabulary 51866):

* ``step``: the decode step's attention of 32 layers, as the reference's ``TritonDecoderBackend`` sequences it
  (runtime.py:134-151: ``self_attn_step_triton(write_cache=True)`` -> ``cross_attn_split_triton`` ->
  ``cross_attn_combine_triton`` per layer; also with the unsplit ``cross_attn_triton``), against
  ``attn_plugin.self_attn_step_triton`` + ``attn_plugin.cross_attn_triton`` -- at config 2 (8 x 5 rows, 80 cached)
  and config 3 (32 x 5 rows, cached U[4, 224]), C = 228;
* ``logits32``: ``logits32_triton`` at 160 rows (attn_plugin.py:549-560);
* ``prompt``: ``self_attn_triton`` at 80 rows x a 224-token prompt (attn_plugin.py:462-479);
* ``beam``: ``beam_kernels.scores`` + the step's ``topk`` (search.py:252-253) against ``slots.best`` at 32 x 5 rows;
* ``decoder``: ``decoder_kernels.ln_linear`` / ``linear_residual`` (autotuned on first call) at 160 rows;
* ``decoder_step``: the whole decode step through the reference's own ``TritonDecoderBackend`` (its kernels, and
  this package installed into its modules) at config 2 and config 3.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "whisper-trt_b200"))

H, D, T, L = 20, 64, 1500, 32

STEP_CONFIGS = {
    "config2": dict(windows=8, beams=5, capacity=228, lo=80, hi=80),
    "config3": dict(windows=32, beams=5, capacity=228, lo=4, hi=224),
}


def _graph(fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def _time(fn, reps: int) -> float:
    """Seconds per call of ``fn`` captured once in a CUDA graph, replayed ``reps`` times after 3 warm-up replays."""
    g = _graph(fn)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) / reps * 1e-3


def _maxdiff(a: torch.Tensor, b: torch.Tensor) -> float:
    return float((a.float() - b.float()).abs().max())


def step(R, ours, name: str, reps: int) -> dict:
    c = STEP_CONFIGS[name]
    W, K, C = c["windows"], c["beams"], c["capacity"]
    N = W * K
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    cache = torch.randn(L, 2, N, H, C, D, generator=g, device=dev, dtype=torch.float16)
    cross = torch.randn(L, 2, W, H, T, D, generator=g, device=dev, dtype=torch.float16)
    qkv = torch.randn(L, N, 1, 3 * H * D, generator=g, device=dev, dtype=torch.float16)
    q = torch.randn(L, W, K, H * D, generator=g, device=dev, dtype=torch.float16)
    off = torch.randint(c["lo"], c["hi"] + 1, (W,), generator=g, device=dev).repeat_interleave(K)
    src = ((torch.arange(N, device=dev) // K * K)[:, None]
           + torch.randint(0, K, (N, C), generator=g, device=dev)).to(torch.int32)
    ys = torch.empty(L, N, 1, H * D, device=dev, dtype=torch.float16)
    yc = torch.empty(L, W, K, H * D, device=dev, dtype=torch.float16)
    ap = ours.attn_plugin

    def ref_self():
        for i in range(L):
            R.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], off, src, write_cache=True)

    def ref_split():
        for i in range(L):
            R.cross_attn_combine_triton(R.cross_attn_split_triton(q[i], cross[i, 0], cross[i, 1]), q[i])

    def ref_unsplit():
        for i in range(L):
            R.cross_attn_triton(q[i], cross[i, 0], cross[i, 1])

    def ref_step():
        for i in range(L):
            R.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], off, src, write_cache=True)
            R.cross_attn_combine_triton(R.cross_attn_split_triton(q[i], cross[i, 0], cross[i, 1]), q[i])

    def ref_step_unsplit():
        for i in range(L):
            R.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], off, src, write_cache=True)
            R.cross_attn_triton(q[i], cross[i, 0], cross[i, 1])

    def our_self():
        for i in range(L):
            ap.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], off, src, write_cache=True, out=ys[i])

    def our_cross():
        for i in range(L):
            ap.cross_attn_triton(q[i], cross[i, 0], cross[i, 1], out=yc[i])

    def our_step():
        for i in range(L):
            ap.self_attn_step_triton(qkv[i], cache[i, 0], cache[i, 1], off, src, write_cache=True, out=ys[i])
            ap.cross_attn_triton(q[i], cross[i, 0], cross[i, 1], out=yc[i])

    # parity on layer 0 (both write the same new keys / values at the offsets, so the caches stay identical)
    r_self = R.self_attn_step_triton(qkv[0], cache[0, 0], cache[0, 1], off, src, write_cache=True)
    r_cross = R.cross_attn_combine_triton(R.cross_attn_split_triton(q[0], cross[0, 0], cross[0, 1]), q[0])
    r_unsplit = R.cross_attn_triton(q[0], cross[0, 0], cross[0, 1])
    o_self = ap.self_attn_step_triton(qkv[0], cache[0, 0], cache[0, 1], off, src, write_cache=True)
    o_cross = ap.cross_attn_triton(q[0], cross[0, 0], cross[0, 1])
    torch.cuda.synchronize()
    nbytes = L * (int(off.sum()) * (H * D * 4 + 4) + N * 20480 + W * T * H * D * 4)
    t = {k: _time(f, reps) for k, f in (("ref_step", ref_step), ("ref_step_unsplit", ref_step_unsplit),
                                        ("ours_step", our_step), ("ref_self", ref_self), ("ref_cross_split", ref_split),
                                        ("ref_cross_unsplit", ref_unsplit), ("ours_self", our_self),
                                        ("ours_cross", our_cross))}
    out = {"section": "step", "workload": name, "rows": N, "windows": W, "capacity": C,
           "cached_mean": round(float(off.float().mean()), 1), "bytes_per_step": nbytes}
    for k, sec in t.items():
        out[f"{k}_us"] = round(sec * 1e6, 1)
    for k in ("ref_step", "ref_step_unsplit", "ours_step"):
        out[f"{k}_gbs"] = round(nbytes / t[k] / 1e9, 1)
    out["speedup_vs_ref_step"] = round(t["ref_step"] / t["ours_step"], 2)
    out["speedup_vs_ref_step_unsplit"] = round(t["ref_step_unsplit"] / t["ours_step"], 2)
    out["max_abs_diff"] = {"self": _maxdiff(o_self, r_self), "cross_vs_split": _maxdiff(o_cross, r_cross),
                           "cross_vs_unsplit": _maxdiff(o_cross, r_unsplit)}
    return out


def logits32(R, ours, reps: int, rows: int = 160, V: int = 51866, d: int = 1280) -> dict:
    dev, n = "cuda", 3
    g = torch.Generator(device=dev).manual_seed(0)
    x = torch.randn(n, rows, 1, d, generator=g, device=dev).half()
    w = (torch.randn(n, V, d, generator=g, device=dev) * 0.02).half()
    yr = torch.empty(rows, 1, V, device=dev)
    yo = torch.empty(rows, 1, V, device=dev)
    R.logits32_triton(x[0], w[0], out=yr)
    ours.attn_plugin.logits32_triton(x[0], w[0], out=yo)
    torch.cuda.synchronize()
    diff = _maxdiff(yo, yr) / float(yr.abs().max())

    def ref():
        for j in range(n):
            R.logits32_triton(x[j], w[j], out=yr)

    def our():
        for j in range(n):
            ours.attn_plugin.logits32_triton(x[j], w[j], out=yo)

    tr, to = _time(ref, reps) / n, _time(our, reps) / n
    return {"section": "logits32", "rows": rows, "vocab": V, "ref_us": round(tr * 1e6, 2),
            "ours_us": round(to * 1e6, 2), "speedup": round(tr / to, 2), "max_rel_diff": diff}


def prompt(R, ours, reps: int, rows: int = 80, S: int = 224, C: int = 448) -> dict:
    dev, n = "cuda", 3
    g = torch.Generator(device=dev).manual_seed(0)
    qkv = torch.randn(n, rows, S, 3 * H * D, generator=g, device=dev).half()
    kc = torch.randn(rows, H, C, D, generator=g, device=dev).half()
    vc = torch.randn(rows, H, C, D, generator=g, device=dev).half()
    off = torch.zeros(rows, dtype=torch.long, device=dev)
    src = torch.arange(rows, dtype=torch.int32, device=dev)[:, None].expand(rows, C).contiguous()
    y = torch.empty(rows, S, H * D, device=dev, dtype=torch.float16)
    r = R.self_attn_triton(qkv[0], kc, vc, off, src)
    o = ours.attn_plugin.self_attn_triton(qkv[0], kc, vc, off, src)
    torch.cuda.synchronize()
    diff = _maxdiff(o, r)

    def ref():
        for j in range(n):
            R.self_attn_triton(qkv[j], kc, vc, off, src)

    def our():
        for j in range(n):
            ours.attn_plugin.self_attn_triton(qkv[j], kc, vc, off, src, out=y)

    tr, to = _time(ref, reps) / n, _time(our, reps) / n
    return {"section": "prompt", "rows": rows, "tokens": S, "ref_us": round(tr * 1e6, 2), "ours_us": round(to * 1e6, 2),
            "speedup": round(tr / to, 2), "max_abs_diff": diff}


def beam(RB, ours, reps: int, W: int = 32, K: int = 5, V: int = 51866) -> dict:
    dev, n = "cuda", 3
    g = torch.Generator(device=dev).manual_seed(0)
    cfg = SimpleNamespace(no_speech=50362, no_timestamps=50363, timestamp_begin=50365, eot=50257, vocab_size=V)
    s = SimpleNamespace(K=K, B=W, cfg=cfg, timestamps=False, mixed=False,
                        suppress=torch.zeros(V, dtype=torch.bool, device=dev),
                        begin=torch.zeros(V, dtype=torch.bool, device=dev),
                        t=torch.full((W,), 5, dtype=torch.int64, device=dev),
                        cum=torch.randn(W * K, generator=g, device=dev),
                        hist=torch.zeros(W * K, 224, dtype=torch.int64, device=dev),
                        max_initial=torch.tensor([50], device=dev),
                        sampling=torch.zeros(W, dtype=torch.bool, device=dev))
    logits = torch.randn(n, W * K, V, generator=g, device=dev) * 3
    scores = torch.empty(W * K, V, device=dev)
    ns_r = torch.empty(W, device=dev)
    ns_o = torch.empty(W, device=dev)
    RB.scores(s, logits[0], scores, ns_r)
    r_s, r_i = scores.view(W, -1).topk(2 * K, dim=1)
    o_s, o_i = ours.slots.best(s, logits[0], ns_o)
    torch.cuda.synchronize()
    same = bool(torch.equal(r_i, o_i))

    def ref():
        for j in range(n):
            RB.scores(s, logits[j], scores, ns_r)
            scores.view(W, -1).topk(2 * K, dim=1)

    def our():
        for j in range(n):
            ours.slots.best(s, logits[j], ns_o)

    tr, to = _time(ref, reps) / n, _time(our, reps) / n
    return {"section": "beam", "windows": W, "beams": K, "vocab": V, "ref_us": round(tr * 1e6, 2),
            "ours_us": round(to * 1e6, 2), "speedup": round(tr / to, 2), "top_tokens_identical": same,
            "max_abs_diff_scores": _maxdiff(o_s, r_s), "max_abs_diff_no_speech": _maxdiff(ns_o, ns_r)}


def decoder(RD, ours, reps: int, rows: int = 160, d: int = 1280) -> dict:
    """Each op rotates through enough weight copies (>= 256 MB, twice the L2) that its weights stream from HBM, as
    the 32 layers' weights of a decoder step do."""
    dev = "cuda"
    dk = ours.decoder_kernels
    g = torch.Generator(device=dev).manual_seed(0)

    def lin(o, i):
        copies = max(3, -(-(256 << 20) // (o * i * 2)))
        return ((torch.randn(copies, o, i, generator=g, device=dev) * 0.02).half(),
                (torch.randn(copies, o, generator=g, device=dev) * 0.02).half())

    Wt = {"qkv": lin(3 * d, d), "out": lin(d, d), "q": lin(d, d), "xout": lin(d, d), "fc1": lin(4 * d, d),
          "fc2": lin(d, 4 * d)}
    ga = (1 + 0.1 * torch.randn(3, d, generator=g, device=dev)).half()
    be = (0.1 * torch.randn(3, d, generator=g, device=dev)).half()
    x = torch.randn(rows, d, generator=g, device=dev).half()
    ya = torch.randn(rows, d, generator=g, device=dev).half()
    h = (torch.randn(rows, 4 * d, generator=g, device=dev) * 0.5).half()
    outs = {k: torch.empty(rows, w.shape[1], device=dev, dtype=torch.float16) for k, (w, _) in Wt.items()}

    def call(mod, name, j):
        w, b = Wt[name][0][j], Wt[name][1][j]
        if name in ("qkv", "q", "fc1"):
            return mod.ln_linear(x, ga[j % 3], be[j % 3], w, b, gelu=name == "fc1", out=outs[name])
        return mod.linear_residual(h if name == "fc2" else ya, w, b, x, out=outs[name])

    res = {"section": "decoder", "rows": rows, "d_model": d}
    tot_r = tot_o = 0.0
    for name in Wt:
        r = call(RD, name, 0).clone()
        o = call(dk, name, 0).clone()
        torch.cuda.synchronize()
        n = Wt[name][0].shape[0]
        tr = _time(lambda: [call(RD, name, j) for j in range(n)], reps) / n
        to = _time(lambda: [call(dk, name, j) for j in range(n)], reps) / n
        tot_r += tr
        tot_o += to
        res[name] = {"ref_us": round(tr * 1e6, 2), "ours_us": round(to * 1e6, 2), "max_abs_diff": _maxdiff(o, r),
                     "identical_frac": round(float((o == r).float().mean()), 4)}
    res["layer_ref_us"] = round(tot_r * 1e6, 1)
    res["layer_ours_us"] = round(tot_o * 1e6, 1)
    res["speedup"] = round(tot_r / tot_o, 2)
    return res


LARGE_V3 = dict(n_mels=128, d_model=1280, enc_layers=32, enc_heads=20, enc_ffn=5120, dec_layers=32, dec_heads=20,
                dec_ffn=5120, vocab_size=51866)


def decoder_step(R, ours, name: str, reps: int, ref_gemm_triton: bool = False) -> dict:
    """The whole decode step: the reference's own ``TritonDecoderBackend.step_fn`` closure (runtime.py:125-174) on
    a whisper-large-v3-shaped random-init decoder (``modeling.Decoder(cfg)``, fp16), captured in a CUDA graph and
    replayed: 32 layers of LayerNorm, QKV, self-attention with the append, out-projection, LayerNorm, query,
    cross-attention, out-projection, MLP; the final LayerNorm and the vocabulary projection. Variants:

    * ``ref_cublas``: the reference as it ships (its Triton attention and LayerNorm kernels, cuBLAS GEMMs, its
      logits32 kernel);
    * ``ours_attn``: the same backend with this package installed into its ``attn_plugin`` (attention, logits32);
    * ``ours_attn_ln``: the same, and this package's ``decoder_kernels`` installed too -- in the cuBLAS step that
      routes the three LayerNorms per layer (``layer_norm_bias``) to this package; the GEMMs stay cuBLAS;
    * ``ours_whole``: its ``gemm="triton"`` variant with this package installed into ``attn_plugin`` and
      ``decoder_kernels``: every kernel of the step but the embedding gather, the final LayerNorm and one cast;
    * ``ref_triton`` (with ``ref_gemm_triton``): the reference's own ``gemm="triton"`` variant (autotunes first).

    The ``gemm="triton"`` variants leave the new keys/values in ``new_kv`` for the search to scatter (the cuBLAS
    variant appends them itself). Inputs: the workload's rows and cache lengths, window-local random slot tables."""
    from whisper_trt import config as RC
    from whisper_trt import decoder_kernels as RDK
    from whisper_trt import modeling as RM
    from whisper_trt import runtime as RR

    c = STEP_CONFIGS[name]
    W, K, C = c["windows"], c["beams"], c["capacity"]
    N = W * K
    cfg = RC.WhisperConfig(**LARGE_V3)
    torch.manual_seed(0)
    with torch.device("cuda"):
        dec = RM.Decoder(cfg)
    dec = dec.half().eval().requires_grad_(False)
    model = SimpleNamespace(cfg=cfg, decoder=dec)
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    tokens = torch.randint(0, 50000, (N, 1), generator=g, device=dev)
    off = torch.randint(c["lo"], c["hi"] + 1, (W,), generator=g, device=dev).repeat_interleave(K)
    src = ((torch.arange(N, device=dev) // K * K)[:, None]
           + torch.randint(0, K, (N, C), generator=g, device=dev)).to(torch.int32)
    cache = torch.randn(L, 2, N, H, C, D, generator=g, device=dev, dtype=torch.float16)
    cross = torch.randn(L, 2, W, H, T, D, generator=g, device=dev, dtype=torch.float16)
    logits = torch.empty(N, 1, cfg.vocab_size, device=dev)
    new_kv = torch.empty(L, 2, N, H, 1, D, device=dev, dtype=torch.float16)
    saved = [(m, dict(vars(m))) for m in (R, RDK)]

    def restore():
        for m, names in saved:
            for k, v in names.items():
                setattr(m, k, v)

    variants = [("ref_cublas", "cublas", False, False), ("ours_attn", "cublas", True, False),
                ("ours_attn_ln", "cublas", True, True), ("ours_whole", "triton", True, True)]
    if ref_gemm_triton:
        variants.append(("ref_triton", "triton", False, False))
    out = {"section": "decoder_step", "workload": name, "rows": N, "windows": W, "capacity": C,
           "cached_mean": round(float(off.float().mean()), 1)}
    # every variant captured first (each with its own cache copy and logits), then timed interleaved over `rounds`
    # rounds -- the median per variant -- so that neither order nor the box's drift favours one. Each variant's step
    # closure (and with it its backend, cache copy and concatenated weights) is kept for as long as its graph: a
    # capture begins with torch.cuda.empty_cache(), which would unmap a dropped variant's buffers under its graph.
    graphs, lgs, alive = {}, {}, {}
    for label, gemm, attn, lin in variants:
        try:
            if attn:
                ours.attn_plugin.install(R)
            if lin:
                ours.decoder_kernels.install(RDK)
            backend = RR.TritonDecoderBackend(model, encoder=None, gemm=gemm)
            lgs[label] = torch.empty_like(logits)
            run = backend.step_fn(tokens, off, cache.clone(), lgs[label], new_kv.clone(), src, cross)
            alive[label] = (backend, run)
            graphs[label] = _graph(run)
        finally:
            restore()
    rounds = 5
    times = {label: [] for label in graphs}
    for _ in range(rounds):
        for label, g in graphs.items():
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            times[label].append(e0.elapsed_time(e1) / reps * 1e3)
    for label in graphs:
        out[f"{label}_us"] = round(sorted(times[label])[rounds // 2], 1)
        out[f"{label}_max_logit_diff_vs_ref_cublas"] = _maxdiff(lgs[label], lgs["ref_cublas"])
    out["timing"] = f"median of {rounds} interleaved rounds of {reps} graph replays per variant"
    del graphs
    del alive
    torch.cuda.empty_cache()
    out["speedup_ours_attn"] = round(out["ref_cublas_us"] / out["ours_attn_us"], 3)
    out["speedup_ours_attn_ln"] = round(out["ref_cublas_us"] / out["ours_attn_ln_us"], 3)
    out["speedup_ours_whole"] = round(out["ref_cublas_us"] / out["ours_whole_us"], 3)
    return out


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--ref", default="baseline/_ref", help="directory holding the reference's whisper_trt package")
    p.add_argument("--sections", default="step,logits32,prompt,beam,decoder,decoder_step")
    p.add_argument("--workloads", default="config3,config2")
    p.add_argument("--reps", type=int, default=10)
    p.add_argument("--ref-gemm-triton", action="store_true",
                   help="decoder_step: also time the reference's own gemm='triton' variant (autotunes first)")
    a = p.parse_args()
    ref = Path(a.ref).resolve()
    if not (ref / "whisper_trt" / "attn_plugin.py").is_file():
        print(json.dumps({"unavailable": f"no reference package under {ref}"}))
        return
    assert torch.cuda.is_available(), "needs a CUDA GPU"
    sys.path.insert(0, str(ref))
    from whisper_trt import attn_plugin as R
    from whisper_trt import beam_kernels as RB
    from whisper_trt import decoder_kernels as RD

    from whisper_trt_b200 import _lib, attn_plugin, decoder_kernels, slots

    _lib.set_launch_flags(_lib.WT_LAUNCH_PDL)  # (as the decoder step launches this package's kernels)
    ours = SimpleNamespace(attn_plugin=attn_plugin, decoder_kernels=decoder_kernels, slots=slots)
    print(json.dumps({"device": torch.cuda.get_device_name(), "torch": torch.__version__,
                      "triton": __import__("triton").__version__}), flush=True)
    for sec in a.sections.split(","):
        if sec == "step":
            for wl in a.workloads.split(","):
                print(json.dumps(step(R, ours, wl, a.reps)), flush=True)
                torch.cuda.empty_cache()
        elif sec == "logits32":
            print(json.dumps(logits32(R, ours, a.reps)), flush=True)
        elif sec == "prompt":
            print(json.dumps(prompt(R, ours, a.reps)), flush=True)
        elif sec == "beam":
            print(json.dumps(beam(RB, ours, a.reps)), flush=True)
        elif sec == "decoder":
            print(json.dumps(decoder(RD, ours, a.reps)), flush=True)
        elif sec == "decoder_step":
            for wl in a.workloads.split(","):
                print(json.dumps(decoder_step(R, ours, wl, a.reps, ref_gemm_triton=a.ref_gemm_triton)), flush=True)
                torch.cuda.empty_cache()
        else:
            raise SystemExit(f"unknown section {sec!r}")
        torch.cuda.empty_cache()
    assert attn_plugin.workspace_errors() == 0


if __name__ == "__main__":
    main()
