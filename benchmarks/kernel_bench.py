"""Time one kernel of the package on synthetic inputs (CUDA events on the launching stream, warm) and print one
JSON line -- the per-kernel numbers beside bench.py's whole-step line, and the commands the ncu summaries use.

    python benchmarks/kernel_bench.py beam_scores --windows 32 --beams 5 [--timestamps] [--reps 20]
    python benchmarks/kernel_bench.py logits32 --rows 160
    python benchmarks/kernel_bench.py prompt --rows 80 --tokens 224 --cached 0
    python benchmarks/kernel_bench.py cross --windows 32 --beams 5
    python benchmarks/kernel_bench.py cross_split --windows 32 --beams 5
    python benchmarks/kernel_bench.py self_step --rows 160 --cache-lo 4 --cache-hi 224
    python benchmarks/kernel_bench.py dec_linear --rows 160

(from the repository root). Inputs are seeded N(0, 1) (weights N(0, 0.02));
several layers' worth of inputs rotate so that consecutive calls do not hit L2 for the bytes they stream.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "whisper-trt_b200"))

from whisper_trt_b200 import attn_plugin as ap  # noqa: E402
from whisper_trt_b200 import slots  # noqa: E402


def _time(fn, reps: int) -> float:
    """Device time per call: the calls are queued behind a spin of the GPU so that the host's launch overhead does
    not space them out."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(100_000_000)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps * 1e-3


def beam_scores(a) -> dict:
    dev, V, W, K = "cuda", a.vocab, a.windows, a.beams
    g = torch.Generator(device=dev).manual_seed(0)
    cfg = SimpleNamespace(no_speech=50362, no_timestamps=50363, timestamp_begin=50365, eot=50257, vocab_size=V)
    s = SimpleNamespace(K=K, cfg=cfg, timestamps=a.timestamps, suppress=torch.zeros(V, dtype=torch.bool, device=dev),
                        begin=torch.zeros(V, dtype=torch.bool, device=dev),
                        t=torch.full((W,), 5, dtype=torch.int64, device=dev),
                        cum=torch.zeros(W * K, device=dev), hist=torch.zeros(W * K, 224, dtype=torch.int64, device=dev),
                        max_initial=torch.tensor([50], device=dev))
    logits = torch.randn(W * K, V, generator=g, device=dev)
    ns = torch.empty(W, device=dev)
    sec = _time(lambda: slots.best(s, logits, ns), a.reps)
    nb = logits.numel() * 4
    return {"kernel": "beam_scores", "windows": W, "beams": K, "vocab": V, "timestamps": a.timestamps,
            "us": round(sec * 1e6, 2), "gbs": round(nb / sec / 1e9, 1)}


def logits32(a) -> dict:
    dev, V, d, n = "cuda", a.vocab, a.d_model, a.rows
    g = torch.Generator(device=dev).manual_seed(0)
    L = 3
    x = torch.randn(L, n, 1, d, generator=g, device=dev).half()
    w = (torch.randn(L, V, d, generator=g, device=dev) * 0.02).half()
    out = torch.empty(n, 1, V, device=dev)
    i = [0]

    def run():
        j = i[0] % L
        i[0] += 1
        ap.logits32_triton(x[j], w[j], out=out)

    sec = _time(run, a.reps)
    nb = V * d * 2 + n * d * 2 + n * V * 4
    return {"kernel": "logits32", "rows": n, "vocab": V, "d_model": d, "us": round(sec * 1e6, 2),
            "gbs": round(nb / sec / 1e9, 1), "tflops": round(2 * n * V * d / sec / 1e12, 1)}


def prompt(a) -> dict:
    dev, N, S, C, H = "cuda", a.rows, a.tokens, a.capacity, 20
    g = torch.Generator(device=dev).manual_seed(0)
    L = 4
    qkv = torch.randn(L, N, S, 3 * H * 64, generator=g, device=dev).half()
    kc = torch.randn(N, H, C, 64, generator=g, device=dev).half()
    vc = torch.randn(N, H, C, 64, generator=g, device=dev).half()
    off = torch.full((N,), a.cached, dtype=torch.long, device=dev)
    src = torch.arange(N, dtype=torch.int32, device=dev)[:, None].expand(N, C).contiguous()
    y = torch.empty(N, S, H * 64, device=dev, dtype=torch.float16)
    i = [0]

    def run():
        j = i[0] % L
        i[0] += 1
        ap.self_attn_triton(qkv[j], kc, vc, off, src, out=y)

    sec = _time(run, a.reps)
    flops = N * H * 64 * 4 * (S * a.cached + S * (S + 1) / 2)
    return {"kernel": "self_attn (prompt)", "rows": N, "tokens": S, "cached": a.cached, "us": round(sec * 1e6, 2),
            "tflops": round(flops / sec / 1e12, 1)}


def cross(a) -> dict:
    dev, W, K, H, T = "cuda", a.windows, a.beams, 20, 1500
    g = torch.Generator(device=dev).manual_seed(0)
    L = max(2, -(-400_000_000 // (W * H * T * 64 * 4)))
    k = torch.randn(L, W, H, T, 64, generator=g, device=dev).half()
    v = torch.randn(L, W, H, T, 64, generator=g, device=dev).half()
    q = torch.randn(L, W, K, H * 64, generator=g, device=dev).half()
    out = torch.empty(W, K, H * 64, device=dev, dtype=torch.float16)
    i = [0]

    def run():
        j = i[0] % L
        i[0] += 1
        ap.cross_attn_triton(q[j], k[j], v[j], out=out)

    sec = _time(run, a.reps)
    nb = W * H * T * 64 * 4 + W * K * H * 64 * 4
    return {"kernel": "cross_attn", "windows": W, "queries": K, "us": round(sec * 1e6, 2),
            "gbs": round(nb / sec / 1e9, 1)}


def cross_split(a) -> dict:
    """The pair the reference's decoder backend calls per layer (runtime.py:144-145): cross_attn_split_triton (the
    stream-K kernel with (window, head, slice) units) then cross_attn_combine_triton, both timed."""
    dev, W, K, H, T = "cuda", a.windows, a.beams, 20, 1500
    g = torch.Generator(device=dev).manual_seed(0)
    L = max(2, -(-400_000_000 // (W * H * T * 64 * 4)))
    k = torch.randn(L, W, H, T, 64, generator=g, device=dev).half()
    v = torch.randn(L, W, H, T, 64, generator=g, device=dev).half()
    q = torch.randn(L, W, K, H * 64, generator=g, device=dev).half()
    part = torch.empty(W, H, ap.SPLITS, K, 66, device=dev)
    out = torch.empty(W, K, H * 64, device=dev, dtype=torch.float16)
    i = [0]

    def run():
        j = i[0] % L
        i[0] += 1
        ap.cross_attn_combine_triton(ap.cross_attn_split_triton(q[j], k[j], v[j], out=part), q[j], out=out)

    sec = _time(run, a.reps)
    nb = W * H * T * 64 * 4 + W * K * H * 64 * 4
    return {"kernel": "cross_attn_split + combine", "windows": W, "queries": K, "us": round(sec * 1e6, 2),
            "gbs": round(nb / sec / 1e9, 1)}


def self_step(a) -> dict:
    dev, N, C, H = "cuda", a.rows, a.capacity, 20
    g = torch.Generator(device=dev).manual_seed(0)
    L = 8
    kc = torch.randn(L, N, H, C, 64, generator=g, device=dev).half()
    vc = torch.randn(L, N, H, C, 64, generator=g, device=dev).half()
    qkv = torch.randn(L, N, 1, 3 * H * 64, generator=g, device=dev).half()
    off = torch.randint(a.cache_lo, a.cache_hi + 1, (N // 5,), generator=g, device=dev).repeat_interleave(5)
    src = ((torch.arange(N, device=dev) // 5 * 5)[:, None]
           + torch.randint(0, 5, (N, C), generator=g, device=dev)).to(torch.int32)
    y = torch.empty(N, 1, H * 64, device=dev, dtype=torch.float16)
    i = [0]

    def run():
        j = i[0] % L
        i[0] += 1
        ap.self_attn_step_triton(qkv[j], kc[j], vc[j], off, src, out=y)

    sec = _time(run, a.reps)
    nb = int(off.sum()) * H * 64 * 4 + N * 3 * H * 64 * 2
    return {"kernel": "self_attn_step", "rows": N, "capacity": C, "us": round(sec * 1e6, 2),
            "gbs": round(nb / sec / 1e9, 1)}


def dec_linear(a) -> dict:
    """The decoder step's six fused linear layers of one layer (whisper-large: d 1280, MLP 5120) at ``rows`` rows:
    qkv = ln_linear(x, 3d), y += out(attn) (linear_residual), q = ln_linear(x, d), y += xout(attn),
    h = ln_linear(x, 4d, gelu), y += fc2(h) -- each timed alone and the six in sequence. Each op rotates through
    enough weight copies (>= 256 MB, twice the L2) that its weights stream from HBM, as a decoder step's 32 layers'
    weights do. Bytes: weights + biases + the rows read and written."""
    from whisper_trt_b200 import _lib
    from whisper_trt_b200 import decoder_kernels as dk

    _lib.set_launch_flags(_lib.WT_LAUNCH_PDL)  # (as the decoder step launches them)
    dev, n, d = "cuda", a.rows, a.d_model
    g = torch.Generator(device=dev).manual_seed(0)

    def lin(o, i):
        copies = max(3, -(-(256 << 20) // (o * i * 2)))  # (the rotation exceeds L2)
        return ((torch.randn(copies, o, i, generator=g, device=dev) * 0.02).half(),
                (torch.randn(copies, o, generator=g, device=dev) * 0.02).half())
    W = {"qkv": lin(3 * d, d), "out": lin(d, d), "q": lin(d, d), "xout": lin(d, d), "fc1": lin(4 * d, d),
         "fc2": lin(d, 4 * d)}
    ln = [((1 + 0.1 * torch.randn(3, d, generator=g, device=dev)).half(),
           (0.1 * torch.randn(3, d, generator=g, device=dev)).half()) for _ in range(3)]
    x = torch.randn(n, d, generator=g, device=dev).half()
    y_attn = torch.randn(n, d, generator=g, device=dev).half()
    qkv = torch.empty(n, 3 * d, device=dev, dtype=torch.float16)
    q = torch.empty(n, d, device=dev, dtype=torch.float16)
    h = torch.empty(n, 4 * d, device=dev, dtype=torch.float16)
    i = [0]
    def wj(name, j):  # this op's weight copy for call j
        w, b = W[name]
        return w[j % w.shape[0]], b[j % w.shape[0]]

    ops = {
        "qkv": lambda j: dk.ln_linear(x, ln[0][0][j % 3], ln[0][1][j % 3], *wj("qkv", j), out=qkv),
        "out": lambda j: dk.linear_residual(y_attn, *wj("out", j), x, out=x),
        "q": lambda j: dk.ln_linear(x, ln[1][0][j % 3], ln[1][1][j % 3], *wj("q", j), out=q),
        "xout": lambda j: dk.linear_residual(y_attn, *wj("xout", j), x, out=x),
        "fc1": lambda j: dk.ln_linear(x, ln[2][0][j % 3], ln[2][1][j % 3], *wj("fc1", j), gelu=True, out=h),
        "fc2": lambda j: dk.linear_residual(h, *wj("fc2", j), x, out=x),
    }
    res = {"kernel": "dec_linear", "rows": n, "d_model": d}
    total_bytes = 0
    for name, op in ops.items():
        def run(op=op):
            j = i[0]
            i[0] += 1
            op(j)
        sec = _time(run, a.reps)
        o, k = W[name][0].shape[1:]
        nb = o * k * 2 + o * 2 + n * k * 2 + n * o * 2 + (n * o * 2 if name in ("out", "xout", "fc2") else 0)
        total_bytes += nb
        xin = {"qkv": x, "out": y_attn, "q": x, "xout": y_attn, "fc1": x, "fc2": h}[name]
        def base(name=name, xin=xin):  # cuBLAS through torch: the GEMM + bias alone, no LayerNorm / residual
            w, b = wj(name, i[0])
            i[0] += 1
            torch.addmm(b, xin, w.t())
        sec_b = _time(base, a.reps)
        res[name] = {"us": round(sec * 1e6, 2), "gbs": round(nb / sec / 1e9, 1), "torch_addmm_us": round(sec_b * 1e6, 2)}
    def layer():
        j = i[0]
        i[0] += 1
        for op in ops.values():
            op(j)
    sec = _time(layer, a.reps)
    res["layer_us"] = round(sec * 1e6, 2)
    res["layer_gbs"] = round(total_bytes / sec / 1e9, 1)
    res["step_32_layers_us"] = round(sec * 1e6 * 32, 1)
    return res


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("kernel", choices=["beam_scores", "logits32", "prompt", "cross", "cross_split", "self_step",
                                      "dec_linear"])
    p.add_argument("--windows", type=int, default=32)
    p.add_argument("--beams", type=int, default=5)
    p.add_argument("--vocab", type=int, default=51866)
    p.add_argument("--timestamps", action="store_true")
    p.add_argument("--rows", type=int, default=160)
    p.add_argument("--d-model", type=int, default=1280)
    p.add_argument("--tokens", type=int, default=224)
    p.add_argument("--cached", type=int, default=0)
    p.add_argument("--capacity", type=int, default=None, help="cache capacity (default: 448 prompt, 228 self_step)")
    p.add_argument("--cache-lo", type=int, default=4)
    p.add_argument("--cache-hi", type=int, default=224)
    p.add_argument("--reps", type=int, default=20)
    a = p.parse_args()
    assert torch.cuda.is_available(), "needs a CUDA GPU"
    if a.capacity is None:
        a.capacity = 228 if a.kernel == "self_step" else 448
    print(json.dumps(globals()[a.kernel](a)))


if __name__ == "__main__":
    main()
