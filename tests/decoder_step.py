"""A Whisper decoder step whose attention runs on these kernels -- the counterpart of the reference's
``TritonDecoderBackend.step_fn`` (runtime.py:125-174, ``run_cublas`` :134-151).

Per layer, in the reference's order: LayerNorm (fp32 statistics) that also adds the next residual GEMM's bias to the
residual stream; the fused Q/K/V GEMM (k bias zero, ``modeling.Attention.fuse_qkv``); self-attention of the new token
through the slot table, which appends its keys/values to the cache (``writes_cache``); the output projection into the
residual; LayerNorm, query GEMM, cross-attention over the window's encoder frames, output projection; LayerNorm,
fc1, GELU, fc2. Then the final LayerNorm and the vocabulary projection with fp32 accumulation (logits fp32).
GEMMs and LayerNorms are PyTorch (cuBLAS); the attention goes through the C ABI (``attn_plugin``).

The weights use the checkpoint's names (``layers.{i}.self_attn.q_proj.weight`` ...); :meth:`Decoder.random` makes a
seeded random-init decoder of any size (whisper-large-v3: 32 layers, d 1280, 20 heads, ffn 5120, 51866 tokens).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn.functional as F

from whisper_trt_b200 import attn_plugin


@dataclass(frozen=True)
class DecoderShape:
    layers: int = 32
    d_model: int = 1280
    heads: int = 20
    ffn: int = 5120
    vocab: int = 51866
    max_positions: int = 448

    @property
    def head_dim(self) -> int:
        return self.d_model // self.heads


class Decoder:
    """Decoder weights (on one device) and the step closure over caller-owned buffers."""

    def __init__(self, shape: DecoderShape, weights: dict[str, torch.Tensor]):
        self.shape, self.w = shape, weights
        d = shape.d_model
        self.layers = []
        for i in range(shape.layers):
            p = f"layers.{i}."
            g = lambda n: weights[p + n]  # noqa: E731
            qkv_w = torch.cat([g("self_attn.q_proj.weight"), g("self_attn.k_proj.weight"),
                               g("self_attn.v_proj.weight")]).contiguous()
            qkv_b = torch.cat([g("self_attn.q_proj.bias"), torch.zeros_like(g("self_attn.q_proj.bias")),
                               g("self_attn.v_proj.bias")]).contiguous()
            self.layers.append({
                "ln1": (g("self_attn_layer_norm.weight"), g("self_attn_layer_norm.bias")),
                "qkv": (qkv_w, qkv_b), "out": (g("self_attn.out_proj.weight"), g("self_attn.out_proj.bias")),
                "ln2": (g("encoder_attn_layer_norm.weight"), g("encoder_attn_layer_norm.bias")),
                "q": (g("encoder_attn.q_proj.weight"), g("encoder_attn.q_proj.bias")),
                "xk": g("encoder_attn.k_proj.weight"),
                "xv": (g("encoder_attn.v_proj.weight"), g("encoder_attn.v_proj.bias")),
                "xout": (g("encoder_attn.out_proj.weight"), g("encoder_attn.out_proj.bias")),
                "ln3": (g("final_layer_norm.weight"), g("final_layer_norm.bias")),
                "fc1": (g("fc1.weight"), g("fc1.bias")), "fc2": (g("fc2.weight"), g("fc2.bias")),
            })
        self.embed = weights["embed_tokens.weight"]
        self.pos = weights["embed_positions.weight"]
        self.final = (weights["layer_norm.weight"], weights["layer_norm.bias"])
        self._embed32 = None
        assert self.embed.shape == (shape.vocab, d)

    @classmethod
    def random(cls, shape: DecoderShape = DecoderShape(), seed: int = 0, device="cuda", dtype=torch.float16,
               std: float = 0.02) -> "Decoder":
        """Seeded random-init weights, N(0, std) (LayerNorm gains 1 + N(0, std), biases N(0, std))."""
        g = torch.Generator(device=device).manual_seed(seed)
        d, f = shape.d_model, shape.ffn

        def rnd(*s, mean=0.0):
            return (torch.randn(*s, generator=g, device=device, dtype=torch.float32) * std + mean).to(dtype)

        w = {"embed_tokens.weight": rnd(shape.vocab, d), "embed_positions.weight": rnd(shape.max_positions, d),
             "layer_norm.weight": rnd(d, mean=1.0), "layer_norm.bias": rnd(d)}
        for i in range(shape.layers):
            p = f"layers.{i}."
            for a in ("self_attn", "encoder_attn"):
                for n in ("q", "k", "v", "out"):
                    w[f"{p}{a}.{n}_proj.weight"] = rnd(d, d)
                    if n != "k":
                        w[f"{p}{a}.{n}_proj.bias"] = rnd(d)
            for n in ("self_attn_layer_norm", "encoder_attn_layer_norm", "final_layer_norm"):
                w[f"{p}{n}.weight"], w[f"{p}{n}.bias"] = rnd(d, mean=1.0), rnd(d)
            w[f"{p}fc1.weight"], w[f"{p}fc1.bias"] = rnd(f, d), rnd(f)
            w[f"{p}fc2.weight"], w[f"{p}fc2.bias"] = rnd(d, f), rnd(d)
        return cls(shape, w)

    def cross_kv(self, enc: torch.Tensor) -> torch.Tensor:
        """Every layer's cross-attention keys/values of encoder states enc [W, T, d] -> [L, 2, W, H, T, D]
        (reference modeling.Decoder.cross_kv, modeling.py:166-172)."""
        s = self.shape
        wn, t, _ = enc.shape
        out = torch.empty(s.layers, 2, wn, s.heads, t, s.head_dim, dtype=enc.dtype, device=enc.device)
        flat = enc.reshape(wn * t, s.d_model)
        for i, p in enumerate(self.layers):
            k = flat @ p["xk"].t()
            v = torch.addmm(p["xv"][1], flat, p["xv"][0].t())
            out[i, 0] = k.view(wn, t, s.heads, s.head_dim).transpose(1, 2)
            out[i, 1] = v.view(wn, t, s.heads, s.head_dim).transpose(1, 2)
        return out

    @staticmethod
    def _ln_bias(x: torch.Tensor, ln: tuple, bias: torch.Tensor) -> torch.Tensor:
        """LN(x) in fp32 statistics -> x's dtype, then x += bias in place (decoder_kernels.layer_norm_bias)."""
        h = F.layer_norm(x.float(), (x.shape[-1],), ln[0].float(), ln[1].float()).to(x.dtype)
        x.add_(bias)
        return h

    def step_fn(self, tokens: torch.Tensor, offset: torch.Tensor, cache: torch.Tensor, logits: torch.Tensor,
                new_kv: torch.Tensor, src: torch.Tensor, cross: torch.Tensor,
                self_attn: Callable | None = None, cross_attn: Callable | None = None) -> Callable[[], None]:
        """A closure running one decoder call of tokens [N, 1] at ``offset`` [N] against the cache
        [L, 2, N, H, C, D] through ``src`` [N, C] and the windows' cross keys/values [L, 2, W, H, T, D], writing
        logits [N, 1, V] fp32 and appending the new keys/values to the cache (``writes_cache = True``; ``new_kv``
        is not used). ``self_attn(qkv, k_cache, v_cache, offset, src)`` (which must append) and
        ``cross_attn(q, k, v)`` default to this package's kernels."""
        s = self.shape
        n, d = tokens.shape[0], s.d_model
        w = cross.shape[2]
        if tokens.shape[1] != 1:
            raise ValueError("one new token per row")
        sa = self_attn or (lambda qkv, kc, vc, off, sr: attn_plugin.self_attn_step_triton(qkv, kc, vc, off, sr,
                                                                                           write_cache=True))
        ca = cross_attn or attn_plugin.cross_attn_triton

        def run() -> None:
            x = (self.embed[tokens[:, 0]] + self.pos[offset]).contiguous()  # [N, d]
            for i, p in enumerate(self.layers):
                h = self._ln_bias(x, p["ln1"], p["out"][1])
                qkv = torch.addmm(p["qkv"][1], h, p["qkv"][0].t())
                y = sa(qkv.view(n, 1, 3 * d), cache[i, 0], cache[i, 1], offset, src)
                x.addmm_(y.view(n, d), p["out"][0].t())
                h = self._ln_bias(x, p["ln2"], p["xout"][1])
                qw = torch.addmm(p["q"][1], h, p["q"][0].t()).view(w, n // w, d)
                a = ca(qw, cross[i, 0], cross[i, 1])
                x.addmm_(a.view(n, d), p["xout"][0].t())
                h = self._ln_bias(x, p["ln3"], p["fc2"][1])
                g = F.gelu(torch.addmm(p["fc1"][1], h, p["fc1"][0].t()).float()).to(x.dtype)
                x.addmm_(g, p["fc2"][0].t())
            xf = F.layer_norm(x.float(), (d,), self.final[0].float(), self.final[1].float())
            if self._embed32 is None:
                self._embed32 = self.embed.float()
            logits.view(n, -1).copy_(xf.to(x.dtype).float() @ self._embed32.t())

        run.writes_cache = True
        run.keep = (tokens, offset, cache, logits, new_kv, src, cross)
        return run
