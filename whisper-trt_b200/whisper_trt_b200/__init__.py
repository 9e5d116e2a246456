"""whisper_trt_b200 -- the Whisper decoder's per-step attention on B200 (sm_100a).

A drop-in for the attention path of whisper-trt (``src/whisper_trt/attn_plugin.py`` launchers and the slot-table
bookkeeping of ``search.py`` / ``beam_kernels.py``) on hand-written CUDA kernels behind a C ABI
(``include/whisper_attn_b200.h``, ``libwhisper_attn_b200.so``):

* :mod:`whisper_trt_b200.attn_plugin` -- self-attention step with cache append, split / combined cross-attention,
  prompt self-attention, the vocabulary projection;
* :mod:`whisper_trt_b200.slots` -- beam scoring, reorder, fused beam update, slot reset;
* :mod:`whisper_trt_b200.decoder_kernels` -- the step's linear layers with LayerNorm / bias / GELU / residual fused;
* :mod:`whisper_trt_b200.build` -- builds the library in-tree for sm_100a.

Each of the three modules has an ``install(module)`` that routes the matching reference module
(``whisper_trt.attn_plugin``, ``whisper_trt.beam_kernels``, ``whisper_trt.decoder_kernels``) to these kernels in
place, so the reference's own ``TritonDecoderBackend`` and ``Search`` run on them unchanged.
"""

from . import _lib  # noqa: F401

__all__ = ["attn_plugin", "slots", "decoder_kernels", "build"]
