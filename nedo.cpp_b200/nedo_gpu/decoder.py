"""The device-resident NedoLM decode forward pass (nedo_gpu_decoder_* in
include/nedo_gpu.h) built from a GGUF file.

`Decoder.from_gguf` reads the configuration with the keys and defaults of
NedoModel::load_schema (src/model.cpp:75-93) and hands the tensors to the
library in its fixed order (token_embd, output_norm, output or tied,
MorphFFN routing table, then nine per layer).  `forward(token, pos)` is one
pass of the reference's `forward` step (src/model.cpp:212-260); `greedy`
is generate_ids with temperature 0 and no BOS insertion
(src/model.cpp:151-281)."""
from __future__ import annotations

import ctypes

import numpy as np

from . import DecoderConfig, Library, NedoGpuError, TensorView, load

_LAYER = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")
_ALIASES = {  # the reference's alternative names (src/model.cpp:94-116)
    "token_embd.weight": ("tok_embeddings.weight", "model.embed_tokens.weight"),
    "output_norm.weight": ("norm.weight",),
    "output.weight": ("lm_head.weight",),
}


def _u(md, keys, default=0):
    for k in keys:
        if k in md:
            return int(md[k])
    return default


def _f(md, keys, default):
    for k in keys:
        if k in md:
            return float(md[k])
    return default


def config_from_gguf(g) -> DecoderConfig:
    md = g.metadata
    c = DecoderConfig()
    tokens = md.get("tokenizer.ggml.tokens", [])
    c.vocab = _u(md, ["nedolm.vocab_size"], len(tokens))
    c.dim = _u(md, ["nedolm.embedding_length", "llama.embedding_length"], 1536)
    c.layers = _u(md, ["nedolm.block_count", "llama.block_count"], 24)
    c.heads = _u(md, ["nedolm.attention.head_count", "llama.attention.head_count"], 12)
    c.kv_heads = _u(md, ["nedolm.attention.head_count_kv", "llama.attention.head_count_kv"], 4)
    c.head_dim = _u(md, ["nedolm.rope.dimension_count"], c.dim // c.heads if c.heads else 0)
    c.ffn = _u(md, ["nedolm.feed_forward_length", "llama.feed_forward_length"], 5632)
    c.context = _u(md, ["nedolm.context_length", "llama.context_length"], 4096)
    c.sliding = _u(md, ["nedolm.attention.sliding_window", "nedolm.sliding_window"], 2048)
    c.morph_layers = _u(md, ["nedolm.morph.layer_count"])
    c.morph_shared = _u(md, ["nedolm.morph.shared_width"])
    c.morph_root = _u(md, ["nedolm.morph.root_width"])
    c.morph_suffix = _u(md, ["nedolm.morph.suffix_width"])
    c.rms_eps = _f(md, ["nedolm.attention.layer_norm_rms_epsilon", "llama.attention.layer_norm_rms_epsilon"], 1e-5)
    c.rope_theta = _f(md, ["nedolm.rope.freq_base", "llama.rope.freq_base"], 10000.0)
    return c


class Decoder:
    """One device-resident model; the KV cache belongs to the sequence being decoded."""

    def __init__(self, lib: Library, cfg: DecoderConfig, views, keepalive=None):
        self.lib = lib
        self.cfg = cfg
        self._keep = keepalive
        arr = (TensorView * len(views))(*views)
        h = ctypes.c_void_p()
        lib._check(lib.lib.nedo_gpu_decoder_create(ctypes.byref(cfg), arr, len(views), ctypes.byref(h)))
        self.h = h
        self.vocab = int(views[2].shape[1] if views[2].data else views[0].shape[1])

    @classmethod
    def from_gguf(cls, g, lib: Library | None = None) -> "Decoder":
        lib = lib or load()
        cfg = config_from_gguf(g)

        def find(name):
            for n in (name,) + _ALIASES.get(name, ()):
                if n in g.tensors:
                    return n
            return None

        def view(name):
            v = TensorView()
            if name is None:
                return v
            tt, shape, off, nb = g.tensors[name]
            v.type = tt
            v.ndims = len(shape)
            for i, d in enumerate(shape[:2]):
                v.shape[i] = d
            v.data = g.buf[off:off + nb].ctypes.data if nb else None
            v.nbytes = nb
            return v

        names = [find("token_embd.weight"), find("output_norm.weight"), find("output.weight"),
                 "blk.0.ffn_gate_tid2eid.weight" if "blk.0.ffn_gate_tid2eid.weight" in g.tensors else None]
        for i in range(cfg.layers):
            names += [f"blk.{i}.{k}.weight" if f"blk.{i}.{k}.weight" in g.tensors else None for k in _LAYER]
        return cls(lib, cfg, [view(n) for n in names], keepalive=g)

    def forward(self, token: int, pos: int, logits: bool = True):
        """(greedy id, logits or None) of one pass for `token` at `pos`."""
        out = np.empty(self.vocab, np.float32) if logits else None
        idx = ctypes.c_uint32()
        self.lib._check(self.lib.lib.nedo_gpu_decoder_forward(self.h, token, pos,
                                                              out.ctypes.data if logits else None,
                                                              ctypes.byref(idx)))
        return int(idx.value), out

    def generate(self, token: int, pos: int, n: int) -> list:
        """n greedy passes with the loop on the device (nedo_gpu_decoder_generate):
        the picks of passes pos .. pos + n - 1, the first fed `token`."""
        ids = np.empty(max(n, 1), np.uint32)
        self.lib._check(self.lib.lib.nedo_gpu_decoder_generate(self.h, token, pos, n, ids.ctypes.data))
        return [int(v) for v in ids[:n]]

    def set_stream(self, stream: int) -> None:
        """Run the passes on a caller's CUDA stream (0 = the decoder's own)."""
        self.lib._check(self.lib.lib.nedo_gpu_decoder_set_stream(self.h, stream or None))

    def logits_dev(self) -> int:
        p = ctypes.c_void_p()
        self.lib._check(self.lib.lib.nedo_gpu_decoder_logits_dev(self.h, ctypes.byref(p)))
        return int(p.value)

    def reset(self) -> None:
        self.lib._check(self.lib.lib.nedo_gpu_decoder_reset(self.h))

    def greedy(self, prompt, max_new, eos=2, logits=True):
        """(logits of every pass or None, generated ids) as generate_ids with
        temperature 0 (src/model.cpp:262-281)."""
        rows, pos, last = [], 0, None
        for t in prompt:
            last, lg = self.forward(t, pos, logits)
            rows.append(lg)
            pos += 1
        out = []
        for _ in range(max_new):
            if pos >= self.cfg.context:
                break
            if last == eos:
                break
            out.append(last)
            last, lg = self.forward(out[-1], pos, logits)
            rows.append(lg)
            pos += 1
        return (np.stack(rows) if logits else None), out

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.lib.nedo_gpu_decoder_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


__all__ = ["Decoder", "config_from_gguf", "NedoGpuError"]
