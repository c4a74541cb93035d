"""Test infrastructure (the oracle): a CPU restatement of the reference's decode
forward pass, NedoModel::generate_ids' `forward` (src/model.cpp:212-260), with
its elementwise kernels (src/kernels.cpp:43-106).  Matvecs and embedding rows
go through the C restatement (nedo_oracle.c, bit-exact with the reference's
kernels); the O(d) steps are restated here in numpy float32 in the reference's
order of operations, with the double accumulations where the reference has
them (RMSNorm's sum of squares, the attention score dots).  Transcendentals
(powf, cosf, sinf, expf) and the compiler's FMA contraction in the reference
build may differ in the last bits, so this restatement agrees with the
reference's logits to a tolerance, not bit for bit; it is pinned against the
logits the reference itself produced (tests/golden/decode_golden.npz, made by
tests/golden/make_decode_golden.py).  Only tests/ and bench.py's CPU legs use
this module.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import oracle as O  # noqa: E402

_F32, _F16 = 0, 1


def _norm_weight(g, name):
    tt, shape, off, nb = g.tensors[name]
    v = g.view(name)
    if tt == _F32:
        return v.view(np.float32).copy()
    if tt == _F16:
        return v.view(np.float16).astype(np.float32)
    raise ValueError(f"unsupported RMSNorm tensor type: {name}")


def rms_norm(x, w, eps):
    # src/kernels.cpp:50-72: ss in double (sequential), inv in float, y = x * inv * w
    x64 = x.astype(np.float64)
    ss = np.cumsum(x64 * x64)[-1] if x.size else 0.0
    inv = np.float32(1.0) / np.sqrt(np.float32(np.float32(ss / x.size) + np.float32(eps)))
    return (x * inv * w).astype(np.float32)


def rope(v, nh, hd, pos, theta):
    # src/kernels.cpp:93-105
    half = hd // 2
    i = np.arange(half, dtype=np.float32)
    freq = np.power(np.float32(theta), np.float32(-2.0) * i / np.float32(hd)).astype(np.float32)
    a = (np.float32(pos) * freq).astype(np.float32)
    c, s = np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)
    v = v.reshape(nh, hd).copy()
    x, y = v[:, :half].copy(), v[:, half:].copy()
    v[:, :half] = x * c - y * s
    v[:, half:] = x * s + y * c
    return v.reshape(-1)


def softmax(x):
    # src/kernels.cpp:92: max, exp(x - m), float sum in order, multiply by 1/s
    m = x.max()
    e = np.exp((x - m).astype(np.float32)).astype(np.float32)
    s = np.float32(0.0)
    for v in e:
        s = np.float32(s + v)
    return (e * (np.float32(1.0) / s)).astype(np.float32)


class DecodeOracle:
    """Greedy or logits-only decoding of a NedoLM GGUF (nedo_gpu.gguf.GgufFile)."""

    def __init__(self, g, orc=None):
        self.g = g
        self.o = orc or O.Oracle()
        md = g.metadata
        self.vocab = int(md.get("nedolm.vocab_size", len(md["tokenizer.ggml.tokens"])))
        self.dim = int(md["nedolm.embedding_length"])
        self.layers = int(md["nedolm.block_count"])
        self.heads = int(md["nedolm.attention.head_count"])
        self.kv_heads = int(md["nedolm.attention.head_count_kv"])
        self.hd = int(md.get("nedolm.rope.dimension_count", self.dim // self.heads))
        self.ffn = int(md["nedolm.feed_forward_length"])
        self.context = int(md["nedolm.context_length"])
        sl = int(md.get("nedolm.attention.sliding_window", 2048))
        self.window = max(1, min(sl if sl else self.context, self.context))
        self.eps = float(md.get("nedolm.attention.layer_norm_rms_epsilon", 1e-5))
        self.theta = float(md.get("nedolm.rope.freq_base", 10000.0))
        self.morph = [int(md.get(k, 0)) for k in ("nedolm.morph.layer_count", "nedolm.morph.shared_width",
                                                  "nedolm.morph.root_width", "nedolm.morph.suffix_width")]
        self.route = (g.view("blk.0.ffn_gate_tid2eid.weight").view(np.float32)
                      if "blk.0.ffn_gate_tid2eid.weight" in g.tensors else None)
        self.head = "output.weight" if "output.weight" in g.tensors else "token_embd.weight"
        self.eos = int(md.get("tokenizer.ggml.eos_token_id", 2))
        kvd = self.kv_heads * self.hd
        self.kc = np.zeros((self.layers, self.window, kvd), np.float32)
        self.vc = np.zeros((self.layers, self.window, kvd), np.float32)

    def _mv(self, name, x):
        tt, shape, off, nb = self.g.tensors[name]
        return self.o.matvec(tt, shape[1], shape[0], self.g.view(name), np.ascontiguousarray(x, np.float32))

    def forward(self, token, pos):
        g, D, H, KH, HD = self.g, self.dim, self.heads, self.kv_heads, self.hd
        tt, shape, off, nb = g.tensors["token_embd.weight"]
        x = self.o.embedding_row(tt, shape[1], shape[0], g.view("token_embd.weight"), token)
        inv_sqrt = np.float32(1.0) / np.sqrt(np.float32(HD))
        qpk = H // KH
        W = self.window
        for li in range(self.layers):
            p = f"blk.{li}."
            xn = rms_norm(x, _norm_weight(g, p + "attn_norm.weight"), self.eps)
            q = self._mv(p + "attn_q.weight", xn)
            k = self._mv(p + "attn_k.weight", xn)
            v = self._mv(p + "attn_v.weight", xn)
            q = rope(q, H, HD, pos, self.theta)
            k = rope(k, KH, HD, pos, self.theta)
            slot = pos % W
            self.kc[li, slot] = k
            self.vc[li, slot] = v
            start = pos + 1 - W if pos + 1 > W else 0
            slots = [(start + j) % W for j in range(pos - start + 1)]
            att = np.zeros(H * HD, np.float32)
            for h in range(H):
                kh = h // qpk
                qh = q[h * HD:(h + 1) * HD].astype(np.float64)
                keys = self.kc[li, slots, kh * HD:(kh + 1) * HD].astype(np.float64)
                sc = ((keys @ qh).astype(np.float32) * inv_sqrt).astype(np.float32)
                a = softmax(sc)
                acc = np.zeros(HD, np.float32)
                for j, sl in enumerate(slots):
                    acc = (acc + a[j] * self.vc[li, sl, kh * HD:(kh + 1) * HD]).astype(np.float32)
                att[h * HD:(h + 1) * HD] = acc
            x = (x + self._mv(p + "attn_output.weight", att)).astype(np.float32)
            xn = rms_norm(x, _norm_weight(g, p + "ffn_norm.weight"), self.eps)
            gate = self._mv(p + "ffn_gate.weight", xn)
            up = self._mv(p + "ffn_up.weight", xn)
            gate = ((gate / (np.float32(1.0) + np.exp(-gate))) * up).astype(np.float32)
            ml, ms, mr, mz = self.morph
            if self.route is not None and li >= self.layers - ml:
                root, suffix = self.route[2 * token], self.route[2 * token + 1]
                if root < 0.5:
                    gate[ms:ms + mr] = 0.0
                if suffix < 0.5:
                    gate[ms + mr:ms + mr + mz] = 0.0
            x = (x + self._mv(p + "ffn_down.weight", gate)).astype(np.float32)
        xn = rms_norm(x, _norm_weight(g, "output_norm.weight"), self.eps)
        return self._mv(self.head, xn)

    def greedy(self, prompt, max_new):
        """(logits of every forward pass, generated ids), as generate_ids with
        temperature 0 and no BOS insertion (src/model.cpp:151-281)."""
        logits, pos = [], 0
        for t in prompt:
            logits.append(self.forward(t, pos))
            pos += 1
        out = []
        for _ in range(max_new):
            if pos >= self.context:
                break
            nxt = int(self.o.argmax(logits[-1]))
            if nxt == self.eos:
                break
            out.append(nxt)
            logits.append(self.forward(nxt, pos))
            pos += 1
        return np.stack(logits), out
