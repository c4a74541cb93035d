"""GGUF v3 files for the NedoLM decoder: a writer for synthetic models and a
reader that maps a file and returns its metadata and tensor views.

The layout follows the reference loader (src/gguf.cpp:78-104): magic
0x46554747, version, tensor count, metadata count, the metadata key/value
records, one info record per tensor (name, rank, shape with the contiguous
dimension first, type, offset relative to the data section), then the data
section at the next multiple of general.alignment (default 32).

`synthetic_model` builds the tensor set NedoModel::load_schema looks for
(src/model.cpp:75-118) with the nedolm.* configuration keys and a surface
tokenizer vocabulary (tokenizer.ggml.tokens, at least the 259 fixed ids of
src/tokenizer.cpp:10-14).
"""
import mmap
import struct

import numpy as np

from . import blocks as B

MAGIC = 0x46554747
# metadata value types (include/nedo/gguf.hpp:12-15)
UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64, FLOAT64 = range(13)
_SCALAR = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i", FLOAT32: "<f", BOOL: "<B",
           UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}
F32, F16, Q4_0, Q8_0 = 0, 1, 2, 8


def tensor_nbytes(ttype, n):
    if ttype == F32:
        return 4 * n
    if ttype == F16:
        return 2 * n
    if ttype in (Q4_0, Q8_0):
        if n % 32:
            raise ValueError("block type elements not block aligned")
        return (n // 32) * (18 if ttype == Q4_0 else 34)
    raise ValueError(f"tensor type {ttype} not supported here")


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype, v):
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        out = struct.pack("<IQ", etype, len(items))
        return out + b"".join(_value(etype, it) for it in items)
    return struct.pack(_SCALAR[vtype], v)


def write_gguf(path, metadata, tensors, alignment=32):
    """metadata: {key: (type, value)} (ARRAY values are (element type, list));
    tensors: [(name, tensor type, shape with the contiguous dimension first, bytes)]."""
    head = struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(metadata))
    for k, (vt, v) in metadata.items():
        head += _str(k) + struct.pack("<I", vt) + _value(vt, v)
    offsets, off = [], 0
    for name, tt, shape, data in tensors:
        n = int(np.prod(shape))
        if len(data) != tensor_nbytes(tt, n):
            raise ValueError(f"{name}: {len(data)} bytes for {n} elements of type {tt}")
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        head += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", tt, off)
        off += len(data)
    data_start = (len(head) + alignment - 1) // alignment * alignment
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_start - len(head)))
        pos = 0
        for (name, tt, shape, data), o in zip(tensors, offsets):
            f.write(b"\0" * (o - pos))
            f.write(bytes(data))
            pos = o + len(data)


class GgufFile:
    """A mapped GGUF file: .metadata {key: value}, .tensors {name: (type, shape, offset, nbytes)},
    .view(name) -> numpy uint8 view of the tensor's bytes (no copy)."""

    def __init__(self, path):
        self._f = open(path, "rb")
        self._m = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = np.frombuffer(self._m, dtype=np.uint8)
        p = 0

        def rd(fmt):
            nonlocal p
            v = struct.unpack_from(fmt, self._m, p)
            p += struct.calcsize(fmt)
            return v[0]

        def rstr():
            nonlocal p
            n = rd("<Q")
            s = bytes(self._m[p:p + n]).decode()
            p += n
            return s

        def rval(vt):
            if vt == STRING:
                return rstr()
            if vt == ARRAY:
                et, n = rd("<I"), rd("<Q")
                return [rval(et) for _ in range(n)]
            return rd(_SCALAR[vt])

        if rd("<I") != MAGIC:
            raise ValueError("not a GGUF file (bad magic)")
        self.version = rd("<I")
        if self.version not in (2, 3):
            raise ValueError("unsupported GGUF version")
        nt, nkv = rd("<Q"), rd("<Q")
        self.metadata = {}
        for _ in range(nkv):
            k = rstr()
            self.metadata[k] = rval(rd("<I"))
        align = int(self.metadata.get("general.alignment", 32))
        infos = []
        for _ in range(nt):
            name = rstr()
            nd = rd("<I")
            shape = [rd("<Q") for _ in range(nd)]
            tt, off = rd("<I"), rd("<Q")
            infos.append((name, tt, shape, off))
        data = (p + align - 1) // align * align
        self.tensors = {}
        for name, tt, shape, off in infos:
            nb = tensor_nbytes(tt, int(np.prod(shape)))
            if data + off + nb > len(self.buf):
                raise ValueError(f"tensor outside GGUF file: {name}")
            self.tensors[name] = (tt, shape, data + off, nb)

    def view(self, name):
        tt, shape, off, nb = self.tensors[name]
        return self.buf[off:off + nb]

    def close(self):
        self.buf = None
        self._m.close()
        self._f.close()


def synthetic_model(path, dim=256, layers=2, heads=4, kv_heads=2, ffn=512, vocab=512, context=64, sliding=16,
                    wtype=Q8_0, emb_type=Q8_0, head_type=F16, norm_type=F32, tied=False, seed=1, rope_theta=10000.0,
                    rms_eps=1e-5, morph=None, shared_layers=False):
    """A NedoLM GGUF with seeded random weights.  Projection weights as the matvec
    configurations draw them (blocks.gen_weight), norm weights
    1 + N(0, 0.1).  morph = (layers, shared, root, suffix) adds the MorphFFN
    routing table blk.0.ffn_gate_tid2eid.weight [2, vocab] F32 of 0/1 flags.
    shared_layers: every layer gets layer 0's bytes (fast to build; still one
    tensor per layer in the file)."""
    if vocab < 259:
        raise ValueError("the surface tokenizer needs at least 259 ids")
    hd = dim // heads
    rng = np.random.default_rng(seed)
    tokens = ["<pad>", "<s>", "</s>"] + [f"<0x{i:02X}>" for i in range(256)]
    tokens += [f"w{i}" for i in range(vocab - len(tokens))]
    md = {
        "general.architecture": (STRING, "nedolm"),
        "general.alignment": (UINT32, 32),
        "nedolm.vocab_size": (UINT32, vocab),
        "nedolm.embedding_length": (UINT32, dim),
        "nedolm.block_count": (UINT32, layers),
        "nedolm.attention.head_count": (UINT32, heads),
        "nedolm.attention.head_count_kv": (UINT32, kv_heads),
        "nedolm.rope.dimension_count": (UINT32, hd),
        "nedolm.feed_forward_length": (UINT32, ffn),
        "nedolm.context_length": (UINT32, context),
        "nedolm.attention.sliding_window": (UINT32, sliding),
        "nedolm.attention.layer_norm_rms_epsilon": (FLOAT32, rms_eps),
        "nedolm.rope.freq_base": (FLOAT32, rope_theta),
        "tokenizer.ggml.tokens": (ARRAY, (STRING, tokens)),
        "tokenizer.ggml.bos_token_id": (UINT32, 1),
        "tokenizer.ggml.eos_token_id": (UINT32, 2),
    }
    if morph is not None:
        ml, ms, mr, mz = morph
        md["nedolm.morph.layer_count"] = (UINT32, ml)
        md["nedolm.morph.shared_width"] = (UINT32, ms)
        md["nedolm.morph.root_width"] = (UINT32, mr)
        md["nedolm.morph.suffix_width"] = (UINT32, mz)

    def norm(n, s):
        r = np.random.default_rng(s)
        v = (1.0 + 0.1 * r.standard_normal(n)).astype(np.float32)
        return (v if norm_type == F32 else v.astype(np.float16)).view(np.uint8).reshape(-1)

    memo = {}

    def _weight(ttype, rows, cols, sd):
        key = (ttype, rows, cols, sd)
        if key not in memo:
            memo[key] = B.gen_weight(ttype, rows, cols, sd).reshape(-1)
        return memo[key]

    t = []
    s = seed * 1000
    t.append(("token_embd.weight", emb_type, [dim, vocab], _weight(emb_type, vocab, dim, s + 1)))
    t.append(("output_norm.weight", norm_type, [dim], norm(dim, s + 2)))
    if not tied:
        t.append(("output.weight", head_type, [dim, vocab], _weight(head_type, vocab, dim, s + 3)))
    if morph is not None:
        flags = (rng.random((vocab, 2)) < 0.5).astype(np.float32)
        t.append(("blk.0.ffn_gate_tid2eid.weight", F32, [2, vocab], flags.view(np.uint8).reshape(-1)))
    kvd = kv_heads * hd
    for i in range(layers):
        b = s + 100 * (1 if shared_layers else i + 1)
        t.append((f"blk.{i}.attn_norm.weight", norm_type, [dim], norm(dim, b)))
        t.append((f"blk.{i}.attn_q.weight", wtype, [dim, dim], _weight(wtype, dim, dim, b + 1)))
        t.append((f"blk.{i}.attn_k.weight", wtype, [dim, kvd], _weight(wtype, kvd, dim, b + 2)))
        t.append((f"blk.{i}.attn_v.weight", wtype, [dim, kvd], _weight(wtype, kvd, dim, b + 3)))
        t.append((f"blk.{i}.attn_output.weight", wtype, [dim, dim], _weight(wtype, dim, dim, b + 4)))
        t.append((f"blk.{i}.ffn_norm.weight", norm_type, [dim], norm(dim, b + 5)))
        t.append((f"blk.{i}.ffn_gate.weight", wtype, [dim, ffn], _weight(wtype, ffn, dim, b + 6)))
        t.append((f"blk.{i}.ffn_up.weight", wtype, [dim, ffn], _weight(wtype, ffn, dim, b + 7)))
        t.append((f"blk.{i}.ffn_down.weight", wtype, [ffn, dim], _weight(wtype, dim, ffn, b + 8)))
    write_gguf(path, md, t)
