"""Regenerate tests/golden/decode_golden.npz from the reference itself.

For each synthetic NedoLM model below, writes the GGUF with
nedo_gpu.gguf.synthetic_model (seeded, so any machine rebuilds the same bytes),
runs the reference's own decode loop on it (oracle/_ref/ref_decode: the
reference's src/model.cpp generate_ids with greedy sampling, compiled from the
reference sources by oracle/Makefile) and stores the LM-head logits of every
forward pass and the generated ids.  The models cover Q8_0, Q4_0 and F16
weights, F32 and F16 norms, a tied head, grouped-query and plain multi-head
attention, a sliding window shorter than the sequence (the cache ring wraps)
and the MorphFFN gate masking.

Usage:  make -C oracle ref && python tests/golden/make_decode_golden.py
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "nedo.cpp_b200"))
from nedo_gpu import gguf as G  # noqa: E402

REF_DECODE = os.path.join(ROOT, "oracle", "_ref", "ref_decode")

# name -> (synthetic_model keyword arguments, prompt ids, new tokens)
MODELS = {
    "q8_gqa_window": (dict(dim=256, layers=2, heads=4, kv_heads=2, ffn=512, vocab=512, context=64, sliding=16,
                           wtype=G.Q8_0, emb_type=G.Q8_0, head_type=G.F16, norm_type=G.F32, seed=11),
                      [5, 300, 301, 302], 24),
    "q4_tied_f16norm": (dict(dim=512, layers=2, heads=8, kv_heads=4, ffn=1024, vocab=640, context=48, sliding=0,
                             wtype=G.Q4_0, emb_type=G.Q4_0, norm_type=G.F16, tied=True, seed=12),
                        [7, 400, 9], 20),
    "f16_mha_morph": (dict(dim=256, layers=3, heads=8, kv_heads=8, ffn=512, vocab=512, context=40, sliding=32,
                           wtype=G.F16, emb_type=G.F16, head_type=G.Q8_0, norm_type=G.F32, seed=13,
                           morph=(2, 256, 128, 128)),
                      [1, 260, 261, 262, 263], 16),
}


def read_ref_out(path):
    b = open(path, "rb").read()
    a = np.frombuffer(b, dtype=np.uint32)
    steps, vocab = int(a[0]), int(a[1])
    logits = np.frombuffer(b, dtype=np.float32, count=steps * vocab, offset=8).reshape(steps, vocab).copy()
    n = int(a[2 + steps * vocab])
    ids = a[3 + steps * vocab:3 + steps * vocab + n].astype(np.int64)
    return logits, ids


def run_reference(gguf_path, prompt, max_new):
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "out.bin")
        subprocess.run([REF_DECODE, gguf_path, out, str(max_new), "0", "0", "0", "0"] + [str(t) for t in prompt],
                       check=True)
        return read_ref_out(out)


def main():
    if not os.path.exists(REF_DECODE):
        sys.exit("build the reference decode loop first: make -C oracle ref")
    arrays, meta = {}, {}
    with tempfile.TemporaryDirectory() as d:
        for name, (kw, prompt, max_new) in MODELS.items():
            path = os.path.join(d, name + ".gguf")
            G.synthetic_model(path, **kw)
            logits, ids = run_reference(path, prompt, max_new)
            arrays[name + "/logits"] = logits
            arrays[name + "/ids"] = ids
            meta[name] = {"prompt": prompt, "max_new": max_new}
            print(name, logits.shape, list(ids))
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(ROOT, "tests", "golden", "decode_golden.npz"), **arrays)


if __name__ == "__main__":
    main()
