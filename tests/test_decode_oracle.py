"""The decode-forward oracle (oracle/decode_oracle.py) pinned against the
reference's own decode loop (src/model.cpp:151-281): the LM-head logits of
every forward pass and the greedy ids in tests/golden/decode_golden.npz, made
by tests/golden/make_decode_golden.py from oracle/_ref/ref_decode.  Also the
GGUF writer/reader round trip the synthetic models rely on."""
import json
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

from conftest import ROOT

sys.path[:0] = [os.path.join(ROOT, "tests", "golden")]
import decode_oracle as DO  # noqa: E402
import make_decode_golden as M  # noqa: E402
from nedo_gpu import gguf as G  # noqa: E402

GOLDEN = np.load(os.path.join(ROOT, "tests", "golden", "decode_golden.npz"))
# the restatement differs from the reference only by the last bits of powf /
# cosf / sinf / expf and FMA contraction: 3.4e-7 of the largest logit measured
REL_TOL = 2e-6


def test_gguf_round_trip(tmp_path):
    p = str(tmp_path / "m.gguf")
    md = {"general.architecture": (G.STRING, "nedolm"), "a.u32": (G.UINT32, 7), "a.f": (G.FLOAT32, 0.5),
          "a.list": (G.ARRAY, (G.STRING, ["x", "yz"])), "general.alignment": (G.UINT32, 64)}
    w = np.arange(64 * 3, dtype=np.float32).view(np.uint8)
    h = np.arange(40, dtype=np.float16).view(np.uint8)
    G.write_gguf(p, md, [("w", G.F32, [64, 3], w), ("h", G.F16, [40], h)], alignment=64)
    g = G.GgufFile(p)
    assert g.version == 3 and g.metadata["a.u32"] == 7 and g.metadata["a.list"] == ["x", "yz"]
    assert abs(g.metadata["a.f"] - 0.5) < 1e-7
    assert g.tensors["w"][0] == G.F32 and g.tensors["w"][1] == [64, 3] and g.tensors["w"][2] % 64 == 0
    assert np.array_equal(g.view("w"), w) and np.array_equal(g.view("h"), h)
    g.close()
    with open(p, "r+b") as f:
        f.write(b"XXXX")
    with pytest.raises(ValueError):
        G.GgufFile(p)


@pytest.mark.parametrize("name", list(M.MODELS))
def test_decode_oracle_matches_reference_logits(name, tmp_path):
    kw, prompt, max_new = M.MODELS[name]
    meta = json.loads(bytes(GOLDEN["meta"]).decode())[name]
    assert meta["prompt"] == prompt and meta["max_new"] == max_new
    p = str(tmp_path / (name + ".gguf"))
    G.synthetic_model(p, **kw)
    g = G.GgufFile(p)
    logits, ids = DO.DecodeOracle(g).greedy(prompt, max_new)
    g.close()
    ref = GOLDEN[name + "/logits"]
    assert logits.shape == ref.shape
    rel = np.abs(logits - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert rel.max() <= REL_TOL, rel
    assert list(ids) == list(GOLDEN[name + "/ids"])


REF_DECODE = os.path.join(ROOT, "oracle", "_ref", "ref_decode")


@pytest.mark.skipif(not os.path.exists(REF_DECODE), reason="reference decode loop not built (make -C oracle ref)")
def test_golden_is_what_the_reference_produces(tmp_path):
    name = "q8_gqa_window"
    kw, prompt, max_new = M.MODELS[name]
    p = str(tmp_path / "m.gguf")
    G.synthetic_model(p, **kw)
    logits, ids = M.run_reference(p, prompt, max_new)
    assert np.array_equal(logits.view(np.uint32), GOLDEN[name + "/logits"].view(np.uint32))
    assert list(ids) == list(GOLDEN[name + "/ids"])
