"""The oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py over oracle/_ref). Needs no reference tree."""
import os

import numpy as np
import pytest

import oracle_lib as O
from xpose_b200.decode import DecodeConfig

G = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_kernels.npz"))


@pytest.mark.parametrize("tag", ["a", "b"])
def test_packer_and_matvec_golden(tag):
    seed, stream, rows, cols = (int(v) for v in G[f"pack_{tag}_seed"])
    w = O.gen_normal(seed, stream, rows * cols, 0.02)
    w[:32] = 0.0
    w[64:96] = np.linspace(-7, 7, 32, dtype=np.float32)
    words, scales = O.pack(w, rows, cols)
    assert np.array_equal(words, G[f"pack_{tag}_words"])
    assert np.array_equal(scales, G[f"pack_{tag}_scales"])
    assert np.array_equal(O.mv(G[f"mv_{tag}_x"], words, scales, rows, cols), G[f"mv_{tag}_y"])


def test_norm_rope_geglu_golden():
    o = O.oracle()
    y = np.zeros(1152, np.float32)
    o.xo_rmsnorm_gemma(y, G["norm_x"], G["norm_w"], 1152, 64, 1e-6)
    assert np.array_equal(y, G["norm_y"])
    r = G["rope_x"].copy()
    o.xo_rope(r, 4, 256, 131, 1e6)
    np.testing.assert_allclose(r, G["rope_y"], rtol=0, atol=1e-5)
    h = np.zeros(512, np.float32)
    o.xo_geglu(h, G["geglu_g"], G["geglu_u"], 512)
    assert np.array_equal(h, G["geglu_h"])


def test_attention_golden():
    out = np.zeros(1024, np.float32)
    k, v = G["attn_k"], G["attn_v"]
    O.oracle().xo_attention(out, G["attn_q"], k.ctypes.data, v.ctypes.data, 0, 4, 1, 256, 131 - 64, 64, 1.0 / 16)
    assert np.array_equal(out, G["attn_out"])


def test_topk_golden():
    v, i = np.zeros(40, np.float32), np.zeros(40, np.uint32)
    x = G["topk_x"]
    assert O.oracle().xo_topk(x, len(x), 40, v, i) == 40
    assert np.array_equal(i, G["topk_i"]) and np.array_equal(v, G["topk_v"])


def test_engine_golden():
    cfg = DecodeConfig(n_layers=2, hidden=128, ffn=256, vocab=256, max_seq=32, sliding_window=8, global_every=2)
    om = O.OracleModel(cfg, seed=9, kv_fp16=False, norm_roundtrip=True)
    prompt = G["engine_prompt"]
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
    ref = G["engine_logits0"]
    assert np.linalg.norm(want - ref) / np.linalg.norm(ref) < 1e-5
    pos = len(prompt)
    for t in G["engine_tokens"]:
        assert int(np.argmax(want)) == int(t)
        want = om.forward(int(t), pos)
        pos += 1
    ref = G["engine_logits1"]
    assert np.linalg.norm(want - ref) / np.linalg.norm(ref) < 1e-5
