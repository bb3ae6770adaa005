"""Regenerates tests/golden/*.npz from the reference build in oracle/_ref
(the reference's own kernels and engine compiled from source). Run here,
where the reference tree exists:

    make -C oracle && python tests/golden/make_golden.py

The fixtures let tests/test_golden.py pin the oracle on machines without the
reference tree."""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle_lib as O  # noqa: E402
from xpose_b200.decode import DecodeConfig  # noqa: E402


def main():
    assert O.ref() is not None, "build oracle/_ref first (make -C oracle)"
    rng = np.random.default_rng(20260719)
    out = {}
    # packer + matvec at two shapes (small enough to commit)
    for tag, rows, cols in (("a", 256, 128), ("b", 1152, 64)):
        w = O.gen_normal(11, 1, rows * cols, 0.02)
        w[:32] = 0.0
        w[64:96] = np.linspace(-7, 7, 32, dtype=np.float32)
        words, scales = O.pack(w, rows, cols, impl="ref")
        x = rng.uniform(-1, 1, rows).astype(np.float32)
        y = np.zeros(cols, np.float32)
        O.ref_launch("mv_km4_bs", cols, y, x, words, scales, rows, cols)
        out.update({f"pack_{tag}_seed": np.array([11, 1, rows, cols]), f"pack_{tag}_words": words,
                    f"pack_{tag}_scales": scales, f"mv_{tag}_x": x, f"mv_{tag}_y": y})
    # norms, rope, geglu
    x = rng.uniform(-1.5, 1.5, 1152).astype(np.float32)
    w = rng.uniform(-0.1, 0.1, 1152).astype(np.float32)
    part, y = np.zeros(64, np.float32), np.zeros(1152, np.float32)
    O.ref_launch("rmsnorm_sumsq", 64, part, x, 1152, 64)
    O.ref_launch("rmsnorm_apply_gemma", 1152, y, x, w, part, 1152, 64, 1e-6)
    out.update({"norm_x": x, "norm_w": w, "norm_y": y})
    q = rng.uniform(-1.5, 1.5, 1024).astype(np.float32)
    r = q.copy()
    O.ref_launch("rope", 512, r, 4, 256, 131, 1e6)
    out.update({"rope_x": q, "rope_y": r})
    g = rng.uniform(-12, 12, 512).astype(np.float32)
    u = rng.uniform(-1.5, 1.5, 512).astype(np.float32)
    h = np.zeros(512, np.float32)
    O.ref_launch("geglu", 512, h, g, u, 512)
    out.update({"geglu_g": g, "geglu_u": u, "geglu_h": h})
    # serial attention, kSeqLen 131 with a 64-wide window
    seq, kvs = 131, 131 - 64
    aq = rng.uniform(-1.5, 1.5, 1024).astype(np.float32)
    kc = rng.uniform(-1.5, 1.5, seq * 256).astype(np.float32)
    vc = rng.uniform(-1.5, 1.5, seq * 256).astype(np.float32)
    sc = np.zeros(4 * 64, np.float32)
    ao = np.zeros(1024, np.float32)
    O.ref_launch("attention_scores", 4 * 64, sc, aq, kc, 4, 1, 256, 64, 1.0 / 16, kvs)
    O.ref_launch("softmax_rows", 4, sc, 4, 64)
    O.ref_launch("attention_apply", 1024, ao, sc, vc, 4, 1, 256, 64, kvs)
    out.update({"attn_q": aq, "attn_k": kc, "attn_v": vc, "attn_out": ao})
    # top-k over a planted duplicate (sampling_test.cpp:428-481)
    n = 16384
    t = rng.uniform(-3, 3, n).astype(np.float32)
    t[1234] = t[9999] = 3.25
    cv, ci = np.zeros(64 * 40, np.float32), np.zeros(64 * 40, np.uint32)
    ov, oi = np.zeros(40, np.float32), np.zeros(40, np.uint32)
    O.ref_launch("topk_partial", 64, cv, ci, t, n, 64, 40)
    O.ref_launch("topk_rank_select", 64 * 40, ov, oi, cv, ci, 64 * 40, 40)
    out.update({"topk_x": t, "topk_v": ov, "topk_i": oi})
    # the reference engine on a tiny random-init model: logits after a prompt
    cfg = DecodeConfig(n_layers=2, hidden=128, ffn=256, vocab=256, max_seq=32, sliding_window=8, global_every=2)
    om = O.OracleModel(cfg, seed=9, kv_fp16=False, norm_roundtrip=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        O.write_model_gguf(om, path, window=cfg.sliding_window)
        rs = O.RefSession(path, cfg.max_seq, cfg.global_every)
        prompt = O.gen_tokens(9, 3, 12, cfg.vocab)
        rs.prefill(prompt)
        l0 = rs.logits(cfg.vocab)
        toks = [rs.decode_step() for _ in range(4)]
        l1 = rs.logits(cfg.vocab)
        rs.close()
    out.update({"engine_prompt": prompt, "engine_logits0": l0, "engine_tokens": np.array(toks, np.uint32),
                "engine_logits1": l1})
    np.savez_compressed(os.path.join(HERE, "reference_kernels.npz"), **out)
    print("wrote", os.path.join(HERE, "reference_kernels.npz"))


if __name__ == "__main__":
    main()
