"""The drop-in, end to end: the reference's OWN engine (examples/llm/decode.cpp:
DecodeSession, record_token, its Batch/Fence use and its kernel lookups by
module and name) compiled against include/xp/vulkore/vulkore.hpp and linked
to libxp_cuda.so (oracle/Makefile target ref_gpu), so every one of its
dispatches runs a B200 kernel of this library. Its logits and greedy tokens
must match the oracle's record_token with fp32 KV, which is the reference's
own cache format on this path."""
import os
import tempfile

import numpy as np
import pytest

import oracle_lib as O
from xpose_b200.decode import DecodeConfig

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(O.ref_gpu() is None, reason="oracle/_ref/libxpref_gpu.so not built")]

# 6 layers, window 16, global every 3: 130 prompt positions cross the
# reference's 128-span switch to its parallel attention forms
# (attention_scores_mq4, softmax_rows_partial/finish/scale, attention_apply_mq4).
CFG = DecodeConfig(n_layers=6, hidden=256, ffn=512, vocab=1024, max_seq=160, sliding_window=16, global_every=3)


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_reference_engine_runs_on_b200_kernels():
    om = O.OracleModel(CFG, seed=4, kv_fp16=False, norm_roundtrip=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        O.write_model_gguf(om, path, window=CFG.sliding_window)
        rs = O.RefSession(path, CFG.max_seq, CFG.global_every, lib=O.ref_gpu())
        try:
            prompt = O.gen_tokens(4, 77, 130, CFG.vocab)
            rs.prefill(prompt)
            want = None
            for p, t in enumerate(prompt):
                want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
            assert rel(rs.logits(CFG.vocab), want) < 1e-4
            pos = len(prompt)
            for _ in range(6):
                tok = rs.decode_step()
                top2 = np.sort(want)[-2:]
                if top2[1] - top2[0] > 1e-4:
                    assert tok == int(np.argmax(want))
                want = om.forward(tok, pos)
                pos += 1
                assert rel(rs.logits(CFG.vocab), want) < 1e-4
        finally:
            rs.close()
