"""The headline configuration itself: random-init Gemma-3-1B (26 layers,
hidden 1152, 4 q-heads / 1 kv-head of 256, FFN 6912, vocab 262,144) decoded by
the engine and by the oracle's record_token restatement (xo_forward) from the
same seeded weights, the way examples/llm/decode.cpp:2240-2329
(verify_against_cpu) checks the GPU engine against its CPU path.

Checked at three points of one sequence:
  * after a 128-token prompt (chunked prefill on the tensor-core engine);
  * 8 single-position decode steps after it (one graph replay each);
  * a greedy multi-position generate() run to position ~1100, where the
    global layers' attention windows exceed 32 splits of the default 32 rows
    and hand their partials over through a grid barrier, and the 4096-unit
    LM-head ring and all 26 layers' unit plans run at full size.
Tolerances: logits within 2e-3 relative L2, greedy
tokens equal except where the oracle's top-2 gap is below 1e-4. Tokens are
teacher-forced: the oracle always consumes the engine's token."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")
from gpu_util import rel_l2  # noqa: E402
from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling  # noqa: E402

SEED = 2026
PROMPT = 128
DECODE = 8
DEEP = 1100


def _gap_ok(logits, tok):
    top2 = np.sort(logits)[-2:]
    return top2[1] - top2[0] <= 1e-4 or tok == int(np.argmax(logits))


def test_gemma3_1b_full_size_matches_oracle():
    cfg = DecodeConfig(max_seq=DEEP + 16)
    sess = DecodeSession.random(cfg, Sampling(greedy=True), seed=SEED)
    om = O.OracleModel(cfg, SEED)
    prompt = O.gen_tokens(SEED, 1, PROMPT, cfg.vocab)

    # 1. chunked prefill
    sess.prefill(prompt)
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == PROMPT - 1))
    err = rel_l2(sess.last_logits(), want)
    assert err < 2e-3, f"after prefill: rel L2 {err:.3e}"
    pos = PROMPT

    # 2. single-position decode steps
    for _ in range(DECODE):
        tok = sess.decode_step()
        assert _gap_ok(want, tok), f"position {pos}: token {tok} vs oracle {int(np.argmax(want))}"
        want = om.forward(tok, pos)
        pos += 1
        err = rel_l2(sess.last_logits(), want)
        assert err < 2e-3, f"position {pos}: rel L2 {err:.3e}"
    assert sess.error_word() == 0

    # 3. multi-position greedy launches deep enough for the >32-split path
    n = DEEP - pos
    toks, _ = sess.generate(n)
    mismatched = []
    for t in toks:
        t = int(t)
        if not _gap_ok(want, t):
            mismatched.append((pos, t, int(np.argmax(want))))
        want = om.forward(t, pos)
        pos += 1
    assert not mismatched, f"greedy tokens differ beyond the 1e-4 gap rule: {mismatched[:5]}"
    assert sess.position() == pos == DEEP
    err = rel_l2(sess.last_logits(), want)
    assert err < 2e-3, f"position {pos}: rel L2 {err:.3e}"
    assert sess.error_word() == 0
