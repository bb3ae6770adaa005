"""Chunked prefill: a prompt of 32 or more tokens runs 64 positions per pass
on the batched tensor-core engine over the session's own KV caches (every
row's k and v appended before any row attends). It must leave the session
where a pass per token leaves it: last logits within 1e-3 relative L2 of the
per-token path and of the oracle, the same position, and KV caches that the
following decode steps read to the same results."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")
from gpu_util import rel_l2  # noqa: E402
from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling  # noqa: E402

# Gemma-3 widths, three layers (local window 16, every second layer global)
CFG = DecodeConfig(n_layers=3, vocab=32768, max_seq=160, global_every=2, sliding_window=16)


def _pair(monkeypatch, sp, seed):
    a = DecodeSession.random(CFG, sp, seed=seed)  # chunked (default threshold 32)
    monkeypatch.setenv("XP_PREFILL_CHUNK_MIN", "1000000")
    b = DecodeSession.random(CFG, sp, seed=seed)  # one pass per token
    monkeypatch.delenv("XP_PREFILL_CHUNK_MIN")
    return a, b


def test_chunked_prefill_matches_per_token_and_oracle(monkeypatch):
    seed = 21
    prompt = O.gen_tokens(seed, 40, 100, CFG.vocab)  # two passes: 64 + 36 rows
    a, b = _pair(monkeypatch, Sampling(greedy=True), seed)
    a.prefill(prompt)
    monkeypatch.setenv("XP_PREFILL_CHUNK_MIN", "1000000")
    b.prefill(prompt)
    monkeypatch.delenv("XP_PREFILL_CHUNK_MIN")
    assert a.position() == b.position() == len(prompt)
    la, lb = a.last_logits(), b.last_logits()
    assert rel_l2(la, lb) < 1e-3, rel_l2(la, lb)
    om = O.OracleModel(CFG, seed)
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
    assert rel_l2(la, want) < 2e-3, rel_l2(la, want)
    # decoding continues from the chunk-written caches
    for _ in range(8):
        top2 = np.sort(b.last_logits())[-2:]
        ta, tb = a.decode_step(), b.decode_step()
        if top2[1] - top2[0] > 1e-3:
            assert ta == tb
        if ta != tb:
            break
        assert rel_l2(a.last_logits(), b.last_logits()) < 1e-3
    assert a.error_word() == 0


def test_chunked_prefill_sampling_and_second_prompt(monkeypatch):
    sp = Sampling(greedy=False, temperature=1.0, top_k=64, top_p=0.95, seed=7, seq_id=2)
    seed = 22
    a, b = _pair(monkeypatch, sp, seed)
    first = O.gen_tokens(seed, 41, 40, CFG.vocab)
    second = O.gen_tokens(seed, 42, 70, CFG.vocab)  # appended after the first prompt
    for s, per_token in ((a, False), (b, True)):
        if per_token:
            monkeypatch.setenv("XP_PREFILL_CHUNK_MIN", "1000000")
        s.prefill(first)
        s.prefill(second)
        monkeypatch.delenv("XP_PREFILL_CHUNK_MIN", raising=False)
    assert a.position() == b.position() == 110
    assert rel_l2(a.last_logits(), b.last_logits()) < 1e-3
    # the token drawn from the chunked prefill's logits is the reference
    # sampler's draw on those logits with the uniform of its position
    la = a.last_logits()
    u = O.oracle().xo_uniform(sp.seed, sp.seq_id, a.position() - 1)
    want_tok = O.oracle().xo_sample(la, CFG.vocab, sp.temperature, sp.top_k, sp.top_p, u)
    assert a.decode_step() == want_tok
    a.reset()
    a.prefill(first)
    b.reset()
    monkeypatch.setenv("XP_PREFILL_CHUNK_MIN", "1000000")
    b.prefill(first)
    assert rel_l2(a.last_logits(), b.last_logits()) < 1e-3
