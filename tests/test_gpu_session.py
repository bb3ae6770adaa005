"""The decode engine (one CUDA graph per token) against the oracle's
record_token restatement on a small random-init model with the Gemma-3
head layout, built from the same seeded generator and stream ids."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")
from gpu_util import rel_l2  # noqa: E402
from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling  # noqa: E402

SMALL = DecodeConfig(n_layers=3, hidden=256, ffn=512, vocab=4096, max_seq=64, sliding_window=16, global_every=3)


def _check_logits(got, want, tol=2e-3):
    assert rel_l2(got, want) < tol, rel_l2(got, want)


def test_session_greedy_matches_oracle():
    cfg = SMALL
    seed = 7
    om = O.OracleModel(cfg, seed)
    sess = DecodeSession.random(cfg, Sampling(greedy=True), seed=seed)
    prompt = O.gen_tokens(seed, 500, 12, cfg.vocab)
    sess.prefill(prompt)
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
    _check_logits(sess.last_logits(), want)
    pos = len(prompt)
    # teacher-forced greedy: both sides consume the engine's token
    for step in range(24):
        top2 = np.sort(want)[-2:]
        tok = sess.decode_step()
        if top2[1] - top2[0] > 1e-4:
            assert tok == int(np.argmax(want))
        want = om.forward(tok, pos)
        pos += 1
        _check_logits(sess.last_logits(), want)
    assert sess.position() == pos


def test_session_from_host_weights_matches_random_init():
    cfg = SMALL
    om = O.OracleModel(cfg, 11)
    a = DecodeSession.random(cfg, Sampling(), seed=11)
    b = DecodeSession.from_weights(cfg, om.weights_dict(), Sampling())
    prompt = O.gen_tokens(11, 9, 5, cfg.vocab)
    a.prefill(prompt)
    b.prefill(prompt)
    assert np.array_equal(a.last_logits(), b.last_logits())
    for _ in range(5):
        assert a.decode_step() == b.decode_step()


def test_session_generate_matches_steps():
    cfg = SMALL
    a = DecodeSession.random(cfg, Sampling(), seed=3)
    b = DecodeSession.random(cfg, Sampling(), seed=3)
    prompt = O.gen_tokens(3, 1, 6, cfg.vocab)
    a.prefill(prompt)
    b.prefill(prompt)
    steps = [a.decode_step() for _ in range(20)]
    toks, ms = b.generate(20)
    assert list(toks) == steps
    assert ms > 0
    assert np.array_equal(a.last_logits(), b.last_logits())


def test_session_sampling_matches_oracle():
    cfg = SMALL
    sp = Sampling(greedy=False, temperature=1.0, top_k=64, top_p=0.95, seed=99, seq_id=3)
    om = O.OracleModel(cfg, 5)
    sess = DecodeSession.random(cfg, sp, seed=5)
    prompt = O.gen_tokens(5, 2, 8, cfg.vocab)
    sess.prefill(prompt)
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
    pos = len(prompt)
    for step in range(16):
        tok = sess.decode_step()
        u = O.oracle().xo_uniform(sp.seed, sp.seq_id, pos - 1)
        exp_tok = O.oracle().xo_sample(want, cfg.vocab, sp.temperature, sp.top_k, sp.top_p, u)
        if tok != exp_tok:
            # logits agree to ~1e-6, so a different draw is only acceptable
            # where the uniform sits on a CDF boundary of the oracle's draw
            lo = O.oracle().xo_sample(want, cfg.vocab, sp.temperature, sp.top_k, sp.top_p, max(0.0, u - 1e-5))
            hi = O.oracle().xo_sample(want, cfg.vocab, sp.temperature, sp.top_k, sp.top_p, min(1.0, u + 1e-5))
            assert lo != hi and tok in (lo, hi), (pos, tok, exp_tok)
        want = om.forward(tok, pos)
        pos += 1


def test_session_errors():
    cfg = SMALL
    sess = DecodeSession.random(cfg, Sampling(), seed=1)
    from xpose_b200 import XpError
    with pytest.raises(XpError) as e:
        sess.decode_step()
    assert e.value.name == "XP_ERR_STATE"
    with pytest.raises(XpError):
        sess.prefill([cfg.vocab])  # out of vocabulary
    sess.reset()
    sess.prefill(O.gen_tokens(1, 1, cfg.max_seq, cfg.vocab))
    with pytest.raises(XpError) as e:
        sess.decode_step()
    assert e.value.name == "XP_ERR_KV_FULL"
    assert sess.error_word() == 0


def test_session_many_splits_and_reset(monkeypatch):
    """Attention windows of more than 32 splits hand their partials to the O
    step through a grid barrier, shorter ones as flagged words; a long
    prompt with 8-row splits runs both kinds in one model (global layers
    past position 256, local layers within their 16-row window), and a
    reset must clear the flags so the same positions decode again."""
    monkeypatch.setenv("XP_TK_CHUNK_MIN", "8")
    cfg = DecodeConfig(n_layers=3, hidden=256, ffn=512, vocab=4096, max_seq=320, sliding_window=16, global_every=3)
    seed = 13
    om = O.OracleModel(cfg, seed)
    sess = DecodeSession.random(cfg, Sampling(greedy=True), seed=seed)
    prompt = O.gen_tokens(seed, 77, 290, cfg.vocab)
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
    for rep in range(2):
        sess.prefill(prompt)
        _check_logits(sess.last_logits(), want)
        toks, _ = sess.generate(8)
        if rep == 0:
            first = list(toks)
        else:
            assert list(toks) == first
        assert sess.error_word() == 0
        sess.reset()


def test_five_kernel_graph_matches_oracle(monkeypatch):
    """The graph of separate kernels per layer (matvec, attention, matvec,
    matvec per layer; the engine's path for shapes the token kernel does not
    plan, forced here with XP_ENGINE_MULTI=1) against the oracle."""
    monkeypatch.setenv("XP_ENGINE_MULTI", "1")
    cfg = SMALL
    seed = 17
    om = O.OracleModel(cfg, seed)
    sess = DecodeSession.random(cfg, Sampling(greedy=True), seed=seed)
    monkeypatch.delenv("XP_ENGINE_MULTI")
    assert sess.stats()["kernels_per_token"] > 1
    prompt = O.gen_tokens(seed, 501, 10, cfg.vocab)
    sess.prefill(prompt)
    want = None
    for p, t in enumerate(prompt):
        want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
    _check_logits(sess.last_logits(), want)
    pos = len(prompt)
    for _ in range(12):
        top2 = np.sort(want)[-2:]
        tok = sess.decode_step()
        if top2[1] - top2[0] > 1e-4:
            assert tok == int(np.argmax(want))
        want = om.forward(tok, pos)
        pos += 1
        _check_logits(sess.last_logits(), want)
    assert sess.error_word() == 0
