"""Batched decode (xp_bdec_*): every sequence of a batch must compute what a
batch-1 DecodeSession computes for it alone on the same weights (the batch-1
engine is itself pinned to the oracle and to the reference's own engine):
teacher-forced logits within 1e-3 relative L2 (the tensor-core matvec carries
~22-bit activations), greedy tokens equal, and sampled tokens equal given the
same (seed, seq_id, position) uniforms."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from xpose_b200.decode import BatchDecode, DecodeConfig, DecodeSession, Sampling  # noqa: E402

CFG = DecodeConfig(n_layers=3, vocab=32768, max_seq=128, global_every=2, sliding_window=16)


def rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _prompts(nseq, n, seed):
    return np.random.default_rng(seed).integers(0, CFG.vocab, (nseq, n), dtype=np.uint32)


@pytest.mark.parametrize("nseq", [4, 33])
def test_teacher_forced_logits_and_greedy_match_batch1(nseq):
    sess = DecodeSession.random(CFG, Sampling(greedy=True), seed=3)
    prompts = _prompts(nseq, 20, 1)  # crosses the 16-row window of the local layers
    bd = BatchDecode(sess, nseq, 64, Sampling(greedy=True))
    try:
        bd.prefill(prompts)
        got = bd.logits()
        toks = bd.step()
        after = bd.logits()
        for b in (0, nseq // 2, nseq - 1):
            sess.reset()
            sess.prefill(prompts[b])
            want = sess.last_logits()
            assert rel(got[b], want) < 1e-3, (b, rel(got[b], want))
            t1 = sess.decode_step()
            assert t1 == toks[b]
            assert rel(after[b], sess.last_logits()) < 1e-3
    finally:
        bd.close()


def test_sampled_tokens_match_the_batch1_sampler():
    """Each sequence's sampled token equals the batch-1 device sampler's draw
    (xp_sample_topk, kernels/llm_sampling.cl + decode.cpp:1873-1917 semantics)
    on the same logits with the uniform of (seed, seq0 + b, position)."""
    from gpu_util import dev, empty, host, ptr, sync
    from xpose_b200._lib import check, lib
    sp = dict(greedy=False, temperature=1.0, top_k=64, top_p=0.95, seed=77)
    sess = DecodeSession.random(CFG, Sampling(greedy=True), seed=5)
    prompts = _prompts(4, 12, 2)
    bd = BatchDecode(sess, 4, 64, Sampling(**sp), seq0=10)
    try:
        bd.prefill(prompts)
        logits = bd.logits()
        toks = bd.step()
        assert bd.position() == 13
        scratch = torch.zeros(lib().xp_sample_scratch_bytes(CFG.vocab) // 4 + 64, dtype=torch.int32, device="cuda")
        pos = dev(np.array([12], np.uint32))
        for b in range(4):
            tok = empty(1, torch.int32)
            check(lib().xp_sample_topk(None, ptr(tok), None, None, ptr(dev(logits[b])), CFG.vocab, 64, 1.0, 0.95, 77,
                                       10 + b, ptr(pos), ptr(scratch)))
            sync()
            assert int(host(tok, np.uint32)[0]) == toks[b], b
    finally:
        bd.close()
