"""GPU parity of the fused attention and the device sampler against the oracle."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import check, lib  # noqa: E402

HD, NH = 256, 4


def f16(a):
    o = O.oracle()
    return np.array([o.xo_f32_to_f16(float(v)) for v in a], np.uint16)


def _oracle_qk_post(raw, w, n_heads, pos, theta, eps=1e-6):
    out = np.empty_like(raw)
    O.oracle().xo_rmsnorm_heads_gemma(out, np.ascontiguousarray(raw), w, n_heads, HD, eps)
    O.oracle().xo_rope(out, n_heads, HD, pos, theta)
    return out


# (pos, window, nsplit): kSeqLen 131 (examples/llm/kernel_tests.cpp:43), a
# windowed case past the window, position 0, and a long global span.
# split counts cover every cluster size of the merge: 16 (one or several
# clusters), 8, 4, 2, and lone CTAs (3 clusters of one; a single CTA)
CASES = [(130, 0, 16), (700, 512, 16), (0, 512, 16), (130, 16, 4), (4095, 0, 64), (8191, 0, 128),
         (300, 0, 8), (300, 512, 6), (200, 0, 3), (8191, 512, 1)]


@pytest.mark.parametrize("pos,window,nsplit", CASES)
def test_attention_decode(pos, window, nsplit):
    max_seq = 8192
    rng_seed = 20260719
    q_raw = O.gen_normal(rng_seed, 1, NH * HD, 1.0)
    k_raw = O.gen_normal(rng_seed, 2, HD, 1.0)
    v_raw = O.gen_normal(rng_seed, 3, HD, 1.0)
    qn = O.gen_normal(rng_seed, 4, HD, 0.02)
    kn = O.gen_normal(rng_seed, 5, HD, 0.02)
    theta = 1e6 if window == 0 else 1e4
    # history ~N(0,1) in fp16; position `pos` is written by the kernel
    kc = np.zeros(max_seq * HD, np.uint16)
    vc = np.zeros(max_seq * HD, np.uint16)
    hist_k = O.gen_normal(rng_seed, 6, pos * HD, 1.0)
    hist_v = O.gen_normal(rng_seed, 7, pos * HD, 1.0)
    kc[: pos * HD] = torch.from_numpy(hist_k).half().numpy().view(np.uint16)
    vc[: pos * HD] = torch.from_numpy(hist_v).half().numpy().view(np.uint16)
    dkc, dvc = dev(kc), dev(vc)
    posd = dev(np.array([pos], np.uint32))
    scratch = empty(lib().xp_attention_scratch_bytes(nsplit) // 4 + 16)
    out = torch.full((NH * HD,), -1e30, device="cuda")
    check(lib().xp_attention_decode(None, ptr(out), ptr(dev(q_raw)), ptr(dev(k_raw)), ptr(dev(v_raw)), ptr(dev(qn)),
                                    ptr(dev(kn)), ptr(dkc), ptr(dvc), ptr(posd), window, theta, 1e-6, 1.0 / 16,
                                    nsplit, max_seq, ptr(scratch)))
    sync()
    assert int(host(scratch, np.uint32)[1]) == 0  # the call's error word
    # oracle: QK-norm + RoPE, fp16 append, serial attention over the window
    q = _oracle_qk_post(q_raw, qn, NH, pos, theta)
    k = _oracle_qk_post(k_raw, kn, 1, pos, theta)
    kc[pos * HD:(pos + 1) * HD] = f16(k)
    vc[pos * HD:(pos + 1) * HD] = f16(v_raw)
    # the appended row must be bit-exact fp16 of the oracle's k and v
    assert np.array_equal(host(dkc, np.uint16)[pos * HD:(pos + 1) * HD], kc[pos * HD:(pos + 1) * HD])
    assert np.array_equal(host(dvc, np.uint16)[pos * HD:(pos + 1) * HD], vc[pos * HD:(pos + 1) * HD])
    seq = pos + 1
    kv_start = 0 if (window == 0 or seq <= window) else seq - window
    want = np.empty(NH * HD, np.float32)
    O.oracle().xo_attention(want, q, kc.ctypes.data, vc.ctypes.data, 1, NH, 1, HD, kv_start, seq - kv_start,
                            1.0 / 16)
    got = host(out)
    assert np.all(got != -1e30)
    assert rel_l2(got, want) < 1e-3, rel_l2(got, want)


def test_attention_window_negative_control():
    """A windowed run must differ from an unwindowed one past the window
    (examples/llm/kernel_tests.cpp:510, :587)."""
    pos, max_seq, nsplit = 600, 1024, 16
    outs = []
    for window in (512, 0):
        torch.manual_seed(0)
        kc = (torch.randn(max_seq * HD, device="cuda")).half()
        vc = (torch.randn(max_seq * HD, device="cuda")).half()
        q = torch.randn(NH * HD, device="cuda")
        k = torch.randn(HD, device="cuda")
        v = torch.randn(HD, device="cuda")
        w = torch.zeros(HD, device="cuda")
        posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
        scratch = empty(lib().xp_attention_scratch_bytes(nsplit) // 4 + 16)
        out = empty(NH * HD)
        check(lib().xp_attention_decode(None, ptr(out), ptr(q), ptr(k), ptr(v), ptr(w), ptr(w), ptr(kc), ptr(vc),
                                        ptr(posd), window, 1e4, 1e-6, 1.0 / 16, nsplit, max_seq, ptr(scratch)))
        sync()
        outs.append(host(out))
    assert rel_l2(outs[0], outs[1]) > 1e-2


def test_sample_topk_matches_oracle():
    n = 262144
    o = O.oracle()
    scratch = empty(lib().xp_sample_scratch_bytes(n) // 4 + 16)
    for trial in range(6):
        logits = O.gen_normal(42, 100 + trial, n, 3.0)
        if trial == 1:
            logits[1234] = logits[9999] = logits.max() + 0.5   # planted duplicate: tie -> lower index
        if trial in (2, 4):
            # coarse values: the 64th largest sits inside a tie group, so the
            # candidate bounds and ranks must order ties by index
            step = 1.0 if trial == 2 else 0.25
            logits = (np.round(logits / step) * step).astype(np.float32)
        tok = empty(1, torch.int32)
        vals = empty(64)
        idx = empty(64, torch.int32)
        pos = trial * 7 + 3
        posd = dev(np.array([pos], np.uint32))
        top_k, T, top_p = 64, 1.0, (0.95 if trial % 2 == 0 else 1.0)
        check(lib().xp_sample_topk(None, ptr(tok), ptr(vals), ptr(idx), ptr(dev(logits)), n, top_k, T, top_p,
                                   77, 5, ptr(posd), ptr(scratch)))
        sync()
        wv = np.empty(64, np.float32)
        wi = np.empty(64, np.uint32)
        assert o.xo_topk(logits, n, 64, wv, wi) == 64
        assert np.array_equal(host(idx, np.uint32), wi)
        assert np.array_equal(host(vals), wv)
        u = O.oracle().xo_uniform(77, 5, pos)
        want = o.xo_sample(logits, n, T, top_k, top_p, u)
        assert int(host(tok, np.uint32)[0]) == want


def test_sample_topk_tie_and_boundary():
    n = 262144
    logits = np.full(n, -5.0, np.float32)
    logits[[7, 190037, n - 3]] = 42.0     # examples/llm/sampling_test.cpp:174-179
    scratch = empty(lib().xp_sample_scratch_bytes(n) // 4 + 16)
    for k in (1, 64):
        tok = empty(1, torch.int32)
        idx = empty(64, torch.int32)
        vals = empty(64)
        posd = dev(np.array([0], np.uint32))
        check(lib().xp_sample_topk(None, ptr(tok), ptr(vals), ptr(idx), ptr(dev(logits)), n, k, 1.0, 1.0, 1, 1,
                                   ptr(posd), ptr(scratch)))
        sync()
        got_idx = host(idx, np.uint32)
        assert list(got_idx[:min(k, 3)]) == [7, 190037, n - 3][:min(k, 3)]
        if k == 1:
            assert int(host(tok, np.uint32)[0]) == 7
