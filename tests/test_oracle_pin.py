"""Pins the CPU oracle (oracle/xp_oracle.c) to the reference itself: the
reference's own kernels and host engine compiled from source into oracle/_ref
(oracle/Makefile). Bit-exact wherever the restatement follows the reference's
fp32 operation order; known-answer cases from the reference's harnesses
(examples/llm/sampling_test.cpp, kernel_tests.cpp). Skipped when oracle/_ref
was not built (the reference tree is not present)."""
import os
import tempfile

import numpy as np
import pytest

import oracle_lib as O
from xpose_b200.decode import DecodeConfig

pytestmark = pytest.mark.skipif(O.ref() is None, reason="oracle/_ref not built (reference tree absent)")

# examples/llm/kernel_tests.cpp:136-137: mt19937(20260719), U(-1.5, 1.5)
RNG = np.random.default_rng(20260719)


def urand(n, lo=-1.5, hi=1.5):
    return RNG.uniform(lo, hi, n).astype(np.float32)


@pytest.mark.parametrize("rows,cols", [(1152, 6912), (128, 64), (6912, 128), (1024, 1152)])
def test_packer_bitexact(rows, cols):
    w = O.gen_normal(0, 1, rows * cols, 0.02)
    w[:32] = 0.0
    w[32:64] = np.float32(1e-30)
    w[96:128] = np.linspace(-7, 7, 32, dtype=np.float32)   # exact multiples: lround ties
    a = O.pack(w, rows, cols)
    b = O.pack(w, rows, cols, impl="ref")
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])


def test_best_bf16_scale_matches():
    o, r = O.oracle(), O.ref()
    for i in range(2000):
        blk = O.gen_normal(5, i, 32, 0.02 * (1 + i % 7))
        s0 = np.float32(np.abs(blk).max() / np.float32(7.0))
        assert o.xo_best_bf16_scale(blk, s0) == r.xpref_best_bf16_scale(blk, s0)


@pytest.mark.parametrize("rows,cols", [(1152, 1024), (1152, 256), (1024, 1152), (6912, 1152), (1152, 8192)])
def test_mv_km4_bs_bitexact(rows, cols):
    w = O.gen_normal(7, 1, rows * cols, 0.02)
    x = urand(rows, -1.0, 1.0)
    words, scales = O.pack(w, rows, cols)
    want = np.zeros(cols, np.float32)
    O.ref_launch("mv_km4_bs", cols, want, x, words, scales, rows, cols)
    assert np.array_equal(O.mv(x, words, scales, rows, cols), want)


def test_mv_split_reduce_bitexact():
    rows, cols, split = 6912, 1152, 4
    w = O.gen_normal(8, 1, rows * cols, 0.02)
    x = urand(rows)
    words, scales = O.pack(w, rows, cols)
    part = np.zeros(split * cols, np.float32)
    out = np.zeros(cols, np.float32)
    O.ref_launch("mv_km4_bs_split", cols * split, part, x, words, scales, rows, cols, split)
    O.ref_launch("mv_reduce", cols, out, part, cols, split)
    assert np.array_equal(O.mv(x, words, scales, rows, cols, split=split), out)


def test_rmsnorm_two_pass_bitexact():
    n, nparts = 1152, 64
    x, w = urand(n), urand(n, -0.1, 0.1)
    part = np.zeros(nparts, np.float32)
    want = np.zeros(n, np.float32)
    O.ref_launch("rmsnorm_sumsq", nparts, part, x, n, nparts)
    O.ref_launch("rmsnorm_apply_gemma", n, want, x, w, part, n, nparts, 1e-6)
    got = np.zeros(n, np.float32)
    O.oracle().xo_rmsnorm_gemma(got, x, w, n, nparts, 1e-6)
    assert np.array_equal(got, want)


def test_heads_norm_bitexact():
    x, w = urand(1024), urand(256, -0.1, 0.1)
    want = np.zeros(1024, np.float32)
    O.ref_launch("rmsnorm_heads_gemma", 1024, want, x, w, 4, 256, 1e-6)
    got = np.zeros(1024, np.float32)
    O.oracle().xo_rmsnorm_heads_gemma(got, x, w, 4, 256, 1e-6)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("pos,theta", [(0, 1e6), (37, 1e4), (4095, 1e6), (8191, 1e4)])
def test_rope_matches(pos, theta):
    x = urand(1024)
    want = x.copy()
    O.ref_launch("rope", 512, want, 4, 256, pos, theta)
    got = x.copy()
    O.oracle().xo_rope(got, 4, 256, pos, theta)
    # the oracle rounds theta^(-2d/hd) once from double; the reference's fp32
    # exp2/log2 can differ by an ulp, which moves the angle by pos * ulp
    np.testing.assert_allclose(got, want, rtol=0, atol=2e-3 if pos > 1000 else 1e-5)


def test_geglu_bitexact():
    g, u = urand(6912, -12, 12), urand(6912)
    want = np.zeros(6912, np.float32)
    O.ref_launch("geglu", 6912, want, g, u, 6912)
    got = np.zeros(6912, np.float32)
    O.oracle().xo_geglu(got, g, u, 6912)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("seq,window", [(131, 0), (131, 64), (700, 512)])
def test_attention_serial_bitexact(seq, window):
    """kSeqLen 131 (kernel_tests.cpp:43); windowed suffix (decode.hpp:327-352)."""
    nh, hd = 4, 256
    q = urand(nh * hd)
    kc, vc = urand(seq * hd), urand(seq * hd)
    kv_start = 0 if (window == 0 or seq <= window) else seq - window
    span = seq - kv_start
    scores = np.zeros(nh * span, np.float32)
    want = np.zeros(nh * hd, np.float32)
    O.ref_launch("attention_scores", nh * span, scores, q, kc, nh, 1, hd, span, 1.0 / 16, kv_start)
    O.ref_launch("softmax_rows", nh, scores, nh, span)
    O.ref_launch("attention_apply", nh * hd, want, scores, vc, nh, 1, hd, span, kv_start)
    got = np.zeros(nh * hd, np.float32)
    O.oracle().xo_attention(got, q, kc.ctypes.data, vc.ctypes.data, 0, nh, 1, hd, kv_start, span, 1.0 / 16)
    assert np.array_equal(got, want)


def test_argmax_known_answers():
    """examples/llm/sampling_test.cpp:136-138 and :174-179."""
    n = 262144
    x = urand(n, -10, 10)
    x[190037] = 99.5
    for logits, best in ((x, 190037),):
        pv, pi = np.zeros(4096, np.float32), np.zeros(4096, np.uint32)
        pv2, pi2 = np.zeros(64, np.float32), np.zeros(64, np.uint32)
        out, oi = np.zeros(2, np.float32), np.zeros(1, np.uint32)
        O.ref_launch("argmax_partial", 4096, pv, pi, logits, n, 4096)
        O.ref_launch("argmax_reduce", 64, pv2, pi2, pv, pi, 4096, 64)
        O.ref_launch("argmax_final", 1, out, oi, pv2, pi2, 64)
        assert oi[0] == best == O.oracle().xo_argmax(logits, n, None)
    y = np.full(n, -1.0, np.float32)
    y[[7, 190037, n - 3]] = 42.0
    assert O.oracle().xo_argmax(y, n, None) == 7


def test_topk_known_answers():
    """k = 40 with a planted duplicate 3.25 at 1234 / 9999 against a stable
    sort (sampling_test.cpp:428-481); k in {1, 64} (:486-500)."""
    n = 262144
    x = urand(n, -3, 3)
    x[1234] = x[9999] = 3.25
    order = np.lexsort((np.arange(n), -x))
    for k in (1, 40, 64):
        nparts = 256
        cv, ci = np.zeros(nparts * k, np.float32), np.zeros(nparts * k, np.uint32)
        ov, oi = np.zeros(k, np.float32), np.zeros(k, np.uint32)
        O.ref_launch("topk_partial", nparts, cv, ci, x, n, nparts, k)
        O.ref_launch("topk_rank_select", nparts * k, ov, oi, cv, ci, nparts * k, k)
        v, i = np.zeros(k, np.float32), np.zeros(k, np.uint32)
        assert O.oracle().xo_topk(x, n, k, v, i) == k
        assert np.array_equal(i, oi) and np.array_equal(i, order[:k].astype(np.uint32))
        assert np.array_equal(v, ov)


def test_topp_keeps_crossing_token():
    """llm_sampling.cl:403-421 / decode.cpp:1902-1905: the token whose mass
    crosses top_p is kept; with one dominant token only it survives."""
    n = 1000
    x = np.full(n, -50.0, np.float32)
    x[10], x[20], x[30] = 10.0, 9.0, 0.0
    o = O.oracle()
    for u in (0.0, 0.5, 0.999):
        assert o.xo_sample(x, n, 1.0, 64, 0.5, u) == 10
    # p = 0.99 keeps 10 and 20 (their mass crosses 0.99 only with both)
    picks = {o.xo_sample(x, n, 1.0, 64, 0.99, u) for u in np.linspace(0, 0.999, 64)}
    assert picks == {10, 20}


def test_softmax_stability():
    """A +1000 offset must not overflow (sampling_test.cpp softmax case)."""
    x = urand(512) + 1000.0
    o = O.oracle()
    t = o.xo_sample(x, 512, 1.0, 64, 0.95, 0.3)
    assert 0 <= t < 512


SMALL = DecodeConfig(n_layers=6, hidden=256, ffn=512, vocab=1024, max_seq=160, sliding_window=16, global_every=3)


def test_reference_engine_matches_oracle():
    """The reference's whole DecodeSession (GGUF load, int4 packer,
    record_token, greedy argmax tree) against the oracle's xo_forward with
    fp32 KV, on a random-init model written as a GGUF file. Spans pass the
    reference's 128-position switch to its parallel attention forms."""
    cfg = SMALL
    om = O.OracleModel(cfg, seed=4, kv_fp16=False, norm_roundtrip=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        O.write_model_gguf(om, path, window=cfg.sliding_window)
        rs = O.RefSession(path, cfg.max_seq, cfg.global_every)
        try:
            prompt = O.gen_tokens(4, 77, 130, cfg.vocab)
            rs.prefill(prompt)
            want = None
            for p, t in enumerate(prompt):
                want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
            got = rs.logits(cfg.vocab)
            assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-5
            pos = len(prompt)
            for _ in range(6):
                tok = rs.decode_step()
                assert tok == int(np.argmax(want))
                want = om.forward(tok, pos)
                pos += 1
                got = rs.logits(cfg.vocab)
                assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-5
        finally:
            rs.close()


# ---- prefill shapes (kernels/llm_sampling.cl:495-736), the shapes of
# examples/llm/sampling_test.cpp:725-1020 (37 rows: not a multiple of 64)
T37 = 37


def test_prefill_softmax_rows_bitexact():
    rows, cols = 4 * T37, T37
    x = urand(rows * cols, -1.5, 1.5)
    x[5 * cols + 3:5 * cols + 9] = -np.inf  # a partly masked row
    x[7 * cols:8 * cols] = -np.inf  # a fully masked row
    st_r, st_o = np.zeros(2 * rows, np.float32), np.zeros(2 * rows, np.float32)
    O.ref_launch("softmax_rows_stats", rows, st_r, x, rows, cols)
    O.oracle().xo_softmax_rows_stats(st_o, x, rows, cols)
    assert np.array_equal(st_r, st_o)
    xr, xo = x.copy(), x.copy()
    O.ref_launch("softmax_rows_apply", rows * cols, xr, st_r, rows, cols)
    O.oracle().xo_softmax_rows_apply(xo, st_o, rows, cols)
    assert np.array_equal(xr, xo)


@pytest.mark.parametrize("window,q_offset", [(0, 0), (8, 0), (0, 20), (16, 40)])
def test_prefill_attention_bitexact(window, q_offset):
    nh, kvh, hd, nq = 4, 1, 256, T37
    seq = q_offset + nq
    q = urand(nh * nq * hd, -1.5, 1.5)
    kc, vc = urand(seq * kvh * hd, -1.5, 1.5), urand(seq * kvh * hd, -1.5, 1.5)
    sr, so = np.zeros(nh * nq * seq, np.float32), np.zeros(nh * nq * seq, np.float32)
    O.ref_launch("attention_scores_prefill", nh * nq * seq, sr, q, kc, nh, kvh, hd, nq, seq, q_offset, window,
                 1.0 / 16)
    O.oracle().xo_attention_scores_prefill(so, q, kc, nh, kvh, hd, nq, seq, q_offset, window, 1.0 / 16)
    assert np.array_equal(sr, so)
    st = np.zeros(2 * nh * nq, np.float32)
    O.oracle().xo_softmax_rows_stats(st, so, nh * nq, seq)
    O.oracle().xo_softmax_rows_apply(so, st, nh * nq, seq)
    outr, outo = np.zeros(nh * nq * hd, np.float32), np.zeros(nh * nq * hd, np.float32)
    O.ref_launch("attention_apply_prefill", nh * nq * hd, outr, so, vc, nh, kvh, hd, nq, seq)
    O.oracle().xo_attention_apply_prefill(outo, so, vc, nh, kvh, hd, nq, seq)
    assert np.array_equal(outr, outo)


def test_prefill_norms_bitexact():
    H = 1152
    x, w = urand(T37 * H, -1.5, 1.5), urand(H, -1.5, 1.5)
    ssr, sso = np.zeros(T37, np.float32), np.zeros(T37, np.float32)
    O.ref_launch("rmsnorm_rows_sumsq", T37, ssr, x, T37, H)
    O.oracle().xo_rmsnorm_rows_sumsq(sso, x, T37, H)
    assert np.array_equal(ssr, sso)
    outr, outo = np.zeros(T37 * H, np.float32), np.zeros(T37 * H, np.float32)
    O.ref_launch("rmsnorm_rows_apply_gemma", T37 * H, outr, x, w, ssr, T37, H, 1e-6)
    O.oracle().xo_rmsnorm_rows_apply_gemma(outo, x, w, sso, T37, H, 1e-6)
    assert np.array_equal(outr, outo)
    x2, w2 = urand(T37 * 4 * 256, -1.5, 1.5), urand(256, -1.5, 1.5)
    hr, ho = np.zeros_like(x2), np.zeros_like(x2)
    O.ref_launch("rmsnorm_heads_rows_gemma", x2.size, hr, x2, w2, T37, 4, 256, 1e-6)
    O.oracle().xo_rmsnorm_heads_rows_gemma(ho, x2, w2, T37, 4, 256, 1e-6)
    assert np.array_equal(hr, ho)


@pytest.mark.parametrize("pos0,theta", [(5, 1e6), (4000, 1e4)])
def test_prefill_rope_matches(pos0, theta):
    x = urand(T37 * 4 * 256, -1.5, 1.5)
    xr, xo = x.copy(), x.copy()
    O.ref_launch("rope_prefill", T37 * 4 * 128, xr, T37, 4, 256, pos0, theta)
    O.oracle().xo_rope_prefill(xo, T37, 4, 256, pos0, theta)
    # theta^(-2d/hd): rounded once from double here, the reference's fp32
    # exp2/log2 can differ by an ulp, which moves the angle by pos * ulp
    np.testing.assert_allclose(xo, xr, rtol=0, atol=2e-3 if pos0 > 1000 else 1e-5)


def test_prefill_plumbing_bitexact():
    row, cap, pos0 = 256, 64, 11
    cache = np.full(row * cap, 7.0, np.float32)
    src = urand(row * T37)
    cr, co = cache.copy(), cache.copy()
    O.ref_launch("kv_append_rows", T37 * row, cr, src, T37, row, pos0)
    O.oracle().xo_kv_append_rows(co, src, T37, row, pos0)
    assert np.array_equal(cr, co)
    vocab, H = 4096, 1152
    table = (np.arange(vocab * H) % 977).astype(np.float32) * np.float32(0.01)
    toks = ((np.arange(T37) * 251 + 13) % vocab).astype(np.uint32)
    er, eo = np.zeros(T37 * H, np.float32), np.zeros(T37 * H, np.float32)
    O.ref_launch("embed_lookup_rows", T37 * H, er, table, toks, T37, H)
    O.oracle().xo_embed_lookup_rows(eo, table, toks, T37, H)
    assert np.array_equal(er, eo)


# ---- GGUF tensor types (examples/llm/model/gguf.cpp:448-634) and the .xpack
# payload hash (examples/llm/decode.cpp:784-834)
@pytest.mark.parametrize("ggml_type", [0, 1, 30, 2, 3, 6, 7, 8, 12, 14])
def test_gguf_dequantize_bitexact(ggml_type):
    import ctypes as C
    from gguf_blocks import random_blocks
    n = 256 * 37
    raw = random_blocks(ggml_type, n, seed=ggml_type)
    want, got = np.zeros(n, np.float32), np.zeros(n, np.float32)
    lib = O.ref()
    lib.xpref_gguf_dequantize.argtypes = [C.c_uint32, C.c_char_p, O.f32p, C.c_uint64]
    assert lib.xpref_gguf_dequantize(ggml_type, raw, want, n) == 0
    O.oracle().xo_gguf_dequantize.argtypes = [C.c_uint32, C.c_char_p, O.f32p, C.c_uint64]
    assert O.oracle().xo_gguf_dequantize(ggml_type, raw, got, n) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("nbytes", [0, 7, 8, 4096 + 3, (4 << 20) * 2 + 12345])
def test_xpack_hash_matches(nbytes):
    import ctypes as C
    data = np.random.default_rng(nbytes).integers(0, 256, nbytes, dtype=np.uint8).tobytes()
    lib, o = O.ref(), O.oracle()
    lib.xpref_xpack_hash.restype = C.c_uint64
    lib.xpref_xpack_hash.argtypes = [C.c_char_p, C.c_uint64]
    lib.xpref_xpack_hash_mt.restype = C.c_uint64
    lib.xpref_xpack_hash_mt.argtypes = [C.c_char_p, C.c_uint64, C.c_uint32]
    o.xo_xpack_hash.restype = C.c_uint64
    o.xo_xpack_hash.argtypes = [C.c_char_p, C.c_uint64]
    o.xo_xpack_hash_chunked.restype = C.c_uint64
    o.xo_xpack_hash_chunked.argtypes = [C.c_char_p, C.c_uint64]
    assert o.xo_xpack_hash(data, nbytes) == lib.xpref_xpack_hash(data, nbytes)
    assert o.xo_xpack_hash_chunked(data, nbytes) == lib.xpref_xpack_hash_mt(data, nbytes, 1)
    assert o.xo_xpack_hash_chunked(data, nbytes) == lib.xpref_xpack_hash_mt(data, nbytes, 4)
