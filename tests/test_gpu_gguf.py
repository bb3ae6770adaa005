"""Real-weight loading: a GGUF model file through xp_session_create_gguf.

* Device dequantisation of every ggml type the loader reads is bit-exact with
  the pinned restatement of examples/llm/model/gguf.cpp:448-634.
* A GGUF of F32 tensors (norms stored as 1 + w) decodes like the oracle's
  record_token on the same weights (the reference load path of
  examples/llm/decode.cpp:1418-1535, norms loaded back as w).
* A GGUF whose matrices are Q8_0 / Q4_K / Q6_K / Q5_0 / Q4_0 / Q4_1 / F16 and
  whose embedding is BF16 gives exactly the logits of a session built from the
  same tensors dequantised and packed on the host.
* The .xpack cache (decode.cpp:711-1328): the first load writes it, the second
  loads from it with identical results; a cache the REFERENCE engine writes for
  the same file is byte-identical to ours and is accepted; a changed model
  (mtime) or a corrupted payload is refused and the planes are repacked."""
import os
import tempfile

import numpy as np
import pytest

import oracle_lib as O
from gguf_blocks import GGML_TYPES, random_blocks

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import ctypes as C  # noqa: E402

from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import check, lib  # noqa: E402
from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling  # noqa: E402

import sys  # noqa: E402
sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from gguf_writer import gemma3_meta, write_gguf  # noqa: E402

CFG = DecodeConfig(n_layers=3, hidden=256, ffn=512, vocab=4096, max_seq=96, sliding_window=16, global_every=3)
MATS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
NORMS = ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm", "attn_q_norm", "attn_k_norm")
# matrix -> ggml type, and a block scale that keeps the weights ~1e-2
MAT_TYPES = (8, 12, 14, 6, 2, 3, 1)
SCALES = {8: 2e-4, 12: 3e-5, 14: 5e-6, 6: 2e-3, 2: 3e-3, 3: 3e-3, 7: 2e-3, 1: 0.0, 0: 0.0, 30: 0.0}


def _deq(t, raw, n):
    out = np.zeros(n, np.float32)
    O.oracle().xo_gguf_dequantize.argtypes = [C.c_uint32, C.c_char_p, O.f32p, C.c_uint64]
    assert O.oracle().xo_gguf_dequantize(t, raw, out, n) == 0
    return out


@pytest.mark.parametrize("ggml_type", sorted(GGML_TYPES))
def test_device_dequantize_bitexact(ggml_type):
    n = 256 * 129
    raw = random_blocks(ggml_type, n, seed=100 + ggml_type)
    src = dev(np.frombuffer(raw, np.uint8).copy())
    out = empty(n)
    check(lib().xp_gguf_dequantize(None, ggml_type, ptr(src), ptr(out), n))
    sync()
    assert np.array_equal(host(out).view(np.uint32), _deq(ggml_type, raw, n).view(np.uint32))


def _quantised_model(path, seed):
    """A GGUF of random-block tensors; returns the fp32 tensors they decode to."""
    rng = np.random.default_rng(seed)
    H, V = CFG.hidden, CFG.vocab
    tensors, host_w = [], {"layers": []}
    emb_raw = random_blocks(30, H * V, seed)
    tensors.append(("token_embd.weight", (H, V), ("raw", 30, emb_raw)))
    for l in range(CFG.n_layers):
        lw = {"words": [], "scales": []}
        for m, (rows, cols) in enumerate(CFG.matrix_shapes()):
            t = MAT_TYPES[m]
            raw = random_blocks(t, rows * cols, seed * 100 + l * 10 + m, scale=SCALES[t])
            tensors.append((f"blk.{l}.{MATS[m]}.weight", (rows, cols), ("raw", t, raw)))
            words, scales = O.pack(_deq(t, raw, rows * cols), rows, cols)
            lw["words"].append(words)
            lw["scales"].append(scales)
        for k, name in enumerate(NORMS):
            n = H if k < 4 else CFG.head_dim
            w = (np.float32(1.0) + rng.normal(0, 0.02, n).astype(np.float32)).astype(np.float32)
            tensors.append((f"blk.{l}.{name}.weight", (n,), w))
            lw[("attn_norm", "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm", "k_norm")[k]] = w - np.float32(1.0)
        host_w["layers"].append(lw)
    fn = (np.float32(1.0) + rng.normal(0, 0.02, H).astype(np.float32)).astype(np.float32)
    tensors.append(("output_norm.weight", (H,), fn))
    write_gguf(path, gemma3_meta(CFG, CFG.rope_theta_global, CFG.sliding_window), tensors)
    embed = _deq(30, emb_raw, H * V)
    host_w["lm_words"], host_w["lm_scales"] = O.pack(embed, H, V)
    host_w["final_norm"] = fn - np.float32(1.0)
    host_w["embed"] = embed
    return host_w


def test_f32_gguf_matches_oracle():
    om = O.OracleModel(CFG, seed=6, norm_roundtrip=True)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        O.write_model_gguf(om, path, window=CFG.sliding_window)
        s = DecodeSession.from_gguf(path, Sampling(greedy=True), max_seq=CFG.max_seq,
                                    global_every=CFG.global_every, pack_cache="")
        assert (s.cfg.n_layers, s.cfg.hidden, s.cfg.vocab, s.cfg.sliding_window) == (3, 256, 4096, 16)
        prompt = O.gen_tokens(6, 3, 20, CFG.vocab)
        s.prefill(prompt)
        want = None
        for p, t in enumerate(prompt):
            want = om.forward(int(t), p, want_logits=(p == len(prompt) - 1))
        assert rel_l2(s.last_logits(), want) < 2e-3
        pos = len(prompt)
        for _ in range(6):
            top2 = np.sort(want)[-2:]
            tok = s.decode_step()
            if top2[1] - top2[0] > 1e-4:
                assert tok == int(np.argmax(want))
            want = om.forward(tok, pos)
            pos += 1
            assert rel_l2(s.last_logits(), want) < 2e-3
        assert s.error_word() == 0


def _logits_after(s, prompt, steps=4):
    s.prefill(prompt)
    out = [s.last_logits()]
    for _ in range(steps):
        s.decode_step()
        out.append(s.last_logits())
    return np.stack(out)


def test_quantised_gguf_equals_host_packed_weights_and_cache_roundtrip():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "q.gguf")
        host_w = _quantised_model(path, seed=3)
        prompt = O.gen_tokens(3, 5, 12, CFG.vocab)
        sp = Sampling(greedy=True)
        want = _logits_after(DecodeSession.from_weights(CFG, host_w, sp), prompt)
        cache = os.path.join(d, "ours.xpack")
        a = DecodeSession.from_gguf(path, sp, max_seq=CFG.max_seq, global_every=CFG.global_every, pack_cache=cache)
        assert a.load_info()[:2] == (False, True), a.load_info()
        assert np.array_equal(_logits_after(a, prompt), want)
        b = DecodeSession.from_gguf(path, sp, max_seq=CFG.max_seq, global_every=CFG.global_every, pack_cache=cache)
        assert b.load_info()[:2] == (True, False), b.load_info()
        assert np.array_equal(_logits_after(b, prompt), want)

        # a corrupted payload byte: the entry fails its checksum, the planes are
        # repacked and the cache rewritten
        with open(cache, "r+b") as f:
            f.seek(128 + 1000)
            byte = f.read(1)
            f.seek(128 + 1000)
            f.write(bytes([byte[0] ^ 0x5A]))
        c = DecodeSession.from_gguf(path, sp, max_seq=CFG.max_seq, global_every=CFG.global_every, pack_cache=cache)
        fc, cw, msg = c.load_info()
        assert (fc, cw) == (False, True) and "checksum" in msg, msg
        assert np.array_equal(_logits_after(c, prompt), want)

        # the model file changes (a new mtime): the cache is not trusted
        st = os.stat(path)
        os.utime(path, ns=(st.st_atime_ns, st.st_mtime_ns + 1_000_000_000))
        e = DecodeSession.from_gguf(path, sp, max_seq=CFG.max_seq, global_every=CFG.global_every, pack_cache=cache)
        fc, cw, msg = e.load_info()
        assert (fc, cw) == (False, True) and "mtime" in msg, msg


@pytest.mark.skipif(O.ref() is None, reason="oracle/_ref not built")
def test_cache_is_interchangeable_with_the_reference_engine():
    """The reference's own DecodeSession (compiled for the host) writes its
    .xpack for the same model file: byte-identical to ours, and ours loads it."""
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "q.gguf")
        _quantised_model(path, seed=4)
        ours, theirs = os.path.join(d, "ours.xpack"), os.path.join(d, "ref.xpack")
        sp = Sampling(greedy=True)
        a = DecodeSession.from_gguf(path, sp, max_seq=CFG.max_seq, global_every=CFG.global_every, pack_cache=ours)
        assert a.load_info()[1]
        rl = O.ref()
        rl.xpref_set_pack_cache.argtypes = [C.c_char_p]
        rl.xpref_set_pack_cache(theirs.encode())
        try:
            rs = O.RefSession(path, CFG.max_seq, CFG.global_every)
            rs.close()
        finally:
            rl.xpref_set_pack_cache(None)
        with open(ours, "rb") as f1, open(theirs, "rb") as f2:
            assert f1.read() == f2.read()
        b = DecodeSession.from_gguf(path, sp, max_seq=CFG.max_seq, global_every=CFG.global_every, pack_cache=theirs)
        assert b.load_info()[0], b.load_info()
