"""The chat front-end (C ABI xp_chat_*, llm_jni.cpp:59-186) on a GGUF model
that carries a SentencePiece vocabulary: prefill wraps the text in the Gemma
turn template with BOS on the first turn only; steps stream one token's text
at a time and equal the same decode run through a session directly; the
concatenated pieces equal the tokenizer's decode of those ids; metrics and
reset behave."""
import ctypes as C
import os
import sys
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
pytest.importorskip("torch")
from test_tokenizer import vocab  # noqa: E402
from xpose_b200._lib import check, lib  # noqa: E402
from xpose_b200.decode import DecodeConfig, DecodeSession, Sampling  # noqa: E402

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from gguf_writer import ARR, BOOL, F32, I32, STR, U32, gemma3_meta, write_gguf  # noqa: E402

V = 1024
CFG = DecodeConfig(n_layers=2, hidden=256, ffn=512, vocab=V, max_seq=128, sliding_window=16, global_every=2)


def write_chat_model(path, seed=1):
    toks, scores = vocab()
    toks += [(f"<unused{i}>", 5) for i in range(V - len(toks))]
    scores += [0.0] * (V - len(scores))
    meta = [m for m in gemma3_meta(CFG, CFG.rope_theta_global, CFG.sliding_window) if not m[0].startswith("tokenizer")]
    meta += [("tokenizer.ggml.model", STR, "llama"),
             ("tokenizer.ggml.tokens", ARR, (STR, [t for t, _ in toks])),
             ("tokenizer.ggml.scores", ARR, (F32, scores)),
             ("tokenizer.ggml.token_type", ARR, (I32, [k for _, k in toks])),
             ("tokenizer.ggml.bos_token_id", U32, 2), ("tokenizer.ggml.eos_token_id", U32, 1),
             ("tokenizer.ggml.unknown_token_id", U32, 3), ("tokenizer.ggml.add_space_prefix", BOOL, True)]
    rng = np.random.default_rng(seed)
    H = CFG.hidden
    names = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
    norms = ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm", "attn_q_norm", "attn_k_norm")
    tensors = [("token_embd.weight", (H, V), rng.normal(0, 0.02, H * V).astype(np.float32))]
    for l in range(CFG.n_layers):
        for m, (r, c) in enumerate(CFG.matrix_shapes()):
            tensors.append((f"blk.{l}.{names[m]}.weight", (r, c), rng.normal(0, 0.02, r * c).astype(np.float32)))
        for k, nm in enumerate(norms):
            n = H if k < 4 else CFG.head_dim
            tensors.append((f"blk.{l}.{nm}.weight", (n,), (1 + rng.normal(0, 0.02, n)).astype(np.float32)))
    tensors.append(("output_norm.weight", (H,), (1 + rng.normal(0, 0.02, H)).astype(np.float32)))
    write_gguf(path, meta, tensors)


def test_chat_turns_match_direct_decoding():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "chat.gguf")
        write_chat_model(path)
        ch = C.c_void_p()
        check(lib().xp_chat_create(0, path.encode(), CFG.max_seq, None, b"", C.byref(ch)))
        tk = C.c_void_p()
        check(lib().xp_tokenizer_create(path.encode(), C.byref(tk)))
        try:
            n = C.c_uint32()
            check(lib().xp_chat_prefill(ch, b"hello world", C.byref(n)))
            prompt = b"<start_of_turn>user\nhello world<end_of_turn>\n<start_of_turn>model\n"
            cnt = C.c_uint32()
            check(lib().xp_tokenizer_encode(tk, prompt, len(prompt), 1, 0, None, 0, C.byref(cnt)))
            ids = np.zeros(cnt.value, np.int32)
            check(lib().xp_tokenizer_encode(tk, prompt, len(prompt), 1, 0, ids.ctypes.data, len(ids), C.byref(cnt)))
            assert n.value == len(ids) and ids[0] == 2  # BOS on the first turn
            pieces, done = [], C.c_int(0)
            buf = C.create_string_buffer(64)
            for _ in range(20):
                check(lib().xp_chat_step(ch, buf, 64, C.byref(done)))
                if done.value:
                    break
                pieces.append(buf.value)
            m = (C.c_double * 7)()
            check(lib().xp_chat_metrics(ch, m))
            assert m[0] > 0 and m[2] >= 1 and m[3] == 1 and m[4] == len(ids) + len(pieces)

            # the same turn through a session: identical tokens and pieces
            s = DecodeSession.from_gguf(path, Sampling(greedy=False, temperature=0.7, top_k=64, top_p=0.95, seed=1234),
                                        max_seq=CFG.max_seq, global_every=6, pack_cache="")
            s.prefill(ids.astype(np.uint32))
            toks = [s.decode_step() for _ in range(len(pieces))]
            ln = C.c_size_t()
            for t, p in zip(toks, pieces):
                pb = C.create_string_buffer(64)
                check(lib().xp_tokenizer_piece(tk, t, pb, 64, C.byref(ln)))
                assert pb.raw[:ln.value] == p

            # a second turn opens with "\n" and no BOS; reset starts over
            check(lib().xp_chat_prefill(ch, b"more", C.byref(n)))
            t2 = b"\n<start_of_turn>user\nmore<end_of_turn>\n<start_of_turn>model\n"
            check(lib().xp_tokenizer_encode(tk, t2, len(t2), 0, 0, None, 0, C.byref(cnt)))
            assert n.value == cnt.value
            check(lib().xp_chat_reset(ch))
            check(lib().xp_chat_prefill(ch, b"hello world", C.byref(n)))
            assert n.value == len(ids)
        finally:
            lib().xp_chat_destroy(ch)
            lib().xp_tokenizer_destroy(tk)
