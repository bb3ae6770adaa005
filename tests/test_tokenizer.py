"""The tokenizer and its GGUF vocabulary (C ABI xp_tokenizer_*, host only)
against the reference's own Tokenizer (examples/llm/model/tokenizer.cpp,
compiled from source into oracle/_ref) on a synthetic SentencePiece
vocabulary: control and unknown tokens (one a prefix of another), 256 byte
tokens, single characters, seeded multi-character pieces with tied scores,
a duplicated spelling, user-defined whitespace runs. Seeded texts mix ASCII,
newlines, multi-byte UTF-8 without vocabulary entries (byte fallback) and
embedded special-token spellings. Every encode, decode and piece must be
identical, and decode(encode(s)) must give s back for text without special
tokens."""
import ctypes as C
import os
import sys
import tempfile

import numpy as np
import pytest

import oracle_lib as O
from xpose_b200._lib import check, lib

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from gguf_writer import ARR, BOOL, F32, I32, STR, U32, write_gguf  # noqa: E402

M = "▁"
WORDS = ["the", "then", "there", "hello", "world", "token", "tokenizer", "decode", "encode", "merge", "blackwell",
         "tensor", "memory", "stream", "int4", "gemma", "model", "turn", "user", "ing", "tion", "er"]


def vocab(seed=5):
    rng = np.random.default_rng(seed)
    toks = [("<pad>", 3), ("<eos>", 3), ("<bos>", 3), ("<unk>", 2), ("<start_of_turn>", 3), ("<end_of_turn>", 3),
            ("<start>", 3)]
    toks += [(f"<0x{b:02X}>", 6) for b in range(256)]
    chars = sorted(set("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789.,!?'-:\n" + M))
    toks += [(c, 1) for c in chars]
    pieces = set()
    for w in WORDS:
        for form in (w, M + w):
            for i in range(len(form)):
                for j in range(i + 2, len(form) + 1):
                    pieces.add(form[i:j])
    pieces = sorted(pieces)
    toks += [(p, 1) for p in pieces if p not in chars]
    toks += [("\n\n", 4), (M + M, 4), ("the", 5)]  # user-defined whitespace, a duplicated spelling
    scores = [0.0] * len(toks)
    for i in range(7 + 256, len(toks)):
        scores[i] = float(np.round(-rng.uniform(0, 20) * 2) / 2)  # half steps: many ties
    return toks, scores


def write_vocab(path):
    toks, scores = vocab()
    meta = [("general.architecture", STR, "gemma3"), ("general.alignment", U32, 32),
            ("tokenizer.ggml.model", STR, "llama"),
            ("tokenizer.ggml.tokens", ARR, (STR, [t for t, _ in toks])),
            ("tokenizer.ggml.scores", ARR, (F32, scores)),
            ("tokenizer.ggml.token_type", ARR, (I32, [k for _, k in toks])),
            ("tokenizer.ggml.bos_token_id", U32, 2), ("tokenizer.ggml.eos_token_id", U32, 1),
            ("tokenizer.ggml.unknown_token_id", U32, 3), ("tokenizer.ggml.padding_token_id", U32, 0),
            ("tokenizer.ggml.add_bos_token", BOOL, True), ("tokenizer.ggml.add_space_prefix", BOOL, True)]
    write_gguf(path, meta, [])
    return len(toks)


def texts(seed=9, n=60):
    rng = np.random.default_rng(seed)
    pool = list("abcdefghijklmnopqrstuvwxyz     .,!?\n") + ["the ", "hello ", "world", "tokenizer", "é", "日本語", "🙂",
                                                           "<start_of_turn>", "<end_of_turn>", "<start>", "<unk>",
                                                           "\n\n", "  ", "ñ", "\t"]
    out = ["", " ", "hello world", "<start_of_turn>user\nhello<end_of_turn>\n<start_of_turn>model\n",
           "the then there", "  two  spaces", "日本語 🙂 é"]
    for _ in range(n):
        out.append("".join(pool[i] for i in rng.integers(0, len(pool), rng.integers(1, 40))))
    return out


@pytest.fixture(scope="module")
def both():
    ref = O.ref()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    ref.xpref_tok_create.restype = C.c_void_p
    ref.xpref_tok_create.argtypes = [C.c_char_p]
    ref.xpref_tok_encode.argtypes = [C.c_void_p, C.c_char_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_uint32]
    ref.xpref_tok_decode.restype = C.c_long
    ref.xpref_tok_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_uint32, C.c_int, C.c_char_p, C.c_size_t]
    ref.xpref_tok_piece.restype = C.c_long
    ref.xpref_tok_piece.argtypes = [C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t]
    ref.xpref_tok_destroy.argtypes = [C.c_void_p]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "vocab.gguf")
        n = write_vocab(path)
        rh = ref.xpref_tok_create(path.encode())
        assert rh, ref.xpref_session_error()
        th = C.c_void_p()
        check(lib().xp_tokenizer_create(path.encode(), C.byref(th)))
        yield ref, rh, th, n
        ref.xpref_tok_destroy(rh)
        lib().xp_tokenizer_destroy(th)


def ours_encode(th, b, bos, eos):
    n = C.c_uint32()
    check(lib().xp_tokenizer_encode(th, b, len(b), bos, eos, None, 0, C.byref(n)))
    out = np.zeros(max(1, n.value), np.int32)
    check(lib().xp_tokenizer_encode(th, b, len(b), bos, eos, out.ctypes.data, len(out), C.byref(n)))
    return out[:n.value]


def ours_decode(th, ids, skip):
    ids = np.ascontiguousarray(ids, np.int32)
    n = C.c_size_t()
    check(lib().xp_tokenizer_decode(th, ids.ctypes.data, len(ids), skip, None, 0, C.byref(n)))
    buf = C.create_string_buffer(n.value + 1)
    check(lib().xp_tokenizer_decode(th, ids.ctypes.data, len(ids), skip, buf, n.value + 1, C.byref(n)))
    return buf.raw[:n.value]


def test_info(both):
    ref, rh, th, n = both
    v, bos, eos, unk, pad = C.c_uint32(), C.c_int32(), C.c_int32(), C.c_int32(), C.c_int32()
    check(lib().xp_tokenizer_info(th, C.byref(v), C.byref(bos), C.byref(eos), C.byref(unk), C.byref(pad)))
    assert (v.value, bos.value, eos.value, unk.value, pad.value) == (n, 2, 1, 3, 0)


@pytest.mark.parametrize("bos,eos", [(0, 0), (1, 0), (1, 1)])
def test_encode_matches_reference(both, bos, eos):
    ref, rh, th, _ = both
    for t in texts():
        b = t.encode()
        want = np.zeros(4 * len(b) + 8, np.int32)
        k = ref.xpref_tok_encode(rh, b, len(b), bos, eos, want.ctypes.data, len(want))
        got = ours_encode(th, b, bos, eos)
        assert list(got) == list(want[:k]), t


@pytest.mark.parametrize("skip", [0, 1])
def test_decode_matches_reference_and_roundtrips(both, skip):
    ref, rh, th, _ = both
    for t in texts(seed=11):
        b = t.encode()
        ids = ours_encode(th, b, 1, 0)
        buf = C.create_string_buffer(8 * len(b) + 64)
        k = ref.xpref_tok_decode(rh, ids.ctypes.data, len(ids), skip, buf, len(buf))
        assert ours_decode(th, ids, skip) == buf.raw[:k], t
        if skip and not any(sp in t for sp in ("<start", "<end_of_turn>", "<unk>")):
            assert ours_decode(th, ids, 1) == b, t  # total: every byte comes back


def test_every_piece_matches_reference(both):
    ref, rh, th, n = both
    buf = C.create_string_buffer(64)
    ob = C.create_string_buffer(64)
    ln = C.c_size_t()
    for i in range(n):
        k = ref.xpref_tok_piece(rh, i, buf, 64)
        check(lib().xp_tokenizer_piece(th, i, ob, 64, C.byref(ln)))
        assert ob.raw[:ln.value] == buf.raw[:k], i
