"""Minimal GGUF v3 writer for the test models (F32 tensors, scalar/string/
array metadata). Written from the published GGUF layout: little-endian header
("GGUF", version, tensor count, kv count), key/value pairs, tensor infos
(name, n_dims, dims fastest-first, ggml type, offset), then the data blob
aligned to `general.alignment` (32)."""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
ALIGN = 32


def _s(b):
    b = b.encode() if isinstance(b, str) else b
    return struct.pack("<Q", len(b)) + b


def _val(t, v):
    if t == U32:
        return struct.pack("<I", v)
    if t == I32:
        return struct.pack("<i", v)
    if t == U64:
        return struct.pack("<Q", v)
    if t == F32:
        return struct.pack("<f", v)
    if t == BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == STR:
        return _s(v)
    raise ValueError(t)


def write_gguf(path, meta, tensors):
    """meta: list of (key, type, value) or (key, ARR, (elem_type, values)).
    tensors: list of (name, shape_fastest_first, float32 array in row-major
    order of the reversed shape); the array may instead be a callable that
    returns it, so a large model is generated one tensor at a time, or a
    ("raw", ggml_type, bytes) tuple holding the tensor already encoded."""
    out = bytearray()
    out += struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta))
    for key, t, v in meta:
        out += _s(key) + struct.pack("<I", t)
        if t == ARR:
            et, vals = v
            out += struct.pack("<IQ", et, len(vals))
            for x in vals:
                out += _val(et, x)
        else:
            out += _val(t, v)
    offs = []
    off = 0
    for name, shape, arr in tensors:
        raw = isinstance(arr, tuple)
        nbytes = len(arr[2]) if raw else 4 * int(np.prod(shape))
        if not raw and not callable(arr):
            assert np.asarray(arr).size * 4 == nbytes
        offs.append(off)
        out += _s(name) + struct.pack("<I", len(shape))
        for d in shape:
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", arr[1] if raw else 0, off)  # ggml type (0 = F32)
        off += (nbytes + ALIGN - 1) // ALIGN * ALIGN
    pad = (-len(out)) % ALIGN
    out += b"\0" * pad
    with open(path, "wb") as f:
        f.write(out)
        for (name, shape, arr), o in zip(tensors, offs):
            if isinstance(arr, tuple):
                b = arr[2]
            else:
                a = np.ascontiguousarray(arr() if callable(arr) else arr, np.float32)
                assert a.nbytes == 4 * int(np.prod(shape))
                b = a.tobytes()
            f.write(b)
            f.write(b"\0" * ((-len(b)) % ALIGN))


def gemma3_meta(cfg, rope_base, window):
    return [
        ("general.architecture", STR, "gemma3"),
        ("general.name", STR, "xpose-b200 test model"),
        ("general.alignment", U32, ALIGN),
        ("gemma3.block_count", U32, cfg.n_layers),
        ("gemma3.embedding_length", U32, cfg.hidden),
        ("gemma3.feed_forward_length", U32, cfg.ffn),
        ("gemma3.attention.head_count", U32, cfg.n_heads),
        ("gemma3.attention.head_count_kv", U32, cfg.n_kv_heads),
        ("gemma3.attention.key_length", U32, cfg.head_dim),
        ("gemma3.attention.value_length", U32, cfg.head_dim),
        ("gemma3.context_length", U32, cfg.max_seq),
        ("gemma3.attention.sliding_window", U32, window),
        ("gemma3.rope.freq_base", F32, rope_base),
        ("gemma3.attention.layer_norm_rms_epsilon", F32, cfg.rms_eps),
        ("tokenizer.ggml.model", STR, "llama"),
        ("tokenizer.ggml.tokens", ARR, (STR, [f"<t{i}>" for i in range(cfg.vocab)])),
    ]
