"""ctypes bindings to the CPU checkers (test infrastructure).

* ``oracle()``  -> oracle/liboracle.so, the C restatement (oracle/xp_oracle.c)
* ``ref()``     -> oracle/_ref/libxpref.so, the reference's own kernels and host
                   engine compiled from source (None when it was not built)
"""
import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_ORACLE = os.path.join(ROOT, "oracle", "liboracle.so")
_REF = os.path.join(ROOT, "oracle", "_ref", "libxpref.so")
# the reference's engine compiled against include/xp (runs on libxp_cuda.so)
_REF_GPU = os.path.join(ROOT, "oracle", "_ref", "libxpref_gpu.so")

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")

_o = None
_r = None


def oracle():
    global _o
    if _o is None:
        lib = C.CDLL(_ORACLE)
        lib.xo_gen_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float, f32p]
        lib.xo_gen_tokens.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint32, u32p]
        lib.xo_uniform.argtypes = [C.c_uint64, C.c_uint64, C.c_uint64]
        lib.xo_uniform.restype = C.c_float
        lib.xo_f32_to_f16.argtypes = [C.c_float]
        lib.xo_f32_to_f16.restype = C.c_uint16
        lib.xo_f16_to_f32.argtypes = [C.c_uint16]
        lib.xo_f16_to_f32.restype = C.c_float
        lib.xo_quantise.argtypes = [C.c_float, C.c_float]
        lib.xo_quantise.restype = C.c_uint32
        lib.xo_best_bf16_scale.argtypes = [f32p, C.c_float]
        lib.xo_best_bf16_scale.restype = C.c_float
        lib.xo_pack_km4bf16.argtypes = [f32p, C.c_uint32, C.c_uint32, u32p, u32p]
        lib.xo_mv_km4_bs.argtypes = [f32p, f32p, u32p, u32p, C.c_uint32, C.c_uint32]
        lib.xo_mv_km4_bs_split.argtypes = [f32p, f32p, u32p, u32p, C.c_uint32, C.c_uint32, C.c_uint32]
        lib.xo_rmsnorm_gemma.argtypes = [f32p, f32p, f32p, C.c_uint32, C.c_uint32, C.c_float]
        lib.xo_rmsnorm_heads_gemma.argtypes = [f32p, f32p, f32p, C.c_uint32, C.c_uint32, C.c_float]
        lib.xo_rope.argtypes = [f32p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]
        lib.xo_geglu.argtypes = [f32p, f32p, f32p, C.c_uint32]
        lib.xo_attention.argtypes = [f32p, f32p, C.c_void_p, C.c_void_p, C.c_int, C.c_uint32,
                                     C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]
        lib.xo_argmax.argtypes = [f32p, C.c_uint32, C.POINTER(C.c_float)]
        lib.xo_argmax.restype = C.c_uint32
        lib.xo_topk.argtypes = [f32p, C.c_uint32, C.c_uint32, f32p, u32p]
        lib.xo_topk.restype = C.c_uint32
        lib.xo_sample.argtypes = [f32p, C.c_uint32, C.c_float, C.c_uint32, C.c_float, C.c_float]
        lib.xo_sample.restype = C.c_uint32
        u32 = C.c_uint32
        lib.xo_softmax_rows_stats.argtypes = [f32p, f32p, u32, u32]
        lib.xo_softmax_rows_apply.argtypes = [f32p, f32p, u32, u32]
        lib.xo_attention_scores_prefill.argtypes = [f32p, f32p, f32p] + [u32] * 7 + [C.c_float]
        lib.xo_attention_apply_prefill.argtypes = [f32p, f32p, f32p] + [u32] * 5
        lib.xo_rmsnorm_rows_sumsq.argtypes = [f32p, f32p, u32, u32]
        lib.xo_rmsnorm_rows_apply_gemma.argtypes = [f32p, f32p, f32p, f32p, u32, u32, C.c_float]
        lib.xo_rmsnorm_heads_rows_gemma.argtypes = [f32p, f32p, f32p, u32, u32, u32, C.c_float]
        lib.xo_rope_prefill.argtypes = [f32p, u32, u32, u32, u32, C.c_float]
        lib.xo_kv_append_rows.argtypes = [f32p, f32p, u32, u32, u32]
        lib.xo_embed_lookup_rows.argtypes = [f32p, f32p, u32p, u32, u32]
        _o = lib
    return _o


class _Arg(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("size", C.c_uint32), ("is_buffer", C.c_int)]


_rg = None


def ref_gpu():
    """The reference engine built on the B200 library (oracle/_ref/libxpref_gpu.so),
    or None if it was not built."""
    global _rg
    if _rg is None:
        if not os.path.exists(_REF_GPU):
            return None
        _rg = _configure(C.CDLL(_REF_GPU), kernels=False)
    return _rg


def ref():
    """The reference build, or None if oracle/_ref was not built."""
    global _r
    if _r is None:
        if not os.path.exists(_REF):
            return None
        _r = _configure(C.CDLL(_REF), kernels=True)
    return _r


def _configure(lib, kernels):
    if kernels:
        lib.xpref_launch.argtypes = [C.c_char_p, C.c_char_p, C.c_uint32, C.POINTER(_Arg), C.c_uint32, C.c_int]
        lib.xpref_last_error.restype = C.c_char_p
    # session and packer entry points (both builds)
    if True:
        lib.xpref_pack_km4bf16.argtypes = [f32p, C.c_uint32, C.c_uint32, u32p, u32p, C.c_void_p]
        lib.xpref_best_bf16_scale.argtypes = [f32p, C.c_float]
        lib.xpref_best_bf16_scale.restype = C.c_float
        lib.xpref_plan_weight_bytes.restype = C.c_uint64
        lib.xpref_plan_dispatches.restype = C.c_uint32
        lib.xpref_session_create.argtypes = [C.c_char_p, C.c_char_p, C.c_uint32, C.c_int, C.c_float,
                                             C.c_uint32, C.c_float, C.c_uint64, C.c_uint32]
        lib.xpref_session_create.restype = C.c_void_p
        lib.xpref_session_error.restype = C.c_char_p
        lib.xpref_session_destroy.argtypes = [C.c_void_p]
        lib.xpref_session_prefill.argtypes = [C.c_void_p, u32p, C.c_uint32]
        lib.xpref_session_step.argtypes = [C.c_void_p]
        lib.xpref_session_step.restype = C.c_int64
        lib.xpref_session_logits.argtypes = [C.c_void_p, f32p, C.c_uint32]
        lib.xpref_session_position.argtypes = [C.c_void_p]
        lib.xpref_session_position.restype = C.c_uint32
    return lib


def ref_launch(name, grid, *args, module=None, threads=0):
    """Run one reference kernel over `grid` work items. numpy arrays are
    buffers (modified in place); Python ints are uint32, floats fp32, and
    (value, ctype) tuples give an explicit POD type."""
    lib = ref()
    keep = []
    arr = (_Arg * max(1, len(args)))()
    for i, a in enumerate(args):
        if isinstance(a, np.ndarray):
            assert a.flags.c_contiguous
            arr[i] = _Arg(a.ctypes.data, 0, 1)
            keep.append(a)
        else:
            if isinstance(a, tuple):
                v = a[1](a[0])
            elif isinstance(a, float):
                v = C.c_float(a)
            else:
                v = C.c_uint32(a)
            keep.append(v)
            arr[i] = _Arg(C.addressof(v), C.sizeof(v), 0)
    rc = lib.xpref_launch(module.encode() if module else None, name.encode(), grid, arr, len(args), threads)
    if rc != 0:
        raise RuntimeError(f"ref kernel {name}: {lib.xpref_last_error().decode()}")


def gen_normal(seed, stream, n, sigma, offset=0):
    out = np.empty(n, np.float32)
    oracle().xo_gen_normal(seed, stream, offset, n, sigma, out)
    return out


def gen_tokens(seed, stream, n, vocab):
    out = np.empty(n, np.uint32)
    oracle().xo_gen_tokens(seed, stream, n, vocab, out)
    return out


def pack(w_cols_rows, rows, cols, impl="oracle"):
    """fp32 [cols][rows] -> (words uint32[cols*rows/8], scales uint32[cols*rows/64])."""
    w = np.ascontiguousarray(w_cols_rows, np.float32).reshape(-1)
    words = np.zeros(cols * rows // 8, np.uint32)
    scales = np.zeros(cols * rows // 64, np.uint32)
    if impl == "oracle":
        rc = oracle().xo_pack_km4bf16(w, rows, cols, words, scales)
    else:
        rc = ref().xpref_pack_km4bf16(w, rows, cols, words, scales, None)
    assert rc == 0
    return words, scales


def mv(x, words, scales, rows, cols, split=1):
    out = np.empty(cols, np.float32)
    if split > 1:
        oracle().xo_mv_km4_bs_split(out, np.ascontiguousarray(x, np.float32), words, scales, rows, cols, split)
    else:
        oracle().xo_mv_km4_bs(out, np.ascontiguousarray(x, np.float32), words, scales, rows, cols)
    return out


# ---- whole-model oracle (xo_forward) -----------------------------------------
class XoQW(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("cols", C.c_uint32), ("wq", C.c_void_p), ("sc", C.c_void_p)]


class XoLayer(C.Structure):
    _fields_ = [(n, XoQW) for n in ("wq", "wk", "wv", "wo", "gate", "up", "down")] + \
               [(n, C.c_void_p) for n in ("attn_norm", "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm",
                                          "k_norm")]


class XoModel(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "hidden", "ffn", "n_heads", "n_kv_heads", "head_dim", "vocab",
                                          "max_seq", "sliding_window", "global_every", "norm_parts")] + \
               [(n, C.c_float) for n in ("rms_eps", "theta_global", "theta_local", "embed_scale", "attn_scale")] + \
               [("kv_fp16", C.c_int), ("layers", C.POINTER(XoLayer)), ("lm_head", XoQW),
                ("final_norm", C.c_void_p), ("embed", C.c_void_p)]


class XoState(C.Structure):
    _fields_ = [("kcache", C.POINTER(C.c_void_p)), ("vcache", C.POINTER(C.c_void_p))]


def tensor_stream(layer, which):
    """Same stream ids as xp_session_tensor_stream (engine random init)."""
    return 0x1000 + layer * 32 + which


def _roundtrip(w):
    """Norm offsets as a GGUF file carries them: stored (1 + w), loaded back
    as (1 + w) - 1 (examples/llm/decode.cpp:1490-1502), both in fp32."""
    return ((np.float32(1.0) + w.astype(np.float32)).astype(np.float32) - np.float32(1.0)).astype(np.float32)


class OracleModel:
    """Random-init model built exactly as xp_session_create_random builds it
    (same generator, same stream ids, same packer), run by xo_forward."""

    def __init__(self, cfg, seed, kv_fp16=True, norm_roundtrip=False):
        o = oracle()
        o.xo_forward.argtypes = [C.POINTER(XoModel), C.POINTER(XoState), C.c_uint32, C.c_uint32, C.c_void_p]
        self.cfg = cfg
        self.seed = seed
        self.keep = []
        H, V = cfg.hidden, cfg.vocab
        L = (XoLayer * cfg.n_layers)()
        self.layers_np = []
        for l in range(cfg.n_layers):
            lw = {"words": [], "scales": []}
            for m, (rows, cols) in enumerate(cfg.matrix_shapes()):
                w = gen_normal(seed, tensor_stream(l, m), rows * cols, 0.02)
                words, scales = pack(w, rows, cols)
                lw["words"].append(words)
                lw["scales"].append(scales)
                q = XoQW(rows, cols, words.ctypes.data, scales.ctypes.data)
                setattr(L[l], ("wq", "wk", "wv", "wo", "gate", "up", "down")[m], q)
            names = ("attn_norm", "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm", "k_norm")
            for n, name in enumerate(names):
                v = gen_normal(seed, tensor_stream(l, 7 + n), H if n < 4 else cfg.head_dim, 0.02)
                if norm_roundtrip:
                    v = _roundtrip(v)
                lw[name] = v
                setattr(L[l], name, v.ctypes.data)
            self.layers_np.append(lw)
        self.embed = gen_normal(seed, tensor_stream(cfg.n_layers, 0), V * H, 0.02)
        self.lm_words, self.lm_scales = pack(self.embed, H, V)
        self.final_norm = gen_normal(seed, tensor_stream(cfg.n_layers, 7), H, 0.02)
        if norm_roundtrip:
            self.final_norm = _roundtrip(self.final_norm)
        m = XoModel()
        for n in ("n_layers", "hidden", "ffn", "n_heads", "n_kv_heads", "head_dim", "vocab", "max_seq",
                  "sliding_window", "global_every"):
            setattr(m, n, getattr(cfg, n))
        m.norm_parts = 64
        m.rms_eps, m.theta_global, m.theta_local = cfg.rms_eps, cfg.rope_theta_global, cfg.rope_theta_local
        m.embed_scale = cfg.embed_scale or float(np.float32(np.sqrt(np.float32(H))))
        m.attn_scale = cfg.attn_scale or float(np.float32(1.0) / np.sqrt(np.float32(cfg.head_dim)))
        m.kv_fp16 = int(kv_fp16)
        m.layers = L
        m.lm_head = XoQW(H, V, self.lm_words.ctypes.data, self.lm_scales.ctypes.data)
        m.final_norm = self.final_norm.ctypes.data
        m.embed = self.embed.ctypes.data
        self.model = m
        self.L = L
        kvd = cfg.n_kv_heads * cfg.head_dim
        dt = np.uint16 if kv_fp16 else np.float32
        self.kc = [np.zeros(cfg.max_seq * kvd, dt) for _ in range(cfg.n_layers)]
        self.vc = [np.zeros(cfg.max_seq * kvd, dt) for _ in range(cfg.n_layers)]
        kp = (C.c_void_p * cfg.n_layers)(*[a.ctypes.data for a in self.kc])
        vp = (C.c_void_p * cfg.n_layers)(*[a.ctypes.data for a in self.vc])
        self.state = XoState(C.cast(kp, C.POINTER(C.c_void_p)), C.cast(vp, C.POINTER(C.c_void_p)))
        self.keep += [kp, vp]

    def weights_dict(self):
        """The packed weights in the layout DecodeSession.from_weights takes."""
        return {"layers": self.layers_np, "lm_words": self.lm_words, "lm_scales": self.lm_scales,
                "final_norm": self.final_norm, "embed": self.embed}

    def forward(self, token, pos, want_logits=True):
        out = np.empty(self.cfg.vocab, np.float32) if want_logits else None
        rc = oracle().xo_forward(C.byref(self.model), C.byref(self.state), token, pos,
                                 out.ctypes.data if want_logits else None)
        assert rc == 0
        return out


def write_model_gguf(om, path, window=512):
    """The OracleModel's fp32 master weights as a Gemma-3 GGUF the reference
    engine loads (norms stored as 1 + w, tied output head)."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    from gguf_writer import gemma3_meta, write_gguf
    cfg = om.cfg
    seed = om.seed
    H = cfg.hidden
    names = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
    norm_names = ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm", "attn_q_norm", "attn_k_norm")
    keys = ("attn_norm", "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm", "k_norm")
    tensors = [("token_embd.weight", (H, cfg.vocab), om.embed)]
    for l in range(cfg.n_layers):
        for m, (rows, cols) in enumerate(cfg.matrix_shapes()):
            w = gen_normal(seed, tensor_stream(l, m), rows * cols, 0.02)
            tensors.append((f"blk.{l}.{names[m]}.weight", (rows, cols), w))
        for n in range(6):
            v = om.layers_np[l][keys[n]]
            tensors.append((f"blk.{l}.{norm_names[n]}.weight", (len(v),), np.float32(1.0) + v))
    tensors.append(("output_norm.weight", (H,), np.float32(1.0) + om.final_norm))
    write_gguf(path, gemma3_meta(cfg, cfg.rope_theta_global, window), tensors)


def write_random_gguf(cfg, seed, path, window=512):
    """The same seeded model as OracleModel(cfg, seed) written as a Gemma-3
    GGUF one tensor at a time (a full-size model is 4 GB of fp32), for timing
    the reference engine without holding the model twice in host memory."""
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
    from gguf_writer import gemma3_meta, write_gguf
    H = cfg.hidden
    names = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
    norm_names = ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm", "attn_q_norm", "attn_k_norm")

    def normal(stream, n):
        return lambda: gen_normal(seed, stream, n, 0.02)

    def norm(stream, n):
        return lambda: np.float32(1.0) + gen_normal(seed, stream, n, 0.02)

    tensors = [("token_embd.weight", (H, cfg.vocab), normal(tensor_stream(cfg.n_layers, 0), cfg.vocab * H))]
    for l in range(cfg.n_layers):
        for m, (rows, cols) in enumerate(cfg.matrix_shapes()):
            tensors.append((f"blk.{l}.{names[m]}.weight", (rows, cols), normal(tensor_stream(l, m), rows * cols)))
        for n in range(6):
            d = H if n < 4 else cfg.head_dim
            tensors.append((f"blk.{l}.{norm_names[n]}.weight", (d,), norm(tensor_stream(l, 7 + n), d)))
    tensors.append(("output_norm.weight", (H,), norm(tensor_stream(cfg.n_layers, 7), H)))
    write_gguf(path, gemma3_meta(cfg, cfg.rope_theta_global, window), tensors)


class RefSession:
    """The reference DecodeSession (examples/llm/decode.cpp) running on the CPU
    stand-in runtime over the reference kernels, from a GGUF file."""

    def __init__(self, gguf_path, max_seq, global_every, greedy=True, lib=None):
        self.lib = lib or ref()
        self.h = self.lib.xpref_session_create(gguf_path.encode(), b"kernels", max_seq, int(greedy), 1.0, 0, 1.0,
                                               1234, global_every)
        if not self.h:
            raise RuntimeError(self.lib.xpref_session_error().decode())

    def prefill(self, toks):
        t = np.ascontiguousarray(toks, np.uint32)
        assert self.lib.xpref_session_prefill(self.h, t, len(t)) == 0, self.lib.xpref_session_error()

    def decode_step(self):
        r = self.lib.xpref_session_step(self.h)
        assert r >= 0, self.lib.xpref_session_error()
        return int(r)

    def logits(self, n):
        out = np.empty(n, np.float32)
        assert self.lib.xpref_session_logits(self.h, out, n) == 0
        return out

    def close(self):
        if self.h:
            self.lib.xpref_session_destroy(self.h)
            self.h = None
