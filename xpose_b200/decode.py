"""DecodeSession over the C ABI (examples/llm/decode.hpp:605-676 surface).

    cfg  = DecodeConfig.gemma3_1b()
    sess = DecodeSession.random(cfg, Sampling(), seed=0)   # random-init weights
    sess.prefill(prompt_ids)
    tok  = sess.decode_step()
"""
import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from ._lib import LayerWeights, ModelConfig, Sampling as _CSampling, check, lib


@dataclass
class Sampling:
    """examples/llm/decode.hpp:158-202 (mode, temperature, top_k, top_p, seed)."""
    greedy: bool = True
    temperature: float = 1.0
    top_k: int = 64
    top_p: float = 1.0
    seed: int = 1234
    seq_id: int = 0

    def _c(self):
        return _CSampling(int(self.greedy), self.temperature, self.top_k, self.top_p, self.seed, self.seq_id)


@dataclass
class DecodeConfig:
    """examples/llm/decode.hpp:204-356; defaults are Gemma 3 1B."""
    n_layers: int = 26
    hidden: int = 1152
    ffn: int = 6912
    n_heads: int = 4
    n_kv_heads: int = 1
    head_dim: int = 256
    vocab: int = 262144
    max_seq: int = 8192
    sliding_window: int = 512
    global_every: int = 6
    rms_eps: float = 1e-6
    rope_theta_global: float = 1e6
    rope_theta_local: float = 1e4
    embed_scale: float = 0.0
    attn_scale: float = 0.0

    @staticmethod
    def gemma3_1b():
        return DecodeConfig()

    def layer_is_global(self, layer):
        return self.global_every == 0 or (layer + 1) % self.global_every == 0

    def attn_kv_start(self, layer, seq_len):
        w = 0 if self.layer_is_global(layer) else self.sliding_window
        return 0 if (w == 0 or seq_len <= w) else seq_len - w

    def matrix_shapes(self):
        """(rows=K, cols=N) of q, k, v, o, gate, up, down."""
        H, F, QD, KVD = self.hidden, self.ffn, self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        return [(H, QD), (H, KVD), (H, KVD), (QD, H), (H, F), (H, F), (F, H)]

    def weight_bytes(self):
        """Nibbles + bf16 scales per token (examples/llm/decode.cpp:288-348)."""
        per_layer = sum(r * c // 2 + r * c // 16 for r, c in self.matrix_shapes())
        return per_layer * self.n_layers + self.hidden * self.vocab // 2 + self.hidden * self.vocab // 16

    def _c(self):
        return ModelConfig(self.n_layers, self.hidden, self.ffn, self.n_heads, self.n_kv_heads, self.head_dim,
                           self.vocab, self.max_seq, self.sliding_window, self.global_every, self.rms_eps,
                           self.rope_theta_global, self.rope_theta_local, self.embed_scale, self.attn_scale)


# trace buffer layout of the token kernel (u64 words)
TRACE_CTA, TRACE_MAXBAR, TRACE_MAXCTA = 512 + 8 * 1024, 160, 160
TRACE_WORDS = TRACE_CTA + 2 * TRACE_MAXBAR * TRACE_MAXCTA


def tensor_stream(layer, which):
    return lib().xp_session_tensor_stream(layer, which)


class DecodeSession:
    def __init__(self, handle, cfg, sampling):
        self._h = handle
        self.cfg = cfg
        self.sampling = sampling

    @staticmethod
    def random(cfg, sampling=None, seed=0, device=0):
        sampling = sampling or Sampling()
        h = C.c_void_p()
        c, s = cfg._c(), sampling._c()
        check(lib().xp_session_create_random(device, C.byref(c), C.byref(s), seed, C.byref(h)))
        return DecodeSession(h, cfg, sampling)

    @staticmethod
    def from_gguf(path, sampling=None, max_seq=8192, global_every=6, pack_cache=None, device=0, policy=None):
        """A session from a GGUF model file (C ABI xp_session_create_gguf):
        shapes from the file, max_seq / global_every (or a whole DecodeConfig
        `policy`) from the caller. pack_cache: None = "<path>.xpack", "" = no
        cache, else the cache path."""
        sampling = sampling or Sampling()
        pol = policy or DecodeConfig(max_seq=max_seq, global_every=global_every, sliding_window=0)
        h = C.c_void_p()
        c, s = pol._c(), sampling._c()
        pc = None if pack_cache is None else pack_cache.encode()
        check(lib().xp_session_create_gguf(device, path.encode(), C.byref(c), C.byref(s), pc, C.byref(h)))
        got = ModelConfig()
        check(lib().xp_session_config(h, C.byref(got)))
        cfg = DecodeConfig(got.n_layers, got.hidden, got.ffn, got.n_heads, got.n_kv_heads, got.head_dim, got.vocab,
                           got.max_seq, got.sliding_window, got.global_every, got.rms_eps, got.rope_theta_global,
                           got.rope_theta_local, got.embed_scale, got.attn_scale)
        return DecodeSession(h, cfg, sampling)

    def load_info(self):
        """(loaded from the cache, wrote the cache, description) of a GGUF session."""
        fc, cw = C.c_int(), C.c_int()
        buf = C.create_string_buffer(512)
        check(lib().xp_session_load_info(self._h, C.byref(fc), C.byref(cw), buf, 512))
        return bool(fc.value), bool(cw.value), buf.value.decode()

    @staticmethod
    def from_weights(cfg, weights, sampling=None, device=0):
        """weights: dict with 'layers' (list of dicts: words[7], scales[7], norms
        attn/post_attn/ffn/post_ffn/q/k), 'lm_words', 'lm_scales', 'final_norm',
        'embed' -- numpy arrays in the reference's packed layouts."""
        sampling = sampling or Sampling()
        keep = []

        def p(a):
            a = np.ascontiguousarray(a)
            keep.append(a)
            return a.ctypes.data

        L = (LayerWeights * cfg.n_layers)()
        for i, lw in enumerate(weights["layers"]):
            for m in range(7):
                L[i].words[m] = p(lw["words"][m])
                L[i].scales[m] = p(lw["scales"][m])
            L[i].attn_norm, L[i].post_attn_norm = p(lw["attn_norm"]), p(lw["post_attn_norm"])
            L[i].ffn_norm, L[i].post_ffn_norm = p(lw["ffn_norm"]), p(lw["post_ffn_norm"])
            L[i].q_norm, L[i].k_norm = p(lw["q_norm"]), p(lw["k_norm"])
        h = C.c_void_p()
        c, s = cfg._c(), sampling._c()
        check(lib().xp_session_create(device, C.byref(c), C.byref(s), L, p(weights["lm_words"]),
                                      p(weights["lm_scales"]), p(weights["final_norm"]), p(weights["embed"]),
                                      C.byref(h)))
        return DecodeSession(h, cfg, sampling)

    def prefill(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        check(lib().xp_session_prefill(self._h, t.ctypes.data, len(t)))

    def decode_step(self):
        t = C.c_uint32()
        check(lib().xp_session_decode_step(self._h, C.byref(t)))
        return t.value

    def generate(self, n, want_tokens=True):
        """n device-resident steps; returns (tokens or None, device ms)."""
        ms = C.c_float()
        toks = np.zeros(max(1, n), np.uint32) if want_tokens else None
        check(lib().xp_session_generate(self._h, n, toks.ctypes.data if want_tokens else None, C.byref(ms)))
        return (toks[:n] if want_tokens else None), ms.value

    def reset(self):
        check(lib().xp_session_reset(self._h))

    def position(self):
        p = C.c_uint32()
        check(lib().xp_session_position(self._h, C.byref(p)))
        return p.value

    def last_logits(self):
        out = np.empty(self.cfg.vocab, np.float32)
        check(lib().xp_session_logits(self._h, out.ctypes.data, self.cfg.vocab))
        return out

    def stats(self):
        k, w = C.c_uint32(), C.c_uint64()
        check(lib().xp_session_stats(self._h, C.byref(k), C.byref(w)))
        return {"kernels_per_token": k.value, "weight_bytes": w.value}

    def debug_ptr(self, name):
        d, b = C.c_void_p(), C.c_size_t()
        check(lib().xp_session_debug_ptr(self._h, name.encode(), C.byref(d), C.byref(b)))
        return d.value, b.value

    def profile_matvec(self, iters=20):
        """(ms, algorithmic bytes, launches) of the token's int4 matvecs
        (26 layers x q, k, v, o, gate, up, down + LM head, on this session's
        packed planes) run alone as one streaming plan."""
        ms, b, n = C.c_float(), C.c_uint64(), C.c_uint32()
        check(lib().xp_session_profile_matvec(self._h, iters, C.byref(ms), C.byref(b), C.byref(n)))
        return ms.value, b.value, n.value

    def timer_start(self):
        check(lib().xp_session_timer(self._h, 0, None))

    def timer_stop(self):
        ms = C.c_float()
        check(lib().xp_session_timer(self._h, 1, C.byref(ms)))
        return ms.value

    def trace(self):
        """Phase timeline of the last token (XP_TRACE=1): list of
        (arrive_ns, leave_ns) per grid barrier, relative to kernel start."""
        buf = np.zeros(TRACE_WORDS, np.uint64)
        check(lib().xp_session_trace(self._h, buf.ctypes.data, len(buf)))
        nb = int(buf[0])
        t0 = int(buf[1])
        bars = [(int(buf[2 * k]) - t0, int(buf[2 * k + 1]) - t0) for k in range(1, nb + 1)]
        marks = [[(int(buf[512 + k * 8 + j]) - t0) if buf[512 + k * 8 + j] else None for j in range(8)]
                 for k in range(nb + 1)]
        return bars, int(buf[2 * nb + 2]) - t0, marks

    def trace_ctas(self):
        """Per-CTA (arrive_ns, leave_ns) of every grid barrier of the last
        token (XP_TRACE=1), relative to kernel start: array [ctas, barriers, 2]."""
        buf = np.zeros(TRACE_WORDS, np.uint64)
        check(lib().xp_session_trace(self._h, buf.ctypes.data, len(buf)))
        nb, t0 = int(buf[0]), int(buf[1])
        per = buf[TRACE_CTA:].reshape(TRACE_MAXCTA, TRACE_MAXBAR, 2)[:, 1:nb + 1].astype(np.int64)
        per = per[per[:, 0, 0] != 0]
        return per - t0

    def tp_handle(self):
        """64-byte IPC handle of this session's LM-head exchange buffer."""
        buf = (C.c_ubyte * 64)()
        check(lib().xp_session_tp_handle(self._h, buf))
        return bytes(buf)

    def tp_attach(self, rank, world, handles, shard_ffn=False):
        """Shard the LM head (and with shard_ffn the FFN) over `world` ranks
        (handles in rank order)."""
        blob = b"".join(handles)
        assert len(blob) == 64 * world
        check(lib().xp_session_tp_attach_ex(self._h, rank, world, blob, 1 if shard_ffn else 0))

    def error_word(self):
        w = C.c_uint32()
        check(lib().xp_session_error_word(self._h, C.byref(w)))
        return w.value

    def close(self):
        if self._h:
            lib().xp_session_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class BatchDecode:
    """nseq independent sequences decoded together over a DecodeSession's
    weights (C ABI xp_bdec_*): tensor-core int4 matvecs for all sequences at
    once, per-sequence attention and sampling. Sequence b samples with the
    uniforms of seq_id = seq0 + b, as a DecodeSession with that seq_id would."""

    def __init__(self, session, nseq, max_seq, sampling=None, seq0=0):
        self.session = session  # keeps the weights alive
        self.nseq = nseq
        self.vocab = session.cfg.vocab
        sp = (sampling or Sampling())._c()
        h = C.c_void_p()
        check(lib().xp_bdec_create(session._h, nseq, max_seq, C.byref(sp), seq0, C.byref(h)))
        self._h = h

    def prefill(self, tokens):
        """tokens: [nseq][n] (one prompt per sequence, equal lengths)."""
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32).T)
        check(lib().xp_bdec_prefill(self._h, t.ctypes.data, t.shape[0]))

    def step(self):
        out = np.zeros(self.nseq, np.uint32)
        check(lib().xp_bdec_step(self._h, out.ctypes.data))
        return out

    def generate(self, n):
        ms = C.c_float()
        check(lib().xp_bdec_generate(self._h, n, C.byref(ms)))
        return ms.value

    def logits(self):
        out = np.empty((self.nseq, self.vocab), np.float32)
        check(lib().xp_bdec_logits(self._h, out.ctypes.data, out.size))
        return out

    def position(self):
        p = C.c_uint32()
        check(lib().xp_bdec_position(self._h, C.byref(p)))
        return p.value

    def close(self):
        if self._h:
            lib().xp_bdec_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
