"""ctypes binding of libxp_cuda.so (include/xp_cuda.h).

The library is the product path: there is no fallback. Loading fails loudly if
the in-tree shared object is missing; every call that returns an error raises
XpError with the library's message (the reference raises vulkore::Error with
the same wording, include/vulkore/check.hpp:16-25).
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libxp_cuda.so")

XP_OK = 0
XP_TIMEOUT = 1
STATUS = {
    0: "XP_OK", 1: "XP_TIMEOUT", -1: "XP_ERR_INVALID", -2: "XP_ERR_NO_KERNEL", -3: "XP_ERR_ARITY",
    -4: "XP_ERR_ARG_KIND", -5: "XP_ERR_ARG_SIZE", -6: "XP_ERR_GRID", -7: "XP_ERR_CUDA", -8: "XP_ERR_OOM",
    -9: "XP_ERR_KV_FULL", -10: "XP_ERR_STATE", -11: "XP_ERR_DEVICE", -12: "XP_ERR_NO_DEVICE",
    -13: "XP_ERR_UNSUPPORTED",
}


class XpError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status
        self.name = STATUS.get(status, str(status))


class Grid(C.Structure):
    _fields_ = [("x", C.c_uint32), ("y", C.c_uint32), ("z", C.c_uint32)]


class Arg(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("size", C.c_uint32), ("kind", C.c_int32)]


class ModelConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "hidden", "ffn", "n_heads", "n_kv_heads", "head_dim",
                                          "vocab", "max_seq", "sliding_window", "global_every")] + \
               [(n, C.c_float) for n in ("rms_eps", "rope_theta_global", "rope_theta_local", "embed_scale",
                                         "attn_scale")]


class Sampling(C.Structure):
    _fields_ = [("greedy", C.c_int), ("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float),
                ("seed", C.c_uint64), ("seq_id", C.c_uint64)]


class LayerWeights(C.Structure):
    _fields_ = [("words", C.c_void_p * 7), ("scales", C.c_void_p * 7)] + \
               [(n, C.c_void_p) for n in ("attn_norm", "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm",
                                          "k_norm")]


_lib = None

_SIGS = {
    "xp_last_error": (C.c_char_p, []),
    "xp_status_name": (C.c_char_p, [C.c_int]),
    "xp_version": (C.c_char_p, []),
    "xp_device_count": (C.c_int, []),
    "xp_context_create": (C.c_int, [C.c_int, C.POINTER(C.c_void_p)]),
    "xp_context_destroy": (C.c_int, [C.c_void_p]),
    "xp_context_stream": (C.c_void_p, [C.c_void_p]),
    "xp_context_device_name": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t]),
    "xp_context_wait_idle": (C.c_int, [C.c_void_p]),
    "xp_alloc": (C.c_int, [C.c_void_p, C.c_size_t, C.c_int, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "xp_free": (C.c_int, [C.c_void_p, C.c_void_p]),
    "xp_upload": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]),
    "xp_download": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t]),
    "xp_kernel_lookup": (C.c_int, [C.c_char_p, C.c_char_p, C.POINTER(C.c_int32)]),
    "xp_kernel_info": (C.c_int, [C.c_int32, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p), C.POINTER(C.c_uint32)]),
    "xp_kernel_arg": (C.c_int, [C.c_int32, C.c_uint32, C.POINTER(C.c_int), C.POINTER(C.c_uint32),
                                C.POINTER(C.c_char_p)]),
    "xp_kernel_count": (C.c_int, []),
    "xp_launch": (C.c_int, [C.c_int32, Grid, C.POINTER(Arg), C.c_uint32, C.c_void_p]),
    "xp_batch_create": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "xp_batch_add": (C.c_int, [C.c_void_p, C.c_int32, Grid, C.POINTER(Arg), C.c_uint32]),
    "xp_batch_size": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "xp_batch_submit": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "xp_batch_destroy": (C.c_int, [C.c_void_p]),
    "xp_context_fence": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "xp_fence_wait": (C.c_int, [C.c_void_p, C.c_uint64]),
    "xp_fence_destroy": (C.c_int, [C.c_void_p]),
    "xp_mv_km4_bs": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_uint32] * 2),
    "xp_mv_km4_bs_split": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_uint32] * 3),
    "xp_mv_reduce": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    "xp_mv_km4_bs_batch_scratch_bytes": (C.c_size_t, [C.c_uint32, C.c_uint32, C.c_uint32]),
    "xp_mv_km4_bs_batch": (C.c_int, [C.c_void_p] * 5 + [C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]),
    "xp_selftest_wait_timeout": (C.c_int, [C.c_uint32, C.POINTER(C.c_uint32)]),
    "xp_session_tp_handle": (C.c_int, [C.c_void_p, C.c_void_p]),
    "xp_session_tp_attach": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "xp_session_tp_attach_ex": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_uint32]),
    "xp_bdec_create": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(Sampling), C.c_uint64,
                                 C.POINTER(C.c_void_p)]),
    "xp_bdec_prefill": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "xp_bdec_step": (C.c_int, [C.c_void_p, C.c_void_p]),
    "xp_bdec_generate": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_float)]),
    "xp_bdec_logits": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "xp_bdec_position": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "xp_bdec_destroy": (None, [C.c_void_p]),
    "xp_mv_plan_create": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p)]),
    "xp_mv_plan_run": (C.c_int, [C.c_void_p, C.c_void_p]),
    "xp_mv_plan_bytes": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint64)]),
    "xp_mv_plan_destroy": (None, [C.c_void_p]),
    "xp_rmsnorm_sumsq": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    "xp_rmsnorm_apply_gemma": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_uint32] * 2 + [C.c_float]),
    "xp_rmsnorm_heads_gemma": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_uint32] * 2 + [C.c_float]),
    "xp_rope": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint32, C.c_float]),
    "xp_geglu": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_uint32]),
    "xp_add_residual": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32]),
    "xp_kv_append": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    "xp_attention_scores": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_uint32] * 4 + [C.c_float, C.c_uint32]),
    "xp_softmax_rows": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    "xp_attention_apply": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_uint32] * 5),
    "xp_argmax": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_uint32]),
    "xp_topk4_partial": (C.c_int, [C.c_void_p] + [C.c_void_p] * 3 + [C.c_uint32] * 2),
    "xp_attention_scratch_bytes": (C.c_size_t, [C.c_uint32]),
    "xp_attention_decode": (C.c_int, [C.c_void_p] + [C.c_void_p] * 9 + [C.c_uint32, C.c_float, C.c_float, C.c_float,
                                                                        C.c_uint32, C.c_uint32, C.c_void_p]),
    "xp_attention_decode_static": (C.c_int, [C.c_void_p] + [C.c_void_p] * 9 + [C.c_uint32, C.c_float, C.c_float,
                                                                               C.c_float, C.c_uint32, C.c_uint32]),
    "xp_attention_static_error_word": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.c_int]),
    "xp_sample_scratch_bytes": (C.c_size_t, [C.c_uint32]),
    "xp_sample_topk": (C.c_int, [C.c_void_p] + [C.c_void_p] * 4 + [C.c_uint32, C.c_uint32, C.c_float, C.c_float,
                                                                   C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p]),
    "xp_pack_km4bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p, C.c_void_p]),
    "xp_gen_normal": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, C.c_uint64, C.c_float]),
    "xp_stream4": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32]),
    "xp_session_create_random": (C.c_int, [C.c_int, C.POINTER(ModelConfig), C.POINTER(Sampling), C.c_uint64,
                                           C.POINTER(C.c_void_p)]),
    "xp_tokenizer_create": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "xp_tokenizer_destroy": (None, [C.c_void_p]),
    "xp_tokenizer_info": (C.c_int, [C.c_void_p] + [C.c_void_p] * 5),
    "xp_tokenizer_encode": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.c_int, C.c_int, C.c_void_p, C.c_uint32,
                                      C.POINTER(C.c_uint32)]),
    "xp_tokenizer_decode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_int, C.c_char_p, C.c_size_t,
                                      C.POINTER(C.c_size_t)]),
    "xp_tokenizer_piece": (C.c_int, [C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "xp_chat_create": (C.c_int, [C.c_int, C.c_char_p, C.c_uint32, C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p)]),
    "xp_chat_prefill": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32)]),
    "xp_chat_step": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.POINTER(C.c_int)]),
    "xp_chat_metrics": (C.c_int, [C.c_void_p, C.POINTER(C.c_double)]),
    "xp_chat_session": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "xp_chat_reset": (C.c_int, [C.c_void_p]),
    "xp_chat_destroy": (None, [C.c_void_p]),
    "xp_session_create_gguf": (C.c_int, [C.c_int, C.c_char_p, C.POINTER(ModelConfig), C.POINTER(Sampling),
                                         C.c_char_p, C.POINTER(C.c_void_p)]),
    "xp_session_load_info": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int), C.c_char_p, C.c_uint32]),
    "xp_session_config": (C.c_int, [C.c_void_p, C.POINTER(ModelConfig)]),
    "xp_gguf_dequantize": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint64]),
    "xp_quant_repack_sizes": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.POINTER(C.c_uint64)]),
    "xp_quant_repack": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32, C.c_uint32] + [C.c_void_p] * 4),
    "xp_session_create": (C.c_int, [C.c_int, C.POINTER(ModelConfig), C.POINTER(Sampling), C.POINTER(LayerWeights),
                                    C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "xp_session_destroy": (C.c_int, [C.c_void_p]),
    "xp_session_tensor_stream": (C.c_uint64, [C.c_uint32, C.c_uint32]),
    "xp_session_prefill": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "xp_session_decode_step": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "xp_session_generate": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.POINTER(C.c_float)]),
    "xp_session_reset": (C.c_int, [C.c_void_p]),
    "xp_session_position": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "xp_session_logits": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "xp_session_stats": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64)]),
    "xp_session_debug_ptr": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]),
    "xp_session_error_word": (C.c_int, [C.c_void_p, C.POINTER(C.c_uint32)]),
    "xp_session_profile_matvec": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_float), C.POINTER(C.c_uint64),
                                            C.POINTER(C.c_uint32)]),
    "xp_session_timer": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_float)]),
    "xp_session_trace": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
}


def lib():
    """Load libxp_cuda.so. Raises if the in-tree library is missing: the
    CUDA path is the only path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"xpose_b200: {LIB_PATH} is missing; build it with `python -m xpose_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(status):
    if status not in (XP_OK,):
        msg = lib().xp_last_error()
        raise XpError(status, msg.decode() if msg else "")
    return status


def exported_symbols():
    """The xp_* names declared in include/xp_cuda.h."""
    return sorted(_SIGS)
