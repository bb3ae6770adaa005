"""The C ABI without a GPU: the library loads, exports every symbol declared
in include/xp_cuda.h, resolves the reference's kernel names by module, and
rejects bad launches with the reference's error categories
(src/launch.cpp:21-131, include/vulkore/program.hpp:107) before touching the
device."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from xpose_b200._lib import LIB_PATH, XpError, exported_symbols, lib

XP_ERR_INVALID = -1
from xpose_b200.vulkore import Grid, Kernel, Program, _marshal, launch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    text = open(os.path.join(ROOT, "include", "xp_cuda.h")).read()
    return sorted(set(re.findall(r"\b(xp_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = C.CDLL(LIB_PATH)
    missing = [s for s in declared() if not hasattr(L, s)]
    assert not missing, missing
    assert set(declared()) == set(exported_symbols())


# every entry point examples/llm/decode.cpp resolves with need_kernel (:1340-1415)
DECODE_KERNELS = {
    "kernels/llm_matvec.spv": ["mv_km4_bs", "mv_km4_bs_split", "mv_reduce"],
    "kernels/llm_transformer.spv": ["rmsnorm_sumsq", "rmsnorm_apply_gemma", "rmsnorm_heads_gemma", "rope", "geglu",
                                    "attention_scores", "softmax_rows", "attention_apply", "add_residual",
                                    "kv_append", "argmax", "softmax_rows_partial", "softmax_rows_finish",
                                    "softmax_rows_scale", "attention_scores_mq4", "attention_apply_mq4",
                                    "attention_apply_reduce"],
    "kernels/llm_sampling.spv": ["argmax_partial", "argmax_reduce", "argmax_final", "topk4_partial"],
}


@pytest.mark.parametrize("module", sorted(DECODE_KERNELS))
def test_registry_resolves_decode_kernels(module):
    prog = Program(None, module)
    for name in DECODE_KERNELS[module]:
        k = prog.kernel(name)
        assert k.name == name and k.module.endswith(module.split("/")[-1])


def test_registry_signatures_match_reference_prototypes():
    k = Program(None, "kernels/llm_matvec.spv").kernel("mv_km4_bs")
    # mv_km4_bs(float* out, const float* in, const uint4* wq, const uint2* sc, uint rows, uint cols)
    assert [a[:2] for a in k.args()] == [(1, 0)] * 4 + [(0, 4)] * 2
    assert "('out')" in k.args()[0][2]
    k = Program(None, "llm_transformer.spv").kernel("rope")
    assert [a[:2] for a in k.args()] == [(1, 0), (0, 4), (0, 4), (0, 4), (0, 4)]


def test_unknown_kernel_lists_the_module():
    with pytest.raises(XpError) as e:
        Program(None, "kernels/llm_transformer.spv").kernel("no_such_kernel")
    assert e.value.name == "XP_ERR_NO_KERNEL"
    assert "rmsnorm_heads_gemma" in str(e.value) and "no_such_kernel" in str(e.value)


class FakeBuf:
    """A non-null pointer value; validation never dereferences it."""
    is_cuda = True

    def data_ptr(self):
        return 0x1000


def test_launch_validation_errors():
    k = Program(None, "kernels/llm_transformer.spv").kernel("add_residual")  # (x, y, n)
    b = FakeBuf()
    with pytest.raises(XpError) as e:
        launch(k, Grid(16), b, b)
    assert e.value.name == "XP_ERR_ARITY" and "expects 3 argument(s)" in str(e.value)
    with pytest.raises(XpError) as e:
        launch(k, Grid(16), b, 3, 16)
    assert e.value.name == "XP_ERR_ARG_KIND" and "('y')" in str(e.value)
    with pytest.raises(XpError) as e:
        launch(k, Grid(16), 5, b, 16)
    assert e.value.name == "XP_ERR_ARG_KIND"
    with pytest.raises(XpError) as e:
        launch(k, Grid(16), b, b, np.uint64(16))
    assert e.value.name == "XP_ERR_ARG_SIZE" and "8-byte" in str(e.value)
    with pytest.raises(XpError) as e:
        launch(Program(None, "llm_sampling.spv").kernel("apply_temperature"), Grid(16), b, np.float64(0.5), 16)
    assert e.value.name == "XP_ERR_ARG_SIZE" and "double literal" in str(e.value)
    with pytest.raises(XpError) as e:
        launch(k, Grid(0), b, b, 16)
    assert e.value.name == "XP_ERR_GRID" and "grid.x must be nonzero" in str(e.value)


def test_status_names_and_version():
    L = lib()
    assert L.xp_status_name(-9) == b"XP_ERR_KV_FULL"
    assert b"sm_100a" in L.xp_version()
    assert L.xp_kernel_count() >= 40


def test_no_device_is_reported_not_crashed():
    if lib().xp_device_count() > 0:
        pytest.skip("a device is present")
    h = C.c_void_p()
    assert lib().xp_context_create(0, C.byref(h)) == -12


def test_fence_null_wait_is_signaled():
    assert lib().xp_fence_wait(None, 0) == 0


def test_mv_plan_validation_on_host():
    """xp_mv_plan_create checks every job before touching a device."""
    class Job(C.Structure):
        _fields_ = [("out", C.c_void_p), ("inp", C.c_void_p), ("wq", C.c_void_p), ("sc", C.c_void_p),
                    ("rows", C.c_uint32), ("cols", C.c_uint32)]
    plan = C.c_void_p()
    bad_shape = (Job * 1)(Job(8, 8, 8, 8, 1152, 100))
    assert lib().xp_mv_plan_create(C.cast(bad_shape, C.c_void_p), 1, C.byref(plan)) == XP_ERR_INVALID
    assert b"multiple" in lib().xp_last_error()
    null_ptr = (Job * 1)(Job(8, None, 8, 8, 1152, 64))
    assert lib().xp_mv_plan_create(C.cast(null_ptr, C.c_void_p), 1, C.byref(plan)) == XP_ERR_INVALID
    assert lib().xp_mv_plan_create(C.cast(null_ptr, C.c_void_p), 0, C.byref(plan)) == XP_ERR_INVALID
    assert not plan.value
    lib().xp_mv_plan_destroy(None)
