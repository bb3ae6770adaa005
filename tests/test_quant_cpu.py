"""Host logic of the GGUF quant repack (no GPU): xp_quant_repack_sizes gives
the plane sizes the reference's host repack (examples/llm/quant_repack.cpp)
allocates for every supported type and shape, and refuses what that repack
refuses (other types, cols not a multiple of 32, or of 256 for the K types)."""
import ctypes as C

import pytest

import oracle_lib as O
from gguf_blocks import random_blocks
from xpose_b200._lib import XpError, check, lib


def sizes_of(t, rows, cols):
    s = (C.c_uint64 * 4)()
    check(lib().xp_quant_repack_sizes(t, rows, cols, s))
    return list(s)


@pytest.mark.skipif(O.ref() is None, reason="oracle/_ref not built")
@pytest.mark.parametrize("t", [8, 6, 12, 14])
@pytest.mark.parametrize("rows,cols", [(1, 256), (64, 512), (100, 1536), (129, 256)])
def test_plane_sizes_match_the_reference_repack(t, rows, cols):
    raw = random_blocks(t, rows * cols, seed=rows + t)
    lib_ref = O.ref()
    lib_ref.xpref_quant_repack.argtypes = [C.c_uint32, C.c_char_p, C.c_uint32, C.c_uint32] + [C.c_void_p] * 4 + [
        C.POINTER(C.c_uint64)]
    want = (C.c_uint64 * 4)()
    assert lib_ref.xpref_quant_repack(t, raw, rows, cols, None, None, None, None, want) == 0
    assert sizes_of(t, rows, cols) == list(want)


@pytest.mark.parametrize("t,rows,cols", [(8, 4, 48), (12, 4, 288), (14, 4, 32), (2, 4, 256), (8, 0, 256)])
def test_unrepackable_shapes_are_refused(t, rows, cols):
    s = (C.c_uint64 * 4)()
    with pytest.raises(XpError) as e:
        check(lib().xp_quant_repack_sizes(t, rows, cols, s))
    assert e.value.name == "XP_ERR_INVALID"
