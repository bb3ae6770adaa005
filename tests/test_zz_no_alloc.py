"""xp_attention_decode_static: attention for callers that cannot allocate
device memory (they run inside an allocator they do not own, or on a path that
must not call cudaMalloc), so the library keeps the scratch itself. Its output
and its fp16 KV append must match xp_attention_decode given caller-allocated
scratch, on two calls in a row (the second reuses the array the first left
behind), and the array's error word, read through
xp_attention_static_error_word, must stay clear. Collected last so a run that
stops at the first failure has already run every other test."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import XpError, check, lib  # noqa: E402

HD, NH, MAX_SEQ = 256, 4, 4096


def _inputs(pos):
    q = O.gen_normal(11, 1, NH * HD, 1.0)
    k = O.gen_normal(11, 2 + pos, HD, 1.0)
    v = O.gen_normal(11, 3 + pos, HD, 1.0)
    qn, kn = O.gen_normal(11, 4, HD, 0.02), O.gen_normal(11, 5, HD, 0.02)
    return [dev(a) for a in (q, k, v, qn, kn)]


def _static_error_word(clear=True):
    w = C.c_uint32(0xFFFFFFFF)
    check(lib().xp_attention_static_error_word(None, C.byref(w), int(clear)))
    return w.value


@pytest.mark.parametrize("nsplit", [1, 64])
def test_static_scratch_matches_caller_scratch_twice(nsplit):
    hist = torch.from_numpy(O.gen_normal(11, 9, MAX_SEQ * HD, 1.0)).half().numpy().view(np.uint16)
    kc_a, vc_a = dev(hist.copy()), dev(hist[::-1].copy())
    kc_b, vc_b = dev(hist.copy()), dev(hist[::-1].copy())
    scratch = empty(lib().xp_attention_scratch_bytes(nsplit) // 4 + 16)
    # nsplit 1 attends to a 512-row window (one split holds it); 64 splits the whole cache
    window = 512 if nsplit == 1 else 0
    _static_error_word(clear=True)
    for pos in (3000, 3001):
        q, k, v, qn, kn = _inputs(pos)
        posd = dev(np.array([pos], np.uint32))
        out_a, out_b = empty(NH * HD), empty(NH * HD)
        check(lib().xp_attention_decode(None, ptr(out_a), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn), ptr(kc_a),
                                        ptr(vc_a), ptr(posd), window, 1e6, 1e-6, 1.0 / 16, nsplit, MAX_SEQ,
                                        ptr(scratch)))
        check(lib().xp_attention_decode_static(None, ptr(out_b), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn),
                                               ptr(kc_b), ptr(vc_b), ptr(posd), window, 1e6, 1e-6, 1.0 / 16, nsplit,
                                               MAX_SEQ))
        sync()
        assert rel_l2(host(out_b), host(out_a)) < 1e-3
        assert np.array_equal(host(kc_b, np.uint16), host(kc_a, np.uint16))
        assert np.array_equal(host(vc_b, np.uint16), host(vc_a, np.uint16))
        assert _static_error_word(clear=False) == 0
        assert int(host(scratch, np.uint32)[1]) == 0  # the caller-scratch call's own error word


@pytest.mark.parametrize("nsplit", [0, 65, 1000])
def test_static_scratch_rejects_split_counts_outside_the_array(nsplit):
    q, k, v, qn, kn = _inputs(0)
    posd = dev(np.array([0], np.uint32))
    with pytest.raises(XpError) as e:
        check(lib().xp_attention_decode_static(None, ptr(empty(NH * HD)), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn),
                                               ptr(empty(HD)), ptr(empty(HD)), ptr(posd), 0, 1e6, 1e-6, 1.0 / 16,
                                               nsplit, MAX_SEQ))
    assert e.value.name == "XP_ERR_INVALID"


def test_static_scratch_reports_a_position_past_the_caches():
    """A device-resident position at max_seq would append past the caches:
    the kernel writes nothing and sets bit 128 of the array's error word,
    which the caller reads back without allocating."""
    max_seq = 64
    q, k, v, qn, kn = _inputs(0)
    guard = 0x5A5A
    kc = dev(np.full(max_seq * HD + 2 * HD, guard, np.uint16))
    vc = dev(np.full(max_seq * HD + 2 * HD, guard, np.uint16))
    posd = dev(np.array([max_seq], np.uint32))
    _static_error_word(clear=True)
    check(lib().xp_attention_decode_static(None, ptr(empty(NH * HD)), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn),
                                           ptr(kc), ptr(vc), ptr(posd), 0, 1e6, 1e-6, 1.0 / 16, 8, max_seq))
    assert _static_error_word(clear=True) == 128
    assert _static_error_word(clear=False) == 0
    assert (host(kc, np.uint16) == guard).all() and (host(vc, np.uint16) == guard).all()
