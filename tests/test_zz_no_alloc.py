"""xp_attention_decode_static: attention for callers that cannot allocate
device memory (they run inside an allocator they do not own, or on a path that
must not call cudaMalloc), so the library keeps the scratch itself. Its output
and its fp16 KV append must match xp_attention_decode given caller-allocated
scratch, on two calls in a row (the second reuses the array the first left
behind). Collected last so a run that stops at the first failure has already
run every other test."""
import numpy as np
import pytest

import oracle_lib as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
from gpu_util import dev, empty, host, ptr, rel_l2, sync  # noqa: E402
from xpose_b200._lib import XpError, check, lib  # noqa: E402

HD, NH, MAX_SEQ, NSPLIT = 256, 4, 4096, 64


def _inputs(pos):
    q = O.gen_normal(11, 1, NH * HD, 1.0)
    k = O.gen_normal(11, 2 + pos, HD, 1.0)
    v = O.gen_normal(11, 3 + pos, HD, 1.0)
    qn, kn = O.gen_normal(11, 4, HD, 0.02), O.gen_normal(11, 5, HD, 0.02)
    return [dev(a) for a in (q, k, v, qn, kn)]


def test_static_scratch_matches_caller_scratch_twice():
    hist = torch.from_numpy(O.gen_normal(11, 9, MAX_SEQ * HD, 1.0)).half().numpy().view(np.uint16)
    kc_a, vc_a = dev(hist.copy()), dev(hist[::-1].copy())
    kc_b, vc_b = dev(hist.copy()), dev(hist[::-1].copy())
    scratch = empty(lib().xp_attention_scratch_bytes(NSPLIT) // 4 + 16)
    for pos in (3000, 3001):
        q, k, v, qn, kn = _inputs(pos)
        posd = dev(np.array([pos], np.uint32))
        out_a, out_b = empty(NH * HD), empty(NH * HD)
        check(lib().xp_attention_decode(None, ptr(out_a), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn), ptr(kc_a),
                                        ptr(vc_a), ptr(posd), 0, 1e6, 1e-6, 1.0 / 16, NSPLIT, MAX_SEQ, ptr(scratch)))
        check(lib().xp_attention_decode_static(None, ptr(out_b), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn),
                                               ptr(kc_b), ptr(vc_b), ptr(posd), 0, 1e6, 1e-6, 1.0 / 16, NSPLIT,
                                               MAX_SEQ))
        sync()
        assert rel_l2(host(out_b), host(out_a)) < 1e-3
        assert np.array_equal(host(kc_b, np.uint16), host(kc_a, np.uint16))
        assert np.array_equal(host(vc_b, np.uint16), host(vc_a, np.uint16))


def test_static_scratch_rejects_oversized_split():
    q, k, v, qn, kn = _inputs(0)
    posd = dev(np.array([0], np.uint32))
    with pytest.raises(XpError) as e:
        check(lib().xp_attention_decode_static(None, ptr(empty(NH * HD)), ptr(q), ptr(k), ptr(v), ptr(qn), ptr(kn),
                                               ptr(empty(HD)), ptr(empty(HD)), ptr(posd), 0, 1e6, 1e-6, 1.0 / 16,
                                               1000, MAX_SEQ))
    assert e.value.name == "XP_ERR_INVALID"
