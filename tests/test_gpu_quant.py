"""The reference's GGUF quant module (kernels/llm_quant.cl) through the kernel
registry, against the reference's own kernels compiled for the host
(oracle/_ref) on the same seeded blocks:

* fp16_decode over all 65536 bit patterns: bit-exact (NaN payloads included);
* dequant_q8_0 / q5_0 / q4_k / q6_k: bit-exact;
* matvec_q8_0 / q5_0 / q4_k / q6_k on the native block layouts and
  matvec_rq* (+ _split, mv_reduce) on the planes of the reference's own host
  repack (examples/llm/quant_repack.cpp): within fp32 rounding, the bar of the
  reference's harness (max |diff| <= 1e-5 max |out|), since the blocks are
  summed in another order here;
* split-K edge cases: more splits than k-blocks (empty splits write 0);
* quant_test.cpp, the reference's harness for this module, runs unchanged on
  the drop-in against a GGUF file holding tensors of all four formats."""
import ctypes as C
import os
import subprocess
import sys
import tempfile

import numpy as np
import pytest

import oracle_lib as O
from gguf_blocks import random_blocks

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(O.ref() is None, reason="oracle/_ref not built")]
pytest.importorskip("torch")
from xpose_b200.vulkore import Context, Grid, Program, launch  # noqa: E402

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))
from gguf_writer import ARR, STR, U32, write_gguf  # noqa: E402

QT = "kernels/llm_quant.spv"
# ggml type id -> (kernel suffix, elements per block, bytes per block)
FORMATS = {8: ("q8_0", 32, 34), 6: ("q5_0", 32, 22), 12: ("q4_k", 256, 144), 14: ("q6_k", 256, 210)}
RQ = {12: "rq4_k", 6: "rq5_0", 14: "rq6_k", 8: "rq8_0"}


@pytest.fixture(scope="module")
def ctx():
    return Context()


def buf(ctx, a):
    b = ctx.alloc(len(a), a.dtype)
    b.upload(a)
    return b


def words(raw):
    """Bytes as a uint32 buffer (the reference's 4-byte element rule), zero-padded."""
    pad = (-len(raw)) % 4
    return np.frombuffer(raw + b"\0" * pad, np.uint32).copy()


def close(got, want):
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5 * max(np.abs(want).max(), 1e-30))


def test_fp16_decode_all_patterns_bitexact(ctx):
    src = np.arange(65536, dtype=np.uint32)
    src = (src[0::2] | (src[1::2] << 16)).astype(np.uint32)
    want = np.zeros(65536, np.float32)
    O.ref_launch("fp16_decode", 65536, want, src, 65536, module=QT)
    out = ctx.alloc(65536)
    launch(Program.from_file(ctx, QT).kernel("fp16_decode"), Grid(65536), out, buf(ctx, src), 65536,
           stream=ctx.stream)
    ctx.wait_idle()
    assert np.array_equal(out.download().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", sorted(FORMATS))
def test_dequant_bitexact(ctx, t):
    name, be, _ = FORMATS[t]
    n = 256 * 37
    src = words(random_blocks(t, n, seed=40 + t))
    want = np.zeros(n, np.float32)
    O.ref_launch("dequant_" + name, n, want, src, n, module=QT)
    out = ctx.alloc(n)
    launch(Program.from_file(ctx, QT).kernel("dequant_" + name), Grid(n), out, buf(ctx, src), n, stream=ctx.stream)
    ctx.wait_idle()
    assert np.array_equal(out.download().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", sorted(FORMATS))
@pytest.mark.parametrize("rows,cols", [(300, 1536), (64, 256), (1, 4096)])
def test_native_matvec(ctx, t, rows, cols):
    name, be, _ = FORMATS[t]
    src = words(random_blocks(t, rows * cols, seed=rows + cols + t))
    x = np.random.default_rng(t).uniform(-1, 1, cols).astype(np.float32)
    want = np.zeros(rows, np.float32)
    O.ref_launch("matvec_" + name, rows, want, x, src, rows, cols, module=QT)
    out = ctx.alloc(rows)
    launch(Program.from_file(ctx, QT).kernel("matvec_" + name), Grid(rows), out, buf(ctx, x), buf(ctx, src), rows,
           cols, stream=ctx.stream)
    ctx.wait_idle()
    close(out.download(), want)


def repack(t, raw, rows, cols):
    """The reference's host repack (quant_repack.cpp): quant, high, scale, bias."""
    lib = O.ref()
    lib.xpref_quant_repack.argtypes = [C.c_uint32, C.c_char_p, C.c_uint32, C.c_uint32] + [C.c_void_p] * 4 + [
        C.POINTER(C.c_uint64)]
    sizes = (C.c_uint64 * 4)()
    assert lib.xpref_quant_repack(t, raw, rows, cols, None, None, None, None, sizes) == 0
    q = np.zeros(sizes[0], np.uint32)
    h = np.zeros(max(sizes[1], 1), np.uint32)
    s = np.zeros(sizes[2], np.float32)
    b = np.zeros(max(sizes[3], 1), np.float32)
    assert lib.xpref_quant_repack(t, raw, rows, cols, q.ctypes.data, h.ctypes.data, s.ctypes.data, b.ctypes.data,
                                  sizes) == 0
    return q, (h if sizes[1] else None), s, (b if sizes[3] else None)


def rq_args(t, planes):
    q, h, s, b = planes
    if t == 12:
        return [q, s, b]
    if t in (6, 14):
        return [q, h, s]
    return [q, s]


@pytest.mark.parametrize("t", sorted(RQ))
@pytest.mark.parametrize("rows,cols", [(1152, 1536), (100, 512)])
def test_repacked_matvec_and_split(ctx, t, rows, cols):
    raw = random_blocks(t, rows * cols, seed=7 * t + rows)
    planes = repack(t, raw, rows, cols)
    x = np.random.default_rng(rows + t).uniform(-1, 1, cols).astype(np.float32)
    prog = Program.from_file(ctx, QT)
    host = rq_args(t, planes)
    dev = [buf(ctx, a) for a in host]
    want = np.zeros(rows, np.float32)
    O.ref_launch("matvec_" + RQ[t], rows, want, x, *host, rows, cols, module=QT)
    out = ctx.alloc(rows)
    launch(prog.kernel("matvec_" + RQ[t]), Grid(rows), out, buf(ctx, x), *dev, rows, cols, stream=ctx.stream)
    ctx.wait_idle()
    close(out.download(), want)
    nkb = cols // 32
    for split in (3, nkb + 5):  # the second leaves empty splits, which write 0
        pw = np.zeros(rows * split, np.float32)
        O.ref_launch("matvec_" + RQ[t] + "_split", rows * split, pw, x, *host, rows, cols, split, module=QT)
        part = ctx.alloc(rows * split)
        launch(prog.kernel("matvec_" + RQ[t] + "_split"), Grid(rows * split), part, buf(ctx, x), *dev, rows, cols,
               split, stream=ctx.stream)
        ctx.wait_idle()
        got = part.download()
        close(got, pw)
        assert np.array_equal(got[pw == 0], pw[pw == 0])
        red = ctx.alloc(rows)
        launch(prog.kernel("mv_reduce"), Grid(rows), red, part, rows, split, stream=ctx.stream)
        ctx.wait_idle()
        red_want = np.zeros(rows, np.float32)
        O.ref_launch("mv_reduce", rows, red_want, got, rows, split, module=QT)
        assert np.array_equal(red.download(), red_want)
        close(red_want, want)


def test_registry_lists_the_quant_module(ctx):
    prog = Program.from_file(ctx, QT)
    names = ["fp16_decode", "mv_reduce"] + [p + f for f in ("q8_0", "q5_0", "q4_k", "q6_k") for p in
                                            ("dequant_", "matvec_")]
    names += ["matvec_" + r + s for r in RQ.values() for s in ("", "_split")]
    for n in names:
        assert prog.kernel(n).name == n
    assert len(names) == 18


def test_quant_test_harness_runs():
    """examples/llm/quant_test.cpp, unchanged, on the drop-in: fp16 sweep,
    synthetic blocks, tensors of every format from a GGUF file, the repacked
    kernels and split-K."""
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "quant_test_gpu")
    if not os.path.exists(exe):
        pytest.skip("quant_test_gpu not built")
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "quant.gguf")
        tensors = []
        for t, (name, be, _) in sorted(FORMATS.items()):
            cols = 1536 if be == 256 else 1152
            tensors.append((f"blk.0.{name}.weight", (cols, 320), ("raw", t, random_blocks(t, cols * 320, seed=t))))
        meta = [("general.architecture", STR, "gemma3"), ("general.alignment", U32, 32),
                ("tokenizer.ggml.tokens", ARR, (STR, ["<t0>"]))]
        write_gguf(path, meta, tensors)
        p = subprocess.run(["stdbuf", "-oL", exe, QT, path], capture_output=True, text=True, timeout=900,
                           cwd=os.path.dirname(exe))
    assert p.returncode == 0, (p.stdout + p.stderr)[-4000:]
    assert "FAIL" not in p.stdout, p.stdout[-4000:]
    assert p.stdout.count("PASS") >= 20, p.stdout[-4000:]
    assert "no 2-D tensor" not in p.stdout and "could not open" not in p.stdout, p.stdout[-4000:]


@pytest.mark.parametrize("t", sorted(RQ))
@pytest.mark.parametrize("rows,cols", [(1152, 1536), (100, 512)])
def test_device_repack_bitexact_and_drives_the_rq_kernels(ctx, t, rows, cols):
    """xp_quant_repack on the device makes the reference host repack's planes
    bit for bit (padding rows zero), and matvec_rq* over them matches."""
    from xpose_b200._lib import check, lib
    raw = random_blocks(t, rows * cols, seed=11 * t + cols)
    want = repack(t, raw, rows, cols)
    sizes = (C.c_uint64 * 4)()
    check(lib().xp_quant_repack_sizes(t, rows, cols, sizes))
    assert [sizes[0], sizes[2]] == [len(want[0]), len(want[2])]
    assert sizes[1] == (0 if want[1] is None else len(want[1])) and sizes[3] == (0 if want[3] is None else len(want[3]))
    src = buf(ctx, words(raw))
    q = ctx.alloc(sizes[0], np.uint32)
    h = ctx.alloc(max(sizes[1], 1), np.uint32)
    s = ctx.alloc(sizes[2])
    b = ctx.alloc(max(sizes[3], 1))
    check(lib().xp_quant_repack(None, t, src.ptr, rows, cols, q.ptr, h.ptr if sizes[1] else None, s.ptr,
                                b.ptr if sizes[3] else None))
    ctx.wait_idle()
    assert np.array_equal(q.download(), want[0])
    assert np.array_equal(s.download().view(np.uint32), want[2].view(np.uint32))
    if want[1] is not None:
        assert np.array_equal(h.download(), want[1])
    if want[3] is not None:
        assert np.array_equal(b.download().view(np.uint32), want[3].view(np.uint32))
    x = np.random.default_rng(t).uniform(-1, 1, cols).astype(np.float32)
    ref = np.zeros(rows, np.float32)
    O.ref_launch("matvec_" + RQ[t], rows, ref, x, *rq_args(t, want), rows, cols, module=QT)
    dev = {12: [q, s, b], 6: [q, h, s], 14: [q, h, s], 8: [q, s]}[t]
    out = ctx.alloc(rows)
    launch(Program.from_file(ctx, QT).kernel("matvec_" + RQ[t]), Grid(rows), out, buf(ctx, x), *dev, rows, cols,
           stream=ctx.stream)
    ctx.wait_idle()
    close(out.download(), ref)
