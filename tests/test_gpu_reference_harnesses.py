"""The reference's own kernel harnesses, compiled unchanged against the
drop-in runtime headers (include/xp/vulkore/vulkore.hpp) and linked to
libxp_cuda.so (oracle/Makefile target `harnesses`): every kernel they look up
by module and name and launch is a B200 kernel of this library.

* examples/llm/kernel_tests.cpp: all of its checks pass (its CPU references,
  its tolerances).
* examples/llm/sampling_test.cpp: every check it prints passes up to its
  "prefill scores == decode scores" step, which calls the 9-argument
  attention_scores with 8 arguments; the launch validation rejects that call
  with the reference's own arity error (src/launch.cpp:63-131 does the same),
  so the harness stops there. The prefill-shape checks it would run after
  that are run through the registry in test_gpu_prefill_entry_points.py.
* examples/llm/attn_bench.cpp: runs to completion (a benchmark; its maxrel
  columns are its own CPU comparisons)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")


def run(name, *args):
    exe = os.path.join(REF, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built (oracle/Makefile target harnesses)")
    p = subprocess.run(["stdbuf", "-oL", exe, *args], cwd=REF, capture_output=True, text=True, timeout=600)
    return p.returncode, p.stdout + p.stderr


def test_kernel_tests_pass():
    rc, out = run("kernel_tests_gpu")
    assert rc == 0, out[-2000:]
    assert " 0 failed" in out and "FAIL" not in out, out[-2000:]


def test_sampling_test_checks_pass_up_to_its_arity_defect():
    rc, out = run("sampling_test_gpu")
    lines = [l for l in out.splitlines() if "PASS" in l or "FAIL" in l]
    assert len(lines) >= 10, out[-2000:]
    assert not [l for l in lines if "FAIL" in l], out[-3000:]
    assert "XP_ERR_ARITY" in out and "'attention_scores' expects 9 argument(s)" in out and "got 8" in out


def test_attn_bench_runs():
    rc, out = run("attn_bench_gpu", "--reps", "8", "--best-of", "2")
    assert rc == 0, out[-2000:]
    assert "apply_mq4" in out
