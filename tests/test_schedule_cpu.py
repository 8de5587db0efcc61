"""Host logic of the tiled kernel's balanced step schedules, no GPU: a small
program compiled against bilinear_tiled.cuh checks that every step with a
non-zero high-part factor is scheduled exactly once and to the right line,
that no lane exceeds the round count, and that the donor masks match the
borrowed segments, for n = 5..10, every sum and null high generators; and
that the config-5 left contraction gets six rounds per sum (16 and 32 on the
row-major sweep); and that the Cl(6,1) route's sign masks equal the tables of
tests/test_cl61_math_cpu.py, which are checked there against the oracle."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not available")
def test_step_schedules(tmp_path):
    exe = tmp_path / "sched_check"
    src = os.path.join(HERE, "native", "sched_check.cu")
    subprocess.run(["nvcc", "-std=c++17", "--expt-relaxed-constexpr",
                    "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(exe), src],
                   check=True, capture_output=True, timeout=600)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True,
                         timeout=120).stdout
    assert "bad 0" in out, out
    for mode in range(3):
        assert f"lc10 mode {mode} rounds 6" in out, out
    from tests.test_cl61_math_cpu import tables
    _, A, B = tables()
    am = sum(1 << k for k in range(64) if A[k] < 0)
    bm = sum(1 << k for k in range(64) if B[k] < 0)
    assert f"phi61 {am:016x} {bm:016x}" in out, out
    active = int(out.split("active ")[1].split()[0])
    inner = int(out.split("inner ")[1].split()[0])
    assert active > 0 and inner > 0, out
