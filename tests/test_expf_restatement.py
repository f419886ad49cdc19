"""The SiLU epilogue's exp is a restatement of the table-driven expf that glibc uses (the
method of ARM's optimized-routines; Rust's f32::exp is the platform expf), so that SiLU is
bit-exact against the reference on the device.  This runs the same double operations on the
host against this machine's libm expf on every float in [-20, 20] -- the whole range SiLU
evaluates exp on -- and on the positive range too."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = str(tmp_path_factory.mktemp("expf") / "expf_check")
    src = os.path.join(HERE, "expf_check.c")
    base = [cc, "-O2", "-ffp-contract=off", "-fno-fast-math", src, "-o", exe, "-lm"]
    if subprocess.run(base + ["-fopenmp"], capture_output=True).returncode != 0:
        subprocess.run(base, check=True)
    return exe


# float bits: [+0, 20] = [0x00000000, 0x41A00000], [-0, -20] = [0x80000000, 0xC1A00000]
@pytest.mark.parametrize("lo,hi", [(0x00000000, 0x41A00001), (0x80000000, 0xC1A00001)], ids=["0_to_20", "0_to_-20"])
def test_expf_restatement_equals_libm(checker, lo, hi):
    r = subprocess.run([checker, hex(lo), hex(hi)], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
