"""The GELU epilogue divides by the constants 3, 5 and 7 without a division instruction
(Brisebarre-Muller-Raina: q = RN(x*z), r = x - q*c by FMA, RN(q + r*z)).  Its operands stay
below 2^17 in magnitude (|t| <= 5 on the polynomial branch, t^7 <= 78125).  These checks run
the same float operations on the host against IEEE division:
- every float in [1, 2) and in [2^16, 2^17): the method commutes with scaling by a power of two
  while every intermediate is a normal float, so one binade stands for all binades between;
- every float below 2^-122, subnormals included: q = RN(x*z) and the quotient leave the
  normal range only below about 2^-123.
(A run over all 2^31 magnitudes below 2^17 found no mismatch either.)"""
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
    exe = str(tmp_path_factory.mktemp("divc") / "gelu_div_check")
    src = os.path.join(HERE, "gelu_div_check.c")
    base = [cc, "-O2", "-ffp-contract=off", "-fno-fast-math", src, "-o", exe, "-lm"]
    if subprocess.run(base + ["-fopenmp"], capture_output=True).returncode != 0:
        subprocess.run(base, check=True)
    return exe


@pytest.mark.parametrize("lo,hi", [(0x3F800000, 0x40000000), (0x47800000, 0x48000000), (0x00000000, 0x02800000)],
                         ids=["binade_1_2", "binade_2^16_2^17", "below_2^-122"])
def test_division_by_constants_is_correctly_rounded(checker, lo, hi):
    r = subprocess.run([checker, hex(lo), hex(hi)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
