"""The quotient of the packed int8 row quantizer (quant_rows16_kernel): Markstein's correction in
place of the IEEE division, checked exhaustively over every fp16 and bf16 pair the quantizer can
meet by tests/quotient_check.c (host IEEE arithmetic, the operations the kernel issues), and a
planted mistake (the uncorrected product x * RN(1/s)) that the check must reject."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "quotient_check.c")


@pytest.fixture(scope="module")
def binaries(tmp_path_factory):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    d = tmp_path_factory.mktemp("quotient_check")
    out = {}
    for name, extra in (("check", []), ("planted", ["-DPLANT_UNCORRECTED"])):
        exe = str(d / name)
        r = subprocess.run([gcc, "-O2", "-mfma", "-ffp-contract=off", *extra, SRC, "-o", exe, "-lm"],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        out[name] = exe
    return out


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_markstein_quotient_equals_the_division(binaries, dtype):
    r = subprocess.run([binaries["check"], dtype], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr[-2000:]
    assert "quotient mismatches 0 code mismatches 0" in r.stdout
    assert int(r.stdout.split("pairs ")[1].split()[0]) > 2 ** 28


def test_planted_uncorrected_quotient_is_rejected(binaries):
    r = subprocess.run([binaries["planted"], "fp16"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 1, r.stdout
