"""The epilogues divide by three (the decoder's /3 after each level's branch sum, pt_v21 graph node
/dec/Div) with a product and one FMA-exact correction instead of the IEEE division routine.  It
must be the correctly rounded quotient: checked here on the CPU (IEEE fp32 multiply and fused
multiply-add, as on the GPU) for every fp32 bit pattern."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc absent")
def test_div3_correctly_rounded_for_every_float(tmp_path):
    exe = str(tmp_path / "div3_check")
    subprocess.run(["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-o", exe,
                    os.path.join(HERE, "cpu_checks", "div3_check.c"), "-lm"], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=600).stdout
    assert int(out.strip()) == 0
