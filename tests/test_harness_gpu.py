"""The standalone C++ harness (blackflash_b200/csrc/harness.cu), the counterpart of the
reference's src/main.cu, run on the reference's own fixture directories: it links the
library through the reference-signature flash_attn_naive_launch and must report PASS
(max |O - o_ref| < 0.02, the reference harness's tolerance, src/main.cu:324)."""
import os
import subprocess

import pytest

from golden_io import GOLDEN_DIR, golden_cases

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", golden_cases())
def test_harness_passes_on_reference_fixtures(case):
    from blackflash_b200.build import build_harness
    exe = build_harness()
    res = subprocess.run([exe, os.path.join(GOLDEN_DIR, case), "5"], capture_output=True, text=True, timeout=120)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "Status: PASS" in res.stdout
