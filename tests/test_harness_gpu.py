"""The standalone C++ harness (blackflash_b200/csrc/harness.cu), the counterpart of the
reference's src/main.cu, run on the reference's own fixture directories: it links the
library through the reference-signature flash_attn_naive_launch and must report PASS
(max |O - o_ref| < 0.02, the reference harness's tolerance, src/main.cu:324)."""
import os
import subprocess
import sys

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


@pytest.mark.parametrize("B,H,N,dist", [(4, 8, 1024, "normal"),
                                        (1, 2, 8192, "peaked")])    # two slices of config 4
def test_harness_passes_on_baseline_distribution_fixtures(tmp_path, B, H, N, dist):
    """Fixtures written by tests/golden/make_ref_data.py with BASELINE's distributions
    (N(0,1); N(0, std 3) / U(-1, 1)) at sizes above the reference fixtures' N <= 192."""
    sys.path.insert(0, GOLDEN_DIR)
    from make_ref_data import write_ref_data
    from blackflash_b200.build import build_harness
    exe = build_harness()
    out = str(tmp_path / "ref_data")
    meta = write_ref_data(out, B, H, N, dist=dist, seed=11)
    assert meta["dist_q"] == ("normal(0,1)" if dist == "normal" else "normal(0,3)")
    res = subprocess.run([exe, out, "5"], capture_output=True, text=True, timeout=300)
    print(res.stdout)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "Status: PASS" in res.stdout
