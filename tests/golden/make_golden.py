"""Regenerate the golden fixtures under tests/golden/ from the reference itself.

Runs the reference's own fixture generator (profile/gen_ref.py) on the CPU of
the build container, once per case, and keeps its outputs unchanged:
q/k/v.bin (bf16), o_ref.bin (bf16, torch SDPA on CPU), s_ref.bin / p_ref.bin
(fp32) and meta.txt. These files pin the CPU oracle (tests/test_oracle.py) and
serve as known inputs/outputs for the GPU parity tests. The reference tree is
not needed at test time; only this script reads it.

    python tests/golden/make_golden.py [/path/to/reference]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

# (B, H, N, seed). gen_ref.py fixes d=64 inputs to U(-0.5, 0.5) (gen_ref.py:54-56).
CASES = [
    (1, 1, 64, 42),    # gen_ref.py defaults
    (1, 2, 128, 42),
    (2, 1, 192, 7),    # N % 128 != 0: exercises the masked KV tail
]


def reference_dir() -> str:
    """The reference checkout: $BLACKFLASH_REFERENCE, else a "reference" directory beside
    this repository."""
    repo = os.path.dirname(os.path.dirname(HERE))
    return os.environ.get("BLACKFLASH_REFERENCE") or os.path.join(os.path.dirname(repo), "reference")


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else reference_dir()
    script = os.path.join(ref, "profile", "gen_ref.py")
    for B, H, N, seed in CASES:
        out = os.path.join(HERE, f"gen_ref_b{B}h{H}n{N}")
        cmd = [sys.executable, script, "--B", str(B), "--H", str(H), "--N", str(N), "--d", "64",
               "--outdir", out, "--seed", str(seed)]
        subprocess.run(cmd, check=True, stdout=subprocess.DEVNULL, env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
        print("wrote", out)


if __name__ == "__main__":
    main()
