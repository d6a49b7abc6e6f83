"""Writes `ref_data` fixture directories in the reference's format
(profile/gen_ref.py:159-197: raw little-endian bf16 q/k/v/o_ref.bin in [B, H, N, d]
order and a key=value meta.txt) for the distributions the benchmark configurations use,
which gen_ref.py cannot draw (it fixes U(-0.5, 0.5), profile/gen_ref.py:54-56).

Test infrastructure: O comes from the CPU oracle (exact softmax attention in double,
oracle/attn_oracle.c), rounded to bf16 like gen_ref's o_ref. s_ref.bin / p_ref.bin are
not written (the harness treats them as optional). meta.txt adds `seed` and
`dist_q` / `dist_k` / `dist_v` to gen_ref's keys; readers that know only gen_ref's keys
skip them.

    python tests/golden/make_ref_data.py --config 2 --outdir ref_data
    python tests/golden/make_ref_data.py --B 1 --H 2 --N 8192 --dist peaked --outdir ref_peaked
"""
from __future__ import annotations

import argparse
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

# Benchmark configurations (B, H, N, distribution); d = 64.
CONFIGS = {"1": (2, 2, 512, "normal"), "2": (4, 8, 1024, "normal"), "3": (64, 64, 1024, "normal"),
           "4": (8, 16, 8192, "peaked"), "5": (1, 32, 65536, "normal")}
# Per-tensor distribution names written to meta.txt (std, not variance, for the normals).
DIST_NAMES = {"normal": ("normal(0,1)",) * 3,
              "peaked": ("normal(0,3)", "normal(0,3)", "uniform(-1,1)"),
              "uniform": ("uniform(-0.5,0.5)",) * 3}


def write_ref_data(outdir: str, B: int, H: int, N: int, d: int = 64, dist: str = "normal", seed: int = 0) -> dict:
    """Draw Q/K/V (blackflash_b200.inputs.make_qkv, seeded), compute O with the oracle and
    write the directory. Returns the meta dictionary."""
    import numpy as np
    import torch

    from blackflash_b200.inputs import make_qkv
    from oracle import oracle
    q, k, v = make_qkv(B, H, N, d=d, dist=dist, seed=seed)
    scale = 1.0 / math.sqrt(d)
    o, _, _ = oracle.attn_exact(q, k, v, scale)
    o_bf16 = torch.from_numpy(np.ascontiguousarray(o, dtype=np.float32)).to(torch.bfloat16)
    os.makedirs(outdir, exist_ok=True)
    for name, t in (("q.bin", q), ("k.bin", k), ("v.bin", v), ("o_ref.bin", o_bf16)):
        t.contiguous().view(torch.uint16).numpy().tofile(os.path.join(outdir, name))
    dq, dk, dv = DIST_NAMES[dist]
    meta = {"B": B, "H": H, "N": N, "d": d, "scale": f"{scale:.10f}", "seed": seed,
            "dist_q": dq, "dist_k": dk, "dist_v": dv}
    with open(os.path.join(outdir, "meta.txt"), "w") as f:
        for key, val in meta.items():
            f.write(f"{key}={val}\n")
    return meta


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", choices=sorted(CONFIGS), help="a benchmark configuration")
    ap.add_argument("--B", type=int)
    ap.add_argument("--H", type=int)
    ap.add_argument("--N", type=int)
    ap.add_argument("--d", type=int, default=64)
    ap.add_argument("--dist", choices=sorted(DIST_NAMES), default="normal")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--outdir", required=True)
    a = ap.parse_args()
    if a.config:
        B, H, N, dist = CONFIGS[a.config]
    else:
        if None in (a.B, a.H, a.N):
            ap.error("give --config or all of --B --H --N")
        B, H, N, dist = a.B, a.H, a.N, a.dist
    print(write_ref_data(a.outdir, B, H, N, a.d, dist, a.seed))


if __name__ == "__main__":
    main()
