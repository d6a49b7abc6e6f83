"""Readers for the reference's fixture format (profile/gen_ref.py:159-197):
raw little-endian bf16 / fp32 files plus a key=value meta.txt."""
from __future__ import annotations

import os

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden_cases() -> list[str]:
    return sorted(d for d in os.listdir(GOLDEN_DIR) if d.startswith("gen_ref_"))


def read_meta(path: str) -> dict:
    meta = {}
    with open(os.path.join(path, "meta.txt")) as f:
        for line in f:
            if "=" in line:
                k, v = line.strip().split("=", 1)
                meta[k] = float(v) if k == "scale" else (int(v) if v.lstrip("-").isdigit() else v)
    return meta


def load_case(name: str) -> dict:
    path = os.path.join(GOLDEN_DIR, name)
    meta = read_meta(path)
    shape = (meta["B"], meta["H"], meta["N"], meta["d"])
    sshape = (meta["B"], meta["H"], meta["N"], meta["N"])

    def bf16(fn):
        return np.fromfile(os.path.join(path, fn), dtype="<u2").reshape(shape)

    def f32(fn):
        return np.fromfile(os.path.join(path, fn), dtype="<f4").reshape(sshape)

    return dict(meta=meta, q=bf16("q.bin"), k=bf16("k.bin"), v=bf16("v.bin"), o_ref=bf16("o_ref.bin"),
                s_ref=f32("s_ref.bin"), p_ref=f32("p_ref.bin"))
