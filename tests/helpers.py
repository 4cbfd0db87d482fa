"""Shared helpers for the parity tests (host side only)."""
from __future__ import annotations

import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
VALIDATE_CASES = ["bf16_f32", "bf16_q8r", "bf16_q4g32", "bf16_mxfp4", "mxfp4_blocks", "mixtral_q4g32",
                  "qwen3moe_q4g32"]


def load_validate_case(name: str, outdir: str):
    """Write the stored reference-converted containers of a validate case
    into outdir and return (outdir, fixture dict)."""
    z = np.load(os.path.join(GOLDEN, f"validate_{name}.npz"))
    os.makedirs(outdir, exist_ok=True)
    z["dense"].tofile(os.path.join(outdir, "dense.midge"))
    z["experts"].tofile(os.path.join(outdir, "experts.midge"))
    return outdir, {k: z[k] for k in ("ids", "tfall", "gen", "ctx")}


def max_rel(a, b):
    """The reference's logit agreement measure (tools/validate.py:133)."""
    return float(np.max(np.abs(a - b)) / (np.max(np.abs(a)) + 1e-9))


def dev(torch, a):
    """numpy -> CUDA tensor (raw bytes kept)."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda()
