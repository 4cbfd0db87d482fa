"""Rewrite a converted model's experts.midge with ue8m0 group scales.

The midge converter stores every MXFP4 group scale as an f16 power of two
(2^e, e in [-24, 15]; tools/convert.py:37-53 of the reference), which the
GPU loader re-expresses as one ue8m0 byte (e + 127) per 32 columns when it
uploads the experts.  This tool does that once on disk: it writes an
experts.midge of dtype "mxfp4e8" (same nibbles and biases, each scale blob
half as long, offsets from the same deterministic layout rule) that the
loader copies to HBM as is.  Opt-in: the reference midged does not read the
new dtype, so the original files stay the interchange format.  A scale that
is not zero or a positive power of two cannot be re-expressed exactly and
stops the conversion.

    python -m midge_b200.convert_ue8m0 <model_dir> <out_dir>
"""
from __future__ import annotations

import os
import shutil
import sys

import numpy as np

from .container import ExpertLayout, ModelDir, write_experts


def f16_to_ue8m0(s16: np.ndarray) -> np.ndarray:
    """f16 scale bits -> ue8m0 codes; ValueError unless every scale is +0 or a
    positive power of two (normal or subnormal)."""
    u = np.asarray(s16, np.uint16)
    exp = (u >> 10) & 0x1F
    man = u & 0x3FF
    sign = u >> 15
    zero = u == 0
    normal_pow2 = (sign == 0) & (exp > 0) & (exp < 31) & (man == 0)
    sub = (sign == 0) & (exp == 0) & (man != 0) & ((man & (man - 1)) == 0)
    if not np.all(zero | normal_pow2 | sub):
        bad = int(np.count_nonzero(~(zero | normal_pow2 | sub)))
        raise ValueError(f"{bad} scales are not zero or a power of two")
    e = np.where(normal_pow2, exp.astype(np.int32) - 15, 0)
    e = np.where(sub, np.log2(np.maximum(man, 1)).astype(np.int32) - 24, e)
    return np.where(zero, 0, e + 127).astype(np.uint8)


def convert(src: str, dst: str) -> str:
    md = ModelDir(src)
    try:
        if md.expert_dt != "mxfp4":
            raise ValueError(f"experts are {md.expert_dt}, not mxfp4")
        s = md.spec
        a = md.layout
        b = ExpertLayout("mxfp4e8", s["hidden"], s["moe"]["ffn"], s["moe"]["experts"], s["n_layers"])
        src_blob = md.expert_blob()
        out = np.zeros(b.total, np.uint8)
        for layer in range(a.n_layers):
            for e in range(a.n_experts):
                for m in ExpertLayout.MATS:
                    r, c = a.rows[m], a.cols[m]
                    nd, ns = r * c // 2, r * (c // 32)
                    o, p = a.offset(layer, e, m, "data"), b.offset(layer, e, m, "data")
                    out[p:p + nd] = src_blob[o:o + nd]
                    o, p = a.offset(layer, e, m, "scales"), b.offset(layer, e, m, "scales")
                    out[p:p + ns] = f16_to_ue8m0(src_blob[o:o + 2 * ns].view(np.uint16))
                    o, p = a.offset(layer, e, m, "bias"), b.offset(layer, e, m, "bias")
                    out[p:p + 4 * r] = src_blob[o:o + 4 * r]
        os.makedirs(dst, exist_ok=True)
        write_experts(os.path.join(dst, "experts.midge"), b, out)
        shutil.copyfile(os.path.join(src, "dense.midge"), os.path.join(dst, "dense.midge"))
        for extra in ("spec.json", "tokenizer.json", "tokenizer_config.json"):
            if os.path.exists(os.path.join(src, extra)):
                shutil.copyfile(os.path.join(src, extra), os.path.join(dst, extra))
    finally:
        md.close()
    return dst


if __name__ == "__main__":
    if len(sys.argv) != 3:
        sys.exit(__doc__)
    print(convert(sys.argv[1], sys.argv[2]))
