"""Generate the golden fixtures under tests/golden/ from the reference itself.

Run in a container that has the reference tree ($MIDGE_REFERENCE, or the
reference_path of BASELINE.json) and the reference engine built by oracle/Makefile (oracle/_ref/midged):

    python tests/golden/make_golden.py

It produces
  * validate_<case>.npz -- the reference's own end-to-end cases
    (tools/validate.py:30-46): a tiny HF checkpoint from tools/make_tiny.py,
    converted by tools/convert.py, then the reference midged's teacher-forced
    logits for ids [1,17,42,5,99,3,77,12,63,8,120,31] (tfall:) and 24 greedy
    tokens (gen: 24) at --ctx 64 --temp 0.  The converted containers are stored
    in the fixture (a few hundred KB) since the GPU box has no reference tools.
  * c1_tiny.npz: the seeded synthetic gpt-oss-shape model
    written by midge_b200.container (seed 0; its sha256 is stored so a test can
    tell the regenerated files are identical), 32 seeded prompt ids, the
    reference's tfall logits for them and 64 greedy tokens after `ids:`.
Logits are parsed from midged's %.7g text (7 significant digits).
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
from oracle.oracle import reference_dir  # noqa: E402

REF = reference_dir()
MIDGED = os.path.join(ROOT, "oracle", "_ref", "midged")

IDS = [1, 17, 42, 5, 99, 3, 77, 12, 63, 8, 120, 31]  # tools/validate.py:39
CASES = [  # tools/validate.py:30-44: (name, make_tiny args, convert flags)
    ("bf16_f32", ["--format", "bf16"], ["--experts", "f32", "--dense", "f32"]),
    ("bf16_q8r", ["--format", "bf16"], ["--experts", "q8r", "--dense", "q8r"]),
    ("bf16_q4g32", ["--format", "bf16"], ["--experts", "q4g32", "--dense", "q8r"]),
    ("bf16_mxfp4", ["--format", "bf16"], ["--experts", "mxfp4", "--dense", "q8r"]),
    ("mxfp4_blocks", ["--format", "mxfp4"], ["--experts", "mxfp4", "--dense", "q8r"]),
    ("mixtral_q4g32", ["--arch", "mixtral"], ["--experts", "q4g32", "--dense", "q8r"]),
    ("qwen3moe_q4g32", ["--arch", "qwen3-moe"], ["--experts", "q4g32", "--dense", "q8r"]),
]


class Engine:
    """The reference midged over its stdin/stdout protocol (engine/midge.c:15-24)."""

    def __init__(self, model_dir, ctx):
        self.p = subprocess.Popen([MIDGED, model_dir, "--ctx", str(ctx), "--temp", "0", "--no-stats"],
                                  stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                  text=True, bufsize=1, env=dict(os.environ, OMP_NUM_THREADS="1"))
        while self._line() != "READY":
            pass

    def _line(self):
        ln = self.p.stdout.readline()
        if not ln:
            raise RuntimeError("reference midged died")
        return ln.rstrip("\n")

    def send(self, s):
        self.p.stdin.write(s + "\n")
        self.p.stdin.flush()

    def tfall(self, ids):
        self.send("tfall: " + " ".join(map(str, ids)))
        out = [np.array(self._line()[2:].split(), np.float32) for _ in ids]
        assert self._line().startswith("DONE")
        return np.stack(out)

    def ids(self, ids):
        self.send("ids: " + " ".join(map(str, ids)))
        ln = self._line()
        assert ln.startswith("OK"), ln

    def gen(self, n):
        self.send(f"gen: {n}")
        toks = []
        while True:
            ln = self._line()
            if ln.startswith("T "):
                toks.append(int(ln[2:]))
            elif ln.startswith("DONE"):
                return np.array(toks, np.int32)

    def close(self):
        self.send("quit")
        self.p.wait(timeout=30)


def sha(path):
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


def validate_cases(tmp):
    for name, mk_args, conv in CASES:
        hf = os.path.join(tmp, "hf-" + "-".join(mk_args).replace("--", ""))
        if not os.path.exists(os.path.join(hf, "model.safetensors")):
            subprocess.run([sys.executable, os.path.join(REF, "tools/make_tiny.py"), hf, *mk_args], check=True,
                           capture_output=True)
        md = os.path.join(tmp, "m_" + name)
        subprocess.run([sys.executable, os.path.join(REF, "tools/convert.py"), hf, md, *conv], check=True,
                       capture_output=True)
        e = Engine(md, 64)  # tools/validate.py:46,61
        logits = e.tfall(IDS)
        toks = e.gen(24)
        e.close()
        np.savez_compressed(
            os.path.join(HERE, f"validate_{name}.npz"),
            dense=np.fromfile(os.path.join(md, "dense.midge"), np.uint8),
            experts=np.fromfile(os.path.join(md, "experts.midge"), np.uint8),
            ids=np.array(IDS, np.int32), tfall=logits, gen=toks, ctx=np.int32(64))
        print(f"validate_{name}: gen={toks[:8]}...")


def c1_case(tmp):
    from midge_b200 import container as ct
    spec, edt = ct.config_spec("c1_tiny")
    md = os.path.join(tmp, "c1")
    ct.write_synthetic_model(md, spec, edt, seed=0)
    prompt = np.random.default_rng(1234).integers(0, spec["vocab"], 32).astype(np.int32)
    ctx = 256
    e = Engine(md, ctx)
    logits = e.tfall(prompt)
    e.close()
    e = Engine(md, ctx)
    e.ids(prompt)
    toks = e.gen(64)
    e.close()
    np.savez_compressed(os.path.join(HERE, "c1_tiny.npz"), prompt=prompt, tfall=logits, gen=toks, ctx=np.int32(ctx),
                        sha_dense=sha(os.path.join(md, "dense.midge")),
                        sha_experts=sha(os.path.join(md, "experts.midge")))
    print("c1_tiny: gen", toks[:8], "...")


def main():
    if not os.path.exists(MIDGED):
        raise SystemExit("build the reference first: make -f oracle/Makefile")
    tmp = tempfile.mkdtemp(prefix="midge_golden_")
    try:
        validate_cases(tmp)
        c1_case(tmp)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    main()
