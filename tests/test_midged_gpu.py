"""The drop-in process: midge_b200/bin/midged driven over the reference's
stdin/stdout protocol exactly as the reference's own acceptance test drives
its engine (tools/validate.py:58-104: tfall: the fixed ids, then gen: 24),
on the seven golden cases made by the reference midged; its exit codes
(engine/midge.c:209-211, :136, :195-201, :554-555); --bench; temperature /
top-p generation on the device; and the --seqs extension (several contexts in
one process) against single-sequence runs."""
import os
import subprocess

import numpy as np
import pytest

from midge_b200 import container as ct
from oracle import oracle as orc
from tests.helpers import VALIDATE_CASES, load_validate_case, max_rel

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MIDGED = os.path.join(ROOT, "midge_b200", "bin", "midged")
IDS = [1, 17, 42, 5, 99, 3, 77, 12, 63, 8, 120, 31]  # tools/validate.py:39


class Engine:
    def __init__(self, model_dir, *args):
        self.p = subprocess.Popen([MIDGED, model_dir, *map(str, args)], stdin=subprocess.PIPE,
                                  stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, bufsize=1)
        while True:
            ln = self.line()
            if ln == "READY":
                break
            assert ln == "LOADING", ln

    def line(self):
        ln = self.p.stdout.readline()
        if not ln:
            raise RuntimeError("engine died: " + self.p.stderr.read())
        return ln.rstrip("\n")

    def send(self, s):
        self.p.stdin.write(s + "\n")
        self.p.stdin.flush()

    def tfall(self, ids):
        self.send("tfall: " + " ".join(map(str, ids)))
        out = []
        for _ in ids:
            ln = self.line()
            assert ln.startswith("L "), ln
            out.append(np.array([float(v) for v in ln[2:].split()], np.float32))
        assert self.line().startswith("DONE")
        return np.stack(out)

    def ids(self, ids):
        self.send("ids: " + " ".join(map(str, ids)))
        ln = self.line()
        assert ln.startswith("OK "), ln
        return int(ln[3:])

    def gen(self, n):
        self.send(f"gen: {n}")
        toks = []
        while True:
            ln = self.line()
            if ln.startswith("T "):
                toks.append(int(ln[2:]))
            elif ln.startswith("DONE"):
                return toks, ln

    def cmd(self, s):
        self.send(s)
        return self.line()

    def genall(self, n, seqs=()):
        self.send(f"genall: {n} " + " ".join(map(str, seqs)))
        out = {}
        while True:
            ln = self.line()
            if ln.startswith("TS "):
                _, s, t = ln.split()
                out.setdefault(int(s), []).append(int(t))
            elif ln.startswith("DONE"):
                return out, ln

    def close(self):
        try:
            self.send("quit")
        except Exception:
            pass
        return self.p.wait(timeout=60)


@pytest.mark.parametrize("case", VALIDATE_CASES)
def test_midged_validate_cases(torch_cuda, case, tmp_path):
    md, g = load_validate_case(case, str(tmp_path / "m"))
    eng = Engine(md, "--ctx", int(g["ctx"]), "--temp", "0", "--no-stats")
    lg = eng.tfall(list(g["ids"]))
    toks, done = eng.gen(len(g["gen"]))
    assert eng.close() == 0
    for i in range(len(g["ids"])):  # the reference's own bar (tools/validate.py:133-136) and the 1e-3 target
        assert np.allclose(g["tfall"][i], lg[i], rtol=2e-3, atol=2e-3)
        assert max_rel(g["tfall"][i], lg[i]) < 1e-3
    assert toks == list(g["gen"])
    assert done.split()[2] == str(len(g["gen"]))
    assert os.path.exists(os.path.join(md, "usage.bin"))


def _c1(tmp_path, seed=0):
    spec, edt = ct.config_spec("c1_tiny")
    return ct.write_synthetic_model(str(tmp_path / "c1"), spec, edt, seed=seed)


def test_midged_exit_codes(torch_cuda, tmp_path):
    def run(args, stdin=""):
        r = subprocess.run([MIDGED, *args], input=stdin, capture_output=True, text=True, errors="replace",
                           timeout=120)
        return r.returncode, r.stderr

    rc, err = run([str(tmp_path / "missing")])
    assert rc == 2 and "cannot open" in err                       # engine/midge.c:209-211
    md = _c1(tmp_path)
    bad = tmp_path / "bad"
    bad.mkdir()
    spec, edt = ct.config_spec("c1_tiny")
    spec["hidden"] = 0                                             # invalid spec: exit 3 (engine/midge.c:136)
    rng = np.random.default_rng(0)
    ct.write_dense(str(bad / "dense.midge"), spec, [("embed", "f32", [4], np.zeros(4, np.float32).tobytes(), b"")])
    os.link(os.path.join(md, "experts.midge"), bad / "experts.midge")
    rc, err = run([str(bad)])
    assert rc == 3, err
    rc, err = run([md, "--ctx", "64"], "ids: 1 2 999999\n")      # token out of range: exit 4 (:555)
    assert rc == 4, err
    rc, err = run([md, "--ctx", "8"], "ids: 1 2 3 4 5 6 7 8 9 10\n")  # context full: exit 4 (:554)
    assert rc == 4, err
    r = subprocess.run([MIDGED, "--bench"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.startswith("BENCH q4g32_gbps=")
    assert float(r.stdout.split("=")[1].split()[0]) > 50.0


def test_midged_sampling_on_device(torch_cuda, tmp_path):
    """--temp / --topp / --seed and set: draw on the device: the same seed
    gives the same tokens, set: reseeds, and every drawn token lies inside
    the oracle's top-p nucleus at that position (the oracle teacher-forced
    along the engine's tokens)."""
    md = _c1(tmp_path)
    prompt = list(np.random.default_rng(4).integers(0, 1024, 20))
    temp, topp = 0.9, 0.8

    def run(seed, reseed=None):
        eng = Engine(md, "--ctx", 128, "--temp", temp, "--topp", topp, "--seed", seed, "--no-stats")
        eng.ids(prompt)
        a, _ = eng.gen(12)
        b = None
        if reseed is not None:
            assert eng.cmd(f"set: {temp} {topp} {reseed}") == "OK set"
            b, _ = eng.gen(6)
        assert eng.close() == 0
        return a, b

    a1, _ = run(7)
    a2, b2 = run(7, reseed=99)
    assert a1 == a2
    a3, _ = run(8)
    assert a3 != a1
    om = orc.OracleModel(md, 128)
    lg = om.prefill(prompt)
    for t in a1:
        e = np.exp((lg.astype(np.float64) - lg.max()) / temp)
        p = e / e.sum()
        order = np.argsort(-p, kind="stable")
        n = int(np.searchsorted(np.cumsum(p[order]), min(1.0, topp + 1e-3))) + 1
        assert t in set(order[:n].tolist())
        lg = om.forward(int(t))
    om.close()


def test_midged_multiple_sequences(torch_cuda, tmp_path):
    """--seqs 3: three contexts in one engine.  Interleaved gen: on two
    sequences and genall: over three give, for every sequence, exactly the
    tokens a single-sequence engine gives it -- greedy, and sampled (sequence
    s draws with the seed the extension derives for it)."""
    md = _c1(tmp_path)
    rng = np.random.default_rng(11)
    prompts = [list(rng.integers(0, 1024, n)) for n in (9, 23, 5)]

    def single(i, n, *flags):
        eng = Engine(md, "--ctx", 128, "--no-stats", *flags)
        eng.ids(prompts[i])
        toks, _ = eng.gen(n)
        assert eng.close() == 0
        return toks

    greedy = [single(i, 8, "--temp", 0) for i in range(3)]
    eng = Engine(md, "--ctx", 128, "--no-stats", "--seqs", 3, "--temp", 0)
    for i in range(3):
        assert eng.cmd(f"seq: {i}") == f"OK seq {i}"
        eng.ids(prompts[i])
    eng.cmd("seq: 0")
    a, _ = eng.gen(4)
    eng.cmd("seq: 1")
    b, _ = eng.gen(4)
    eng.cmd("seq: 0")
    a2, _ = eng.gen(4)
    assert a + a2 == greedy[0]
    out, done = eng.genall(4, [2, 1])
    assert out[2] == greedy[2][:4] and b + out[1] == greedy[1]
    assert done.split()[2] == "8"
    assert eng.close() == 0

    seed, temp, topp = 42, 0.8, 0.9
    derived = [seed] + [((seed ^ (0x9E3779B97F4A7C15 * s)) & 0xFFFFFFFFFFFFFFFF) | 1 for s in (1, 2)]
    sampled = [single(i, 6, "--temp", temp, "--topp", topp, "--seed", derived[i]) for i in range(3)]
    eng = Engine(md, "--ctx", 128, "--no-stats", "--seqs", 3, "--temp", temp, "--topp", topp, "--seed", seed)
    for i in range(3):
        eng.cmd(f"seq: {i}")
        eng.ids(prompts[i])
    out, _ = eng.genall(6)
    assert eng.close() == 0
    for i in range(3):
        assert out[i] == sampled[i], i
