"""The reference's own CPU layer loop as a checker (test infrastructure).

oracle/_ref/ref_session is engine/src/session.cpp (Session::step / forward and
the host helpers it calls) compiled from the reference sources by
`make -C oracle ref`, driven through a stand-in for class GPU whose shader
calls are the oracle's restatement (oracle/ref_session.cpp).  These helpers run
it on a container and compare the oracle against it; tests/golden/
reference_logits.npz keeps its logits for hosts where it is not built.
"""
from __future__ import annotations

import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_SESSION = os.path.join(ROOT, "oracle", "_ref", "ref_session")
FIXTURE = os.path.join(HERE, "golden", "reference_logits.npz")

# teacher-forced positions per configuration (the prompt's first n tokens)
POSITIONS = {"tiny_q8": 8, "tiny_q4": 8, "tiny_flat_q8": 8, "tiny_moe_q4": 8, "tiny_t3": 8,
             "c0": 6, "c0r": 6, "c1": 6, "c2": 6, "c3": 2, "c4": 6}


def available() -> bool:
    return os.access(REF_SESSION, os.X_OK)


def run(path: str, kv_bits: int, tokens, literal_matvec: bool = True) -> np.ndarray:
    """Logits (len(tokens) x vocab floats) of the reference layer loop,
    teacher-forced at positions 0..n-1.  A q8 cache selects the reference's
    KV8_SIM=1 read-time quantiser (session.cpp:51-69); a q16 cache is the CPU
    path's float K/V."""
    env = dict(os.environ)
    env.pop("KV8_SIM", None)
    if kv_bits == 8:
        env["KV8_SIM"] = "1"
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "logits.bin")
        cmd = [REF_SESSION, path, "1" if literal_matvec else "0", out, str(len(tokens))] + [str(int(t)) for t in tokens]
        r = subprocess.run(cmd, env=env, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("ref_session failed (%d): %s" % (r.returncode, r.stderr[-2000:]))
        return np.fromfile(out, np.float32).reshape(len(tokens), -1)


def oracle_logits(om, kv_bits: int, tokens, mode: int) -> np.ndarray:
    """The oracle session in `mode` (0 canonical, 1 literal, 2 literal with
    the float cache), teacher-forced like `run`."""
    import oracle
    h = oracle.lib().orc_session_new(om._h, kv_bits, mode)
    if not h:
        raise RuntimeError("oracle session refused")
    s = oracle.Session.__new__(oracle.Session)
    s._h, s.vocab, s.model = h, om.info.vocab, om
    try:
        return np.stack([s.step(t, p) for p, t in enumerate(tokens)])
    finally:
        s.close()


def literal_mode(kv_bits: int) -> int:
    """The oracle's literal mode that restates the reference CPU path's cache:
    the packed q8 cache equals KV8_SIM's read-time grid, a q16 cache is float."""
    return 1 if kv_bits == 8 else 2
