"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run here, where the reference tree is mounted (it does not exist on the GPU
host).  For every synthetic configuration it

  1. writes the seeded HuggingFace directory (vc4b200.synth),
  2. packs it with the reference's own packer, unchanged:
       python engine/tools/mmcf_pack.py --in DIR --out F --quant Q --seq S
              --rms-eps 1e-6 --template plain [--head-dedup] --verify
  3. records the container's sha256 and size, and
  4. loads it with the reference's own C++ loader (oracle/_ref, built from
     engine/src/model.cpp et al. by oracle/Makefile) and records the decoded
     summary (shapes, scales, FNV digests of every tensor's values).

It also lifts the x_pack byte vectors out of engine/tests/test_xformat.cpp.
Output: tests/golden/golden.json.  With --session it instead runs the
reference's own CPU layer loop (engine/src/session.cpp, built into
oracle/_ref/ref_session) on every configuration's seeded prompt and writes
its logits to tests/golden/reference_logits.npz.

    python tests/golden/make_golden.py [--ref REFERENCE_CHECKOUT] [--full]

--ref defaults to the environment variable VC4_REFERENCE.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "vc4-gles2-inference_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from vc4b200 import synth  # noqa: E402
import oracle  # noqa: E402


def xformat_vectors(ref: str) -> list:
    """CHECK_BYTES(pack({values}, XFormat::F), bytes...) cases of test_xformat.cpp."""
    text = open(os.path.join(ref, "engine/tests/test_xformat.cpp")).read()
    text = re.sub(r"//[^\n]*", "", text)
    out = []
    for m in re.finditer(r"CHECK_BYTES\(\s*pack\(\{([^}]*)\},\s*XFormat::(\w+)\)\s*,(.*?)\);", text, re.S):
        vals = [float(v.strip().rstrip("f")) for v in m.group(1).split(",") if v.strip()]
        raw = [v.strip() for v in m.group(3).split(",") if v.strip()]
        out.append({"format": m.group(2), "values": vals, "bytes": [int(b, 0) for b in raw]})
    return out


def pack_with_reference(ref: str, cfg: synth.Config, workdir: str) -> tuple:
    d = os.path.join(workdir, cfg.key + "_hf")
    synth.write_hf_dir(d, cfg)
    out = os.path.join(workdir, cfg.key + ".mmcf")
    cmd = [sys.executable, os.path.join(ref, "engine/tools/mmcf_pack.py"), "--in", d, "--out", out,
           "--quant", cfg.quant, "--seq", str(cfg.seq), "--rms-eps", "1e-6", "--template", "plain",
           "--verify"]
    if cfg.head_dedup:
        cmd.append("--head-dedup")
    if cfg.extra.get("q8_row"):
        cmd.append("--q8-row-scale")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise SystemExit("reference packer failed for %s:\n%s\n%s" % (cfg.key, r.stdout, r.stderr))
    return out, r.stdout


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("VC4_REFERENCE"))
    ap.add_argument("--full", action="store_true", help="also pack the five full-size configurations")
    ap.add_argument("--only", default="", help="comma-separated configurations to (re)pack; the others keep "
                                               "their recorded entries")
    ap.add_argument("--session", action="store_true",
                    help="only record the reference layer loop's logits (oracle/_ref/ref_session) into "
                         "reference_logits.npz")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(os.path.join(args.ref, "engine", "src")):
        raise SystemExit("name the reference checkout with --ref or VC4_REFERENCE")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", "REF=" + args.ref], check=True)
    if args.session:
        reference_session_logits()
        return
    golden = {"xformat": xformat_vectors(args.ref), "containers": {}}
    cfgs = dict(synth.TINY_CONFIGS)
    if args.full:
        cfgs.update({k: v for k, v in synth.CONFIGS.items() if k in ("c0", "c0r", "c1", "c2", "c3", "c4")})
    if args.only:
        allc = dict(synth.TINY_CONFIGS, **synth.CONFIGS)
        cfgs = {k: allc[k] for k in args.only.split(",")}
    with tempfile.TemporaryDirectory() as wd:
        for key, cfg in cfgs.items():
            path, log = pack_with_reference(args.ref, cfg, wd)
            data = open(path, "rb").read()
            entry = {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data),
                     "packer_log": [l for l in log.splitlines() if l.startswith(("residual", "ffn hidden", "rope", "verify"))],
                     "reference_load": oracle.ref_summary(path)}
            golden["containers"][key] = entry
            print(key, entry["bytes"], entry["sha256"][:16], flush=True)
    prev = {}
    gp = os.path.join(HERE, "golden.json")
    if os.path.exists(gp):
        prev = json.load(open(gp))
    for k, v in prev.get("containers", {}).items():
        golden["containers"].setdefault(k, v)
    with open(gp, "w") as f:
        json.dump(golden, f, indent=1, sort_keys=True)


def reference_session_logits() -> None:
    """The reference's own CPU layer loop (engine/src/session.cpp compiled by
    `make -C oracle ref`, shader calls through the oracle's restatement) on
    the seeded prompts of every configuration, teacher-forced; the logits are
    on the q16 grid and are stored as int16 (value * 256)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import numpy as np
    import refsession
    from vc4b200 import mmcf_writer
    out = {}
    cfgs = dict(synth.TINY_CONFIGS, **{k: synth.CONFIGS[k] for k in ("c0", "c0r", "c1", "c2", "c3", "c4")})
    with tempfile.TemporaryDirectory() as wd:
        for key, n in refsession.POSITIONS.items():
            cfg = cfgs[key]
            path = os.path.join(wd, key + ".mmcf")
            mmcf_writer.write_config(cfg, path)
            toks = synth.prompt_tokens(cfg)[:n]
            lg = refsession.run(path, cfg.kv_bits, toks)
            q = np.rint(lg * 256.0)
            assert np.array_equal(q / 256.0, lg) and np.abs(q).max() < 32768
            out[key] = q.astype(np.int16)
            out[key + "_tokens"] = np.array(toks, np.int32)
            print(key, lg.shape, flush=True)
    np.savez_compressed(os.path.join(HERE, "reference_logits.npz"), **out)


if __name__ == "__main__":
    main()
