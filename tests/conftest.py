import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "vc4-gles2-inference_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); parity against the CPU oracle")


@pytest.fixture(scope="session")
def tiny_paths(tmp_path_factory):
    """The five tiny parity containers, written by the MMCF writer."""
    from vc4b200 import synth, mmcf_writer
    d = tmp_path_factory.mktemp("mmcf")
    out = {}
    for key, cfg in synth.TINY_CONFIGS.items():
        p = str(d / (key + ".mmcf"))
        mmcf_writer.write_config(cfg, p)
        out[key] = p
    return out


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)


def full_model_path(key: str) -> str:
    """The container of a benchmark configuration at its full shape, written
    once per host by the MMCF writer (c3b32 shares c3's container)."""
    import tempfile
    from vc4b200 import mmcf_writer, synth
    cfg = synth.CONFIGS[key]
    key = cfg.extra.get("model", "c3" if key == "c3b32" else key)
    cfg = synth.CONFIGS[key]
    d = os.path.join(tempfile.gettempdir(), "vc4b200_models")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, "%s_%d.mmcf" % (key, cfg.seed))
    if not os.path.exists(p):
        tmp = p + ".%d.tmp" % os.getpid()
        mmcf_writer.write_config(cfg, tmp)
        os.replace(tmp, p)
    return p
