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
