"""Test setup: marker registration and import paths.

`gpu` tests need a CUDA device and run only with `-m gpu`; every other test runs on
the CPU.  The package lives in navi-tts_b200/ (a directory name that is not a
Python identifier), so its parent is put on sys.path here and in the entry points.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "navi-tts_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


@pytest.fixture(scope="session")
def small_navi(tmp_path_factory):
    from navi_b200 import model_spec
    path = tmp_path_factory.mktemp("navi") / "small.navi"
    model_spec.write_synthetic(path, model_spec.small_config())
    return str(path)


@pytest.fixture(scope="session")
def full_navi(tmp_path_factory):
    """The benchmark-size model (configs[1]-[3] shapes), written once per session (~2 GB)."""
    from navi_b200 import model_spec
    path = os.environ.get("NAVI_BENCH_NAVI", "/tmp/navi_bench_full.navi")
    if not os.path.exists(path):
        model_spec.write_synthetic(path, model_spec.full_config(1024))
    return path


@pytest.fixture(scope="session")
def layer_navi(tmp_path_factory):
    """configs[0]'s model: the benchmark shapes with one talker layer, talker weights from seed 0."""
    from navi_b200 import model_spec
    path = tmp_path_factory.mktemp("navi") / "layer.navi"
    model_spec.write_synthetic(path, model_spec.layer_config(), seed_offset=model_spec.LAYER_SEED_OFFSET)
    return str(path)
