import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ai-agent-framework_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def built_lib():
    import b2decode
    if not os.path.exists(b2decode.LIB_PATH):
        b2decode.build()
    return b2decode.lib()


@pytest.fixture(scope="session")
def oracle_lib():
    import goref
    goref.build()
    return goref


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


def _write(model_dir, name, shape, seed=0):
    from b2decode import gguf_writer as gw
    path = os.path.join(str(model_dir), f"{name}-s{seed}.gguf")
    if not os.path.exists(path):
        gw.write_model(path, shape, seed=seed)
    return path


@pytest.fixture(scope="session")
def tiny_gguf(model_dir):
    from b2decode import gguf_writer as gw
    return _write(model_dir, "tiny", gw.SHAPES["tiny"])


@pytest.fixture(scope="session")
def tiny_q4_gguf(model_dir):
    from b2decode import gguf_writer as gw
    return _write(model_dir, "tiny-llama-q4", gw.SHAPES["tiny-llama-q4"])


@pytest.fixture(scope="session")
def write_model(model_dir):
    def f(name, shape, seed=0):
        return _write(model_dir, name, shape, seed)
    return f
