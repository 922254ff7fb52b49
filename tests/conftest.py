import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (runs the CUDA path)")
    config.addinivalue_line("markers", "ref: needs the compiled reference oracle/_ref/libdsref.so")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    import oracle as O
    for it in items:
        if "gpu" in it.keywords and not HAS_GPU:
            it.add_marker(pytest.mark.skip(reason="no CUDA device"))
        if "ref" in it.keywords and not O.ref_available():
            it.add_marker(pytest.mark.skip(reason="oracle/_ref/libdsref.so not built (reference tree absent)"))


@pytest.fixture(scope="session")
def orc():
    import oracle as O
    return O.oracle()


@pytest.fixture(scope="session")
def cuda_ctx():
    from ds_ocr_b200 import cuda
    ctx = cuda.Context(0)
    yield ctx
    ctx.close()


@pytest.fixture(scope="session")
def moe_weights():
    """One full-size MoE layer (64 experts + shared), generated once."""
    from ds_ocr_b200 import synth
    return synth.MoeWeights(synth.Dims(), 1)


def rel_l2(a, b):
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
