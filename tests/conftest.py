import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device")
    config.addinivalue_line("markers", "slow: full-size model cases")


@pytest.fixture(scope="session")
def tiny_models():
    """Seeded tiny decoders in q8/q6/q4: head_dim 128 like the benchmark model,
    but 4 q heads over 2 kv heads (GQA group 2; the benchmark model has group 8,
    covered by tests/test_gpu_bench_shapes.py)."""
    from rapidocrvl_b200 import synth

    return {q: synth.ensure("tiny", q) for q in ("q8", "q6", "q4")}


@pytest.fixture(scope="session")
def oracle_lib():
    import pyoracle

    return pyoracle.lib()
