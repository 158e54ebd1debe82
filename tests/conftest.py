import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("llm-mojo_b200", "oracle", "tests"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libmoe_b200.so")
    config.addinivalue_line("markers", "slow: long CPU oracle run")


@pytest.fixture(scope="session")
def ctx():
    import moe_b200
    c = moe_b200.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def full_layer(ctx):
    """Gemma-4-26B-A4B-shaped layer (d=2816, F=704, E=128, top-8), seed 0, on the GPU
    plus a host copy for the oracle."""
    import oracle as O
    import synth
    dev = synth.make_layer(ctx, seed=0)
    host = synth.to_host(dev)
    check_layer_stats(host)
    return dev, host, O.make_layer(host)


def check_layer_stats(host):
    """The dequantised weights must look like N(0, 0.02): catches a layer
    built from memory the generator had not written yet."""
    import numpy as np
    p = host["gu_p"][: 1408 * 1408].astype(np.int32)
    s = host["gu_s"][: 1408 * 88]
    v = (np.stack([(p & 15) - 8, (p >> 4) - 8], 1).reshape(-1, 32) * s[:, None])
    assert 0.018 < float(v.std()) < 0.022, float(v.std())
    assert 0.005 < float(host["dn_s"].mean()) < 0.009


@pytest.fixture(scope="session")
def small_layer(ctx):
    """Reduced layer (d=256, F=64, E=16, top-4) for fast edge-case sweeps."""
    import oracle as O
    import synth
    dev = synth.make_layer(ctx, d=256, F_=64, E_=16, top_k=4, seed=3)
    host = synth.to_host(dev)
    return dev, host, O.make_layer(host)
