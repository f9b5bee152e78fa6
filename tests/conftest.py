import json
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "triton-xdna_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_index() -> dict:
    with open(os.path.join(GOLDEN, "index.json")) as f:
        return json.load(f)


def load_golden(case: str) -> dict:
    return torch.load(os.path.join(GOLDEN, f"{case}.pt"), weights_only=False)


def _numpy_seed42_inputs(a: dict) -> dict:
    """The f32 GEMM example's inputs, regenerated exactly as it makes them
    (np.random.seed(42); A[:, :M] = rand(K, M) * 4; B[:, :N] = rand(K, N) * 4,
    zero padding beyond M / N)."""
    import numpy as np

    np.random.seed(42)
    out = {}
    for name, used in (("A", a["M"]), ("B", a["N"])):
        shape = a[name]["numpy_seed_42"]
        t = np.zeros(shape, dtype=np.float32)
        t[:, :used] = (np.random.rand(shape[0], used) * 4).astype(np.float32)
        out[name] = torch.from_numpy(t)
    return out


def materialize_args(blob: dict) -> dict:
    """Fixture args with the recorded output slot turned into a fresh tensor."""
    args = {}
    regen = {}
    if any(isinstance(v, dict) and "numpy_seed_42" in v for v in blob["args"].values()):
        regen = _numpy_seed42_inputs(blob["args"])
    for k, v in blob["args"].items():
        if k in regen:
            args[k] = regen[k]
            continue
        if isinstance(v, dict) and "empty" in v:
            t = torch.empty_strided(v["empty"], v["stride"], dtype=getattr(torch, v["dtype"]))
            t.fill_(float("nan") if t.is_floating_point() else -1)  # canary
            args[k] = t
        else:
            args[k] = v
    return args


def output_name(blob: dict) -> str:
    return [k for k, v in blob["args"].items() if isinstance(v, dict) and "empty" in v][0]
