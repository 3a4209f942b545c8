"""Shared test set-up: the ``gpu`` marker, the package import and the golden fixtures."""

from __future__ import annotations

import importlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_package():
    """The product package lives in the directory ``spikingbrain-cpu_b200``."""
    return importlib.import_module("spikingbrain-cpu_b200")


def golden_cases(kind: str | None = None) -> list[str]:
    meta = json.loads((GOLDEN / "golden_meta.json").read_text())["cases"]
    return sorted(n for n, m in meta.items() if kind is None or m["kind"] == kind)


_NPZ = None


def golden(name: str) -> dict:
    global _NPZ
    if _NPZ is None:
        _NPZ = dict(np.load(GOLDEN / "golden.npz"))
    meta = json.loads((GOLDEN / "golden_meta.json").read_text())["cases"][name]
    out = {k.split("/", 1)[1]: v for k, v in _NPZ.items() if k.startswith(name + "/")}
    out["meta"] = meta
    return out


def golden_cfg3() -> dict:
    """Configuration 3's reference digests (golden_cfg3.json) and sampled output rows (golden_cfg3.npz)."""
    info = json.loads((GOLDEN / "golden_cfg3.json").read_text())
    info["y_rows"] = np.load(GOLDEN / "golden_cfg3.npz")["y_rows"]
    return info


def cfg3_inputs():
    """Configuration 3's seeded inputs, made by the package's workload generators (CPU tensors):
    weight fp32 [4096, 4096], activation fp16 [512, 4096]."""
    info = json.loads((GOLDEN / "golden_cfg3.json").read_text())
    wl = importlib.import_module("spikingbrain-cpu_b200.workloads")
    cfg = wl.CONFIGS[3]
    w = wl.float_weight(cfg["n"], cfg["k"], seed=info["seeds"]["w"])
    x = wl.activation(cfg["m"], cfg["k"], seed=info["seeds"]["x"])
    return w, x


def sha256(a) -> str:
    import hashlib

    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="session")
def sbq():
    return load_package()
