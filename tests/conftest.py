"""Shared pytest setup: the ``gpu`` marker, repo imports and golden-fixture loading."""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


_TORCH_DTYPE = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def golden_manifest() -> dict:
    return json.loads((GOLDEN / "manifest.json").read_text())


def load_golden(name: str) -> tuple[dict, dict]:
    """Return (tensors, meta) of one golden case; 16-bit floats restored."""
    meta = golden_manifest()[name]
    data = np.load(GOLDEN / f"{name}.npz")
    out = {}
    for k in data.files:
        arr = data[k]
        tag = meta.get("dtypes", {}).get(k)
        if tag in ("float16", "bfloat16"):
            out[k] = torch.from_numpy(arr.view(np.int16).copy()).view(_TORCH_DTYPE[tag])
        else:
            out[k] = torch.from_numpy(arr.copy())
    return out, meta


def decode_cases() -> list[str]:
    return sorted(k for k, v in golden_manifest().items()
                  if not k.startswith("_") and ("expected_torch" in _files(k) or "expected_eager" in _files(k)))


def _files(name: str) -> list[str]:
    return list(np.load(GOLDEN / f"{name}.npz").files)


def reference_root() -> Path | None:
    """Where the reference's Python runtime can be imported from: the checkout
    named by LLM_SERVING_RUNTIME_ROOT, else the unmodified copy that build()
    stages in baseline/_ref (it travels with the working tree)."""
    for root in (os.environ.get("LLM_SERVING_RUNTIME_ROOT"), str(REPO / "baseline" / "_ref")):
        if root and (Path(root) / "runtime" / "phase2" / "paged_attention_triton.py").exists():
            return Path(root)
    return None
