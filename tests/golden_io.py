"""Loaders for the committed golden fixtures (tests/golden/)."""

from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


@lru_cache(maxsize=None)
def metadata_cases():
    return json.loads((GOLDEN / "metadata.json").read_text())


@lru_cache(maxsize=None)
def pack_npz():
    return dict(np.load(GOLDEN / "pack.npz"))


@lru_cache(maxsize=None)
def _attention_npz():
    return dict(np.load(GOLDEN / "attention.npz"))


@lru_cache(maxsize=None)
def attention_manifest():
    return json.loads((GOLDEN / "attention_manifest.json").read_text())


def torch_dtype(name: str) -> torch.dtype:
    return torch.float16 if name == "f16" else torch.bfloat16


def attention_case(name: str):
    """Returns (params, tensors): float inputs as torch tensors in the case dtype (CPU), ints as int32, out fp32."""
    params = next(c for c in attention_manifest() if c["name"] == name)
    dt = torch_dtype(params["dtype"])
    z = _attention_npz()
    tensors = {}
    prefix = name + "__"
    for key, arr in z.items():
        if not key.startswith(prefix):
            continue
        k = key[len(prefix):]
        if k == "out":
            tensors[k] = torch.from_numpy(arr.astype(np.float32))
        elif arr.dtype == np.float16:
            tensors[k] = torch.from_numpy(arr)
        elif arr.dtype == np.int16:
            tensors[k] = torch.from_numpy(arr).view(torch.bfloat16)
        else:
            tensors[k] = torch.from_numpy(arr.astype(np.int32))
    assert all(t.dtype == dt for k, t in tensors.items() if t.is_floating_point() and k != "out")
    return params, tensors
