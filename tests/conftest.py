"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a CUDA device);
* puts the repository root on ``sys.path`` so ``import mini_vllm_b200`` and
  ``import oracle`` resolve;
* builds ``libmvb200.so`` (nvcc, sm_100a) and the oracle's ``liboracle.so``
  (gcc) once per session when they are missing or older than their sources.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    import mini_vllm_b200.build as build
    import oracle

    build.build_native()
    build.build_torch_binding()
    oracle.build_oracle()
    yield


@pytest.fixture(scope="session")
def golden():
    import make_golden

    return make_golden.load_golden()


# ---------------------------------------------------------------------------
# numpy <-> torch helpers for bf16 stored as uint16 bits
# ---------------------------------------------------------------------------
TORCH_DTYPES = {"f32": "float32", "f16": "float16", "bf16": "bfloat16"}


def np_to_torch(a: np.ndarray, dtype: str, device="cpu"):
    import torch

    if dtype == "bf16":
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).view(torch.bfloat16)
    else:
        t = torch.from_numpy(np.ascontiguousarray(a).copy())
    return t.to(device)


def torch_to_np(t, dtype: str) -> np.ndarray:
    import torch

    t = t.detach().cpu().contiguous()
    if dtype == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def dtype_tag(torch_dtype) -> str:
    import torch

    return {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}[torch_dtype]
