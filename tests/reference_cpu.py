"""Test helper: run pieces of the reference's Python search drivers on the CPU.

The reference's orchestrators (hive_fnn/fnn_mcts_orchestrator.py) hard-code
``device="cuda"`` in their tensor factories and call ``.cuda()`` on inputs.
``torch_on_cpu`` maps both to the CPU while a reference function runs and
records every ``torch.rand`` draw; ``reference_module`` imports a reference
module with the reference tree on ``sys.path`` for the import only (the tree
has a ``tests`` package of its own that must not shadow this repository's).
Used by the fixture generators in tests/golden/ and by CPU tests that compare
this package's host-side search logic with the reference's own functions.
"""
from __future__ import annotations

import contextlib
import importlib
import sys

import torch

from oracle import oracle as O


def reference_available() -> bool:
    return O.reference_available()


def reference_module(name: str):
    """Import `name` from the reference tree (e.g. "hive_fnn.fnn_mcts_orchestrator")."""
    saved = list(sys.path)
    sys.path.append(O.reference_dir())
    try:
        return importlib.import_module(name)
    finally:
        sys.path[:] = saved


@contextlib.contextmanager
def torch_on_cpu(draws: list | None = None):
    """Map device="cuda" factory calls and Tensor.cuda() to the CPU and record
    torch.rand draws into `draws` (a list) while the block runs."""
    saved = {k: getattr(torch, k) for k in ("zeros", "ones", "full", "arange", "rand")}
    saved_cuda = torch.Tensor.cuda

    def strip(fn, record=False):
        def f(*a, **k):
            if k.get("device") is not None and str(k["device"]).startswith("cuda"):
                k["device"] = "cpu"
            out = fn(*a, **k)
            if record and draws is not None:
                draws.append(out.numpy().copy())
            return out
        return f

    for k, fn in saved.items():
        setattr(torch, k, strip(fn, record=(k == "rand")))
    torch.Tensor.cuda = lambda self, *a, **k: self
    try:
        yield
    finally:
        for k, fn in saved.items():
            setattr(torch, k, fn)
        torch.Tensor.cuda = saved_cuda
