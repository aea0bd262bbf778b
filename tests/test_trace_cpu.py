"""Tracing utilities and debug switches (CPU)."""
import json

import torch

from predicitivecoding_b200 import ops
from predicitivecoding_b200.utils import trace


def test_nvtx_range_is_a_noop_when_off_and_profile_writes_a_trace(tmp_path):
    trace.set_tracing(False)
    with trace.nvtx_range("x"):
        pass
    x = torch.randn(64, 64)
    path = trace.profile_steps(lambda: x @ x, 2, str(tmp_path / "t.json"))
    data = json.load(open(path))
    assert "traceEvents" in data and len(data["traceEvents"]) > 0


def test_deterministic_switch():
    ops.set_deterministic(True)
    assert ops.deterministic()
    ops.set_deterministic(False)
    assert not ops.deterministic()
