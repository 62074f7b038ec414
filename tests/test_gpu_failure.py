"""Failure detection without a GPU fault: a bounded wait that runs out reports, never hangs.

Every pipeline wait of the kernels is bounded; when one runs out the CTA raises its abort
flag and the device error word's timeout bit, and the kernel returns.  The self-test makes
a wait run out on an mbarrier nothing arrives on (short limit) and checks the status the
host reads; the context stays usable for the next launch.
"""
from __future__ import annotations

import pytest
import torch

import jetspec_b200 as jb
from jetspec_b200 import _lib, workloads

pytestmark = pytest.mark.gpu
TIMEOUT_BIT = 4


def test_wait_that_runs_out_reports_and_returns():
    jb.read_device_errors()  # clear
    completed, abort, cycles = _lib.selftest_bounded_wait(2_000_000)
    assert completed == 0
    assert abort == 1
    assert cycles >= 2_000_000
    assert jb.read_device_errors() & TIMEOUT_BIT
    assert jb.read_device_errors() == 0  # read-and-clear


def test_context_usable_after_timeout():
    _lib.selftest_bounded_wait(1_000_000)
    jb.read_device_errors()
    dev = torch.device("cuda", 0)
    batch = workloads.config1()
    q, k, v = workloads.make_tensors(batch, dev)
    out = jb.packed_tree_attention_gqa(q, k, v, batch.metadata(dev), batch.head_dim ** -0.5,
                                       batch.groups)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert jb.read_device_errors() == 0


def test_limit_is_validated():
    with pytest.raises(ValueError):
        _lib.selftest_bounded_wait(0)
