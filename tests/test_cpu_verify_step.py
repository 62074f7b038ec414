"""Config 5 under tensor parallelism, host side: the reference's dense MLP seam at TP 2.

The reference's packed verifier calls ``Qwen3MLP.forward_dense`` (qwen3.py:348-355), which
splits the merged gate/up weight at the global intermediate size and therefore fails on a
rank of a TP > 1 model (the reference's packed runtime requires TP 1,
llm_engine.py:355-356).  ``verify_step`` runs TP > 1 with the split at the rank's width;
two gloo ranks on the CPU show that it reproduces the unsharded MLP.
"""
from __future__ import annotations

from pathlib import Path
import socket

import pytest
import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
pytestmark = pytest.mark.skipif(not (REF / "nanovllm").is_dir(),
                                reason="reference package not installed under baseline/_ref")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_rank_width_dense_mlp_at_tp2_equals_the_unsharded_mlp(tmp_path):
    result = str(tmp_path / "mlp.pt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    import _gloo_worker
    procs = [ctx.Process(target=_gloo_worker.run_dense_mlp, args=(r, 2, port, result))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    data = torch.load(result)
    gen = torch.Generator().manual_seed(11)
    gate = torch.randn((96, 64), generator=gen) * 0.1
    up = torch.randn((96, 64), generator=gen) * 0.1
    down = torch.randn((64, 96), generator=gen) * 0.1
    x = torch.randn((5, 64), generator=gen)
    full = F.linear(F.silu(F.linear(x, gate)) * F.linear(x, up), down)
    torch.testing.assert_close(data["out"], full, rtol=1e-5, atol=1e-5)
    # The reference's own method cannot run on a TP 2 rank.
    assert data["reference_error"] is not None
