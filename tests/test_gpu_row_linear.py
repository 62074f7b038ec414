"""Fused row-parallel linear + all-reduce on the GPU.

Checked against the reference's golden (RowParallelLinear under gloo ranks), against a
float32 torch reference at the model's shapes (o_proj: 4096 -> 4096, rows = 32 requests x
64 tree nodes) with the per-element bound of oracle/row_linear.tolerance, on one rank and
with 2 / 4 / 8 ranks played by one launch on this GPU, plus the bounded wait for a peer
that never arrives.  A real multi-GPU run goes through NCCL ranks when the box has the GPUs.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import _row_linear_worker
import jetspec_b200 as jb
from golden_cases import GOLDEN
from jetspec_b200 import _lib
from jetspec_b200.row_linear import row_parallel_linear, row_parallel_linear_emulated
from oracle import row_linear as orl

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
torch.backends.cuda.matmul.allow_tf32 = False  # the float32 reference stays float32


def _golden(name):
    z = np.load(GOLDEN / "row_linear.npz")
    bf16 = lambda key: torch.from_numpy(z[f"{name}_{key}"].astype(np.int16)).view(torch.bfloat16)
    bias = bf16("bias").to(DEV) if int(z[f"{name}_has_bias"]) else None
    return bf16("x").to(DEV), bf16("weight").to(DEV), bias, int(z[f"{name}_world"]), bf16("y")


def _shards(x, weight, world):
    k = x.shape[1] // world
    return ([x[:, r * k:(r + 1) * k].contiguous() for r in range(world)],
            [weight[:, r * k:(r + 1) * k].contiguous() for r in range(world)])


def _torch_reference(xs, ws, bias, dtype):
    """float32 partials rounded to the dtype and summed, with the per-element bound of
    oracle/row_linear.tolerance (one ulp of each partial and of the sum, plus the float32
    accumulation bound K 2^-24 sum |x_i w_i| of each partial)."""
    parts = [(x.float() @ w.float().T + (bias.float() if (r == 0 and bias is not None) else 0))
             .to(dtype).float() for r, (x, w) in enumerate(zip(xs, ws))]
    stacked = torch.stack(parts)
    total = stacked.sum(0).to(dtype).float()
    eps = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    absdot = sum(x.float().abs() @ w.float().abs().T for x, w in zip(xs, ws))
    k = xs[0].shape[1]
    return total, eps * (stacked.abs().sum(0) + total.abs()) + k * 2.0 ** -24 * absdot + 1e-6


def _assert_close(out, ref, tol):
    err = (out.float() - ref).abs()
    assert (err <= tol).all(), f"{int((err > tol).sum())} elements outside the bound"
    # In aggregate the two roundings differ by well under one ulp.
    assert err.mean() <= 2.0 ** -9 * ref.abs().mean()


def _run(xs, ws, bias, workspaces=None):
    if len(xs) == 1:
        return [row_parallel_linear(xs[0], ws[0], bias)]
    return row_parallel_linear_emulated(xs, ws, bias, workspaces=workspaces)


@pytest.mark.parametrize("name", ["w1", "w2", "w4"])
def test_matches_reference_golden(name):
    x, weight, bias, world, y = _golden(name)
    xs, ws = _shards(x, weight, world)
    outs = _run(xs, ws, bias)
    torch.cuda.synchronize()
    xn, wn = x.float().cpu().numpy(), weight.float().cpu().numpy()
    bn = bias.float().cpu().numpy() if bias is not None else None
    tol = torch.from_numpy(orl.tolerance(xn, wn, bn, world))
    for out in outs:
        assert ((out.float().cpu() - y.float()).abs() <= tol).all()
        assert torch.equal(out, outs[0])  # every rank holds the same bits
    assert jb.read_device_errors() == 0


@pytest.mark.parametrize("world,m,n,k,dtype", [
    (1, 300, 544, 512, torch.bfloat16),
    (1, 2048, 4096, 4096, torch.bfloat16),
    (2, 2048, 4096, 4096, torch.bfloat16),
    (4, 1000, 4096, 2048, torch.float16),
    (8, 2048, 4096, 4096, torch.bfloat16),
    (8, 77, 12288 // 3, 12288, torch.bfloat16),
])
def test_matches_float32_reference(world, m, n, k, dtype):
    gen = torch.Generator(device=DEV).manual_seed(world * 131 + m)
    x = torch.randn(m, k, generator=gen, device=DEV).to(dtype)
    weight = (torch.randn(n, k, generator=gen, device=DEV) / k ** 0.5).to(dtype)
    bias = torch.randn(n, generator=gen, device=DEV).to(dtype)
    xs, ws = _shards(x, weight, world)
    outs = _run(xs, ws, bias)
    ref, tol = _torch_reference(xs, ws, bias, dtype)
    for out in outs:
        _assert_close(out, ref, tol)
    assert jb.read_device_errors() == 0


def test_two_calls_reuse_the_exchange_workspaces():
    world, m, n, k = 2, 600, 1024, 1024
    nbytes = int(_lib.load_library().jt_row_linear_workspace_size(m, n, world))
    buffers = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
    for epoch in (1, 2, 3):
        gen = torch.Generator(device=DEV).manual_seed(epoch)
        x = torch.randn(m, k, generator=gen, device=DEV).bfloat16()
        weight = (torch.randn(n, k, generator=gen, device=DEV) / k ** 0.5).bfloat16()
        xs, ws = _shards(x, weight, world)
        outs = row_parallel_linear_emulated(xs, ws, None, workspaces=(buffers, epoch))
        ref, tol = _torch_reference(xs, ws, None, torch.bfloat16)
        for out in outs:
            _assert_close(out, ref, tol)
    assert jb.read_device_errors() == 0


def test_device_epoch_counter_and_graph_replay():
    """epoch 0: every call takes its epoch from the workspaces' own counters, so repeated
    calls and replays of one captured launch (inputs changed in place) stay correct."""
    world, m, n, k = 4, 384, 768, 1024
    nbytes = int(_lib.load_library().jt_row_linear_workspace_size(m, n, world))
    buffers = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(world)]
    gen = torch.Generator(device=DEV).manual_seed(21)
    x = torch.randn(m, k, generator=gen, device=DEV).bfloat16()
    weight = (torch.randn(n, k, generator=gen, device=DEV) / k ** 0.5).bfloat16()
    xs, ws = _shards(x, weight, world)
    for _ in range(3):
        outs = row_parallel_linear_emulated(xs, ws, None, workspaces=(buffers, 0))
        ref, tol = _torch_reference(xs, ws, None, torch.bfloat16)
        for out in outs:
            _assert_close(out, ref, tol)
    graph = torch.cuda.CUDAGraph()
    stream = torch.cuda.Stream(DEV)
    stream.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph):
            outs = row_parallel_linear_emulated(xs, ws, None, workspaces=(buffers, 0))
    torch.cuda.current_stream(DEV).wait_stream(stream)
    for seed in (22, 23):
        gen = torch.Generator(device=DEV).manual_seed(seed)
        for xr in xs:
            xr.copy_(torch.randn(xr.shape, generator=gen, device=DEV).bfloat16())
        graph.replay()
        ref, tol = _torch_reference(xs, ws, None, torch.bfloat16)
        for out in outs:
            _assert_close(out, ref, tol)
    torch.cuda.synchronize()
    assert jb.read_device_errors() == 0


def test_strided_input_rows_and_leading_dims():
    m, n, k = 130, 256, 320
    gen = torch.Generator(device=DEV).manual_seed(9)
    wide = torch.randn(2, m // 2, k + 64, generator=gen, device=DEV).bfloat16()
    x = wide[..., 16:16 + k]  # row stride k + 64, 16-byte aligned start
    weight = (torch.randn(n, k, generator=gen, device=DEV) / k ** 0.5).bfloat16()
    out = row_parallel_linear(x, weight)
    assert out.shape == (2, m // 2, n)
    ref, tol = _torch_reference([x.reshape(m, k)], [weight], None, torch.bfloat16)
    _assert_close(out.reshape(m, n), ref, tol)


def test_shapes_the_kernel_does_not_take_are_rejected():
    x = torch.randn(8, 64, device=DEV).bfloat16()
    with pytest.raises(ValueError, match="multiple of 32"):
        row_parallel_linear(x, torch.randn(40, 64, device=DEV).bfloat16())
    with pytest.raises(ValueError):
        row_parallel_linear(x, torch.randn(64, 64, device=DEV).half())


def test_peer_that_never_arrives_times_out_and_the_context_stays_usable():
    """Rank 0 of a two-rank group launched alone: its wait for rank 1's partials gives up
    after the limit, sets the timeout bit, and the next launch is correct."""
    m, n, k = 256, 512, 256
    lib = _lib.load_library()
    nbytes = int(lib.jt_row_linear_workspace_size(m, n, 2))
    buffers = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(2)]
    x = torch.randn(m, k, device=DEV).bfloat16()
    weight = torch.randn(n, k, device=DEV).bfloat16()
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    import ctypes
    array = (ctypes.c_void_p * 2)(*[b.data_ptr() for b in buffers])
    p = _lib.JtRowLinearParams()
    p.x, p.weight, p.bias, p.out = x.data_ptr(), weight.data_ptr(), None, out.data_ptr()
    p.m, p.n, p.k, p.x_stride, p.w_stride = m, n, k, k, k
    p.dtype, p.rank, p.world, p.workspaces, p.epoch = _lib.JT_BF16, 0, 2, array, 1
    p.wait_limit_cycles = 2_000_000  # ~1 ms
    jb.read_device_errors()
    _lib.check(lib.jt_row_linear_launch(ctypes.byref(p),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert jb.read_device_errors() & 4
    y = row_parallel_linear(x, weight)
    ref, tol = _torch_reference([x], [weight], None, torch.bfloat16)
    _assert_close(y, ref, tol)
    assert jb.read_device_errors() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_ranks_on_separate_gpus(tmp_path):
    world = min(torch.cuda.device_count(), 4)
    result = str(tmp_path / "rank")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_row_linear_worker.gpu_rank, args=(r, world, 29811, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for r in range(world):
        with open(f"{result}.{r}") as handle:
            report = json.load(handle)
        assert report["ok"], report
        assert report["device_errors"] == 0, report
