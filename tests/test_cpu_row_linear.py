"""Row-parallel linear on the CPU: the oracle pinned to the reference's golden, the layer's
host logic (shards, bias on rank 0) under gloo ranks, and the workspace size rule."""
from __future__ import annotations

import numpy as np
import pytest
import torch.multiprocessing as mp

import _row_linear_worker
from golden_cases import GOLDEN
from oracle import row_linear as orl


def _case(name):
    z = np.load(GOLDEN / "row_linear.npz")
    g = lambda key: z[f"{name}_{key}"]
    bias = orl.bf16_to_f32(g("bias")) if int(g("has_bias")) else None
    return (orl.bf16_to_f32(g("x")), orl.bf16_to_f32(g("weight")), bias, int(g("world")),
            g("y"))


@pytest.mark.parametrize("name", ["w1", "w2", "w4"])
def test_oracle_matches_reference_golden(name):
    x, weight, bias, world, y_bits = _case(name)
    y = orl.bf16_to_f32(y_bits)
    ours = orl.row_parallel_linear(x, weight, bias, world)
    assert (np.abs(ours - y) <= orl.tolerance(x, weight, bias, world)).all()
    if world <= 2:  # one rounding of the sum either way: bit-exact
        assert np.array_equal(ours, y)


def test_bf16_rounding_is_nearest_even():
    values = np.array([1 + 2 ** -8, 1 + 3 * 2 ** -8, -(1 + 2 ** -8), 1 + 2 ** -9, 3.0],
                      dtype=np.float32)
    assert orl.round_bf16(values).tolist() == [1.0, 1 + 2 ** -6, -1.0, 1.0, 3.0]


@pytest.mark.parametrize("name,world,port", [("w2", 2, 29731), ("w4", 4, 29741)])
def test_layer_shards_and_bias_rule_under_gloo(tmp_path, name, world, port):
    """The layer's weight_loader and rank-0 bias rule give the reference's output bits."""
    out = tmp_path / "y.npy"
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_row_linear_worker.cpu_rank, args=(r, world, port, name, str(out)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    z = np.load(GOLDEN / "row_linear.npz")
    assert np.array_equal(np.load(out).view(np.uint16), z[f"{name}_y"])


def test_workspace_rule():
    from jetspec_b200 import _lib

    lib = _lib.load_library()
    assert lib.jt_row_linear_workspace_size(2048, 4096, 1) == 0
    assert lib.jt_row_linear_workspace_size(0, 4096, 2) == -1
    assert lib.jt_row_linear_workspace_size(10, 64, 9) == -1
    tiles = 16 * 16  # a group of GPUs uses 128 x 256 output tiles
    for world in (2, 4, 8):
        owned = -(-tiles // world)
        flags = 256 + -(-tiles * (world + 1) * 4 // 256) * 256  # control block + flags
        if world == 2:  # a pair: receive slots for every tile, both epoch parities
            expect = flags + tiles * 2 * world * 65536
        else:  # owners: receive slots for the owned tiles, then the inbox
            expect = flags + owned * world * 65536 + tiles * 65536
        assert lib.jt_row_linear_workspace_size(2048, 4096, world) == expect


def test_c_abi_rejects_bad_arguments_before_any_cuda_call():
    """jt_row_linear_launch validates its parameters on the host and answers
    JT_ERR_INVALID with a message; these checks need no GPU."""
    import ctypes

    from jetspec_b200 import _lib

    lib = _lib.load_library()

    def launch(**fields):
        p = _lib.JtRowLinearParams()
        p.x, p.weight, p.out = 4096, 8192, 12288  # never dereferenced: rejected first
        p.m, p.n, p.k, p.x_stride, p.w_stride = 64, 256, 128, 128, 128
        p.dtype, p.rank, p.world, p.epoch = _lib.JT_BF16, 0, 1, 0
        for key, value in fields.items():
            setattr(p, key, value)
        status = lib.jt_row_linear_launch(ctypes.byref(p), None)
        return status, lib.jt_last_error().decode()

    assert lib.jt_row_linear_launch(None, None) == -1
    cases = [({"dtype": _lib.JT_F32}, "bf16 or f16"), ({"n": 40}, "multiple of 32"),
             ({"k": 12}, "multiple of 8"), ({"world": 9}, "world"), ({"rank": 2, "world": 2},
             "rank"), ({"out": None}, "null"), ({"x": 4100}, "alignment"),
             ({"x_stride": 100}, "strides"), ({"world": 2}, "workspaces")]
    for fields, text in cases:
        status, message = launch(**fields)
        assert status == -1 and text in message, (fields, message)
