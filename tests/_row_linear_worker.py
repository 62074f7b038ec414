"""Entry points of the spawned ranks of the row-parallel linear tests (imports nothing at load)."""
from __future__ import annotations


def _setup_paths():
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for path in (str(root), str(root / "tests")):
        if path not in sys.path:
            sys.path.insert(0, path)
    import __graft_entry__
    __graft_entry__.load_package()


def cpu_rank(rank: int, world: int, port: int, case: str, result_path: str):
    """gloo rank on the CPU: this package's RowParallelLinear shards and bias rule, with the
    reference's arithmetic (F.linear on the shard, all_reduce) on top, against the golden."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    _setup_paths()
    from jetspec_b200.row_linear import RowParallelLinear

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from golden_cases import GOLDEN

        z = np.load(GOLDEN / "row_linear.npz")
        bf16 = lambda key: torch.from_numpy(z[f"{case}_{key}"].astype(np.int16)).view(torch.bfloat16)
        x, weight, bias = bf16("x"), bf16("weight"), bf16("bias")
        has_bias = bool(z[f"{case}_has_bias"])
        layer = RowParallelLinear(x.shape[1], weight.shape[0], bias=has_bias).to(torch.bfloat16)
        assert layer.tp_size == world and layer.tp_rank == rank
        layer.weight_loader(layer.weight, weight)
        if has_bias:
            layer.weight_loader(layer.bias, bias)
        shard = x.shape[1] // world
        assert torch.equal(layer.weight.data, weight[:, rank * shard:(rank + 1) * shard])
        with torch.no_grad():
            y = F.linear(x.chunk(world, 1)[rank].contiguous(), layer.weight,
                         layer.bias if layer.tp_rank == 0 else None)
            dist.all_reduce(y)
        if rank == 0:
            np.save(result_path, y.view(torch.int16).numpy())
    finally:
        dist.destroy_process_group()


def gpu_rank(rank: int, world: int, port: int, result_path: str):
    """NCCL rank on its own GPU: the fused layer twice in a row (the second call reuses the
    exchange workspaces), against a float32 reference and the NCCL all-reduce path."""
    import datetime
    import json

    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    _setup_paths()
    from jetspec_b200 import read_device_errors
    from jetspec_b200.row_linear import RowParallelLinear, group_state_for

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    report = {"rank": rank, "ok": True, "errors": []}
    try:
        m, fin, fout = 1000, 4096, 4096
        layer = RowParallelLinear(fin, fout, bias=True).to(dev, torch.bfloat16)
        for call in range(2):
            gen = torch.Generator(device=dev).manual_seed(100 + call)
            x = torch.randn(m, fin, generator=gen, device=dev).bfloat16()
            weight = (torch.randn(fout, fin, generator=gen, device=dev) / fin ** 0.5).bfloat16()
            bias = torch.randn(fout, generator=gen, device=dev).bfloat16()
            layer.weight_loader(layer.weight, weight)
            layer.weight_loader(layer.bias, bias)
            shard = fin // world
            xs = x[:, rank * shard:(rank + 1) * shard].contiguous()
            y = layer(xs)
            nccl = F.linear(xs, layer.weight, layer.bias if rank == 0 else None)
            dist.all_reduce(nccl)
            parts = [(x[:, r * shard:(r + 1) * shard].float() @
                      weight[:, r * shard:(r + 1) * shard].float().T +
                      (bias.float() if r == 0 else 0)).bfloat16().float() for r in range(world)]
            ref = torch.stack(parts).sum(0).bfloat16().float()
            absdot = sum(x[:, r * shard:(r + 1) * shard].float().abs() @
                         weight[:, r * shard:(r + 1) * shard].float().abs().T for r in range(world))
            tol = (2.0 ** -7 * (torch.stack(parts).abs().sum(0) + ref.abs()) +
                   shard * 2.0 ** -24 * absdot + 1e-6)
            err = (y.float() - ref).abs()
            report[f"call{call}_max_over_tol"] = float((err / tol).max())
            report[f"call{call}_vs_nccl_max_abs"] = float((y.float() - nccl.float()).abs().max())
            if not bool((err <= tol).all()):
                report["ok"] = False
        torch.cuda.synchronize()
        report["device_errors"] = int(read_device_errors())
        group_state_for(dev).close()
    except Exception as exc:  # reported to the test, which fails on it
        report["ok"] = False
        report["errors"].append(repr(exc))
    finally:
        dist.destroy_process_group()
    with open(f"{result_path}.{rank}", "w") as handle:
        json.dump(report, handle)
