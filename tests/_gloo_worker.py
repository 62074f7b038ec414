"""Entry point of the spawned gloo ranks of test_cpu_sharding (imports nothing at load)."""
from __future__ import annotations


def run(rank: int, world: int, port: int, result_path: str):
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for path in (str(root), str(root / "tests")):
        if path not in sys.path:
            sys.path.insert(0, path)
    import torch
    import torch.distributed as dist

    import __graft_entry__
    __graft_entry__.load_package()
    from golden_cases import load_attn_case
    from jetspec_b200.sharding import shard_for_rank
    from oracle import tree_attention as attn_oracle

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        case = load_attn_case("ragged3")
        shard = shard_for_rank(case.kv_heads, case.groups, world, rank)
        local = attn_oracle.masked_sdpa(shard.slice_queries(case.q), shard.slice_pool(case.k_pool),
                                        shard.slice_pool(case.v_pool), case.prefixes, case.tables,
                                        case.tree_slots, case.parents, case.scale, case.groups)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        elapsed = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        if rank == 0:
            torch.save({"gathered": torch.cat(parts, dim=1), "max": elapsed.item()}, result_path)
    finally:
        dist.destroy_process_group()


def run_dense_mlp(rank: int, world: int, port: int, result_path: str):
    """The reference's Qwen3MLP at tensor parallelism `world`, weights loaded through its
    own loaders from full seeded tensors; the rank-width forward_dense of verify_step and
    (recorded, not raised) the reference's own forward_dense."""
    import datetime
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for path in (str(root), str(root / "baseline" / "_ref")):
        if path not in sys.path:
            sys.path.insert(0, path)
    import torch
    import torch.distributed as dist

    import __graft_entry__
    __graft_entry__.load_package()

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from nanovllm.models.qwen3 import Qwen3MLP
        from jetspec_b200.verify_step import _dense_mlp_rank_width

        hidden, inter = 64, 96
        gen = torch.Generator().manual_seed(11)
        gate = torch.randn((inter, hidden), generator=gen) * 0.1
        up = torch.randn((inter, hidden), generator=gen) * 0.1
        down = torch.randn((hidden, inter), generator=gen) * 0.1
        x = torch.randn((5, hidden), generator=gen)
        mlp = Qwen3MLP(hidden, inter, "silu")
        with torch.no_grad():
            p = mlp.gate_up_proj.weight
            p.weight_loader(p, gate, 0)
            p.weight_loader(p, up, 1)
            p = mlp.down_proj.weight
            p.weight_loader(p, down)
            out = _dense_mlp_rank_width(mlp)(x)
            try:
                mlp.forward_dense(x)
                reference_error = None
            except RuntimeError as exc:
                reference_error = str(exc)
        if rank == 0:
            torch.save({"out": out, "reference_error": reference_error}, result_path)
    finally:
        dist.destroy_process_group()
