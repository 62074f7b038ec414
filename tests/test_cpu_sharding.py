"""KV-head sharding across ranks: world_size-2 gloo processes on the CPU.

Each rank runs the oracle on its KV-head shard of the golden ragged batch; the gathered
shards equal the unsharded result, and the ranks' timing reduction is a max.
"""
from __future__ import annotations

import socket

import pytest
import torch
import torch.multiprocessing as mp

from jetspec_b200.sharding import shard_for_rank


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_partition_heads():
    for world in (1, 2, 4, 8):
        shards = [shard_for_rank(8, 4, world, r) for r in range(world)]
        kv = [h for s in shards for h in range(s.kv_head_begin, s.kv_head_end)]
        qh = [h for s in shards for h in range(s.q_head_begin, s.q_head_end)]
        assert kv == list(range(8)) and qh == list(range(32))
    with pytest.raises(ValueError):
        shard_for_rank(8, 4, 3, 0)
    with pytest.raises(ValueError):
        shard_for_rank(8, 4, 2, 2)


def test_gloo_two_rank_shards_reassemble_the_full_result(tmp_path):
    from golden_cases import load_attn_case
    from oracle import tree_attention as attn_oracle

    result = str(tmp_path / "gathered.pt")
    ctx = mp.get_context("spawn")
    port = _free_port()
    import _gloo_worker
    procs = [ctx.Process(target=_gloo_worker.run, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    data = torch.load(result)
    case = load_attn_case("ragged3")
    full = attn_oracle.masked_sdpa(case.q, case.k_pool, case.v_pool, case.prefixes, case.tables,
                                   case.tree_slots, case.parents, case.scale, case.groups)
    assert data["max"] == 2.0
    torch.testing.assert_close(data["gathered"], full, rtol=0, atol=1e-6)
