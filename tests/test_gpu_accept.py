"""Device acceptance walk: exact against the reference's accept_batch golden and the oracle."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import jetspec_b200 as jb
from golden_cases import load_npz
from oracle import accept as accept_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _device_case(z, dtype):
    logits = torch.from_numpy(z["logits"]).to(DEV, dtype)
    return (logits, torch.from_numpy(z["token_ids"]).to(DEV),
            torch.from_numpy(z["parents"]).to(DEV), torch.from_numpy(z["offsets"]).to(DEV),
            torch.from_numpy(z["depths"]).to(DEV))


def _check(results, path, accepted, correction, outputs):
    path, accepted = path.cpu().numpy(), accepted.cpu().numpy()
    correction, outputs = correction.cpu().numpy(), outputs.cpu().numpy()
    for r, res in enumerate(results):
        length = len(res["path"])
        assert path[r, :length].tolist() == res["path"]
        assert (path[r, length:] == -1).all()
        assert int(accepted[r]) == res["accepted_length"]
        assert int(correction[r]) == res["correction"]
        assert outputs[r, :length].tolist() == res["outputs"]


def test_matches_reference_golden_fp32():
    z = load_npz("accept.npz")
    logits, tokens, parents, offsets, depths = _device_case(z, torch.float32)
    out = jb.accept_walk(logits, tokens, parents, offsets, int(z["max_depth"]), depths=depths)
    torch.cuda.synchronize()
    results = [{"path": z["path"][r, :int(z["accepted_length"][r]) + 1].tolist(),
                "accepted_length": int(z["accepted_length"][r]),
                "correction": int(z["correction"][r]),
                "outputs": z["outputs"][r, :int(z["accepted_length"][r]) + 1].tolist()}
               for r in range(len(z["offsets"]) - 1)]
    _check(results, *out)
    assert jb.read_device_errors() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_matches_oracle_on_operand_dtypes(dtype):
    z = load_npz("accept.npz")
    logits, tokens, parents, offsets, depths = _device_case(z, dtype)
    expected = accept_oracle.accept_batch(logits.float().cpu().numpy(), z["token_ids"],
                                          z["parents"], z["depths"], z["offsets"],
                                          int(z["max_depth"]))
    out = jb.accept_walk(logits, tokens, parents, offsets, int(z["max_depth"]), depths=depths)
    _check(expected, *out)


def test_reference_signature_wrapper():
    z = load_npz("accept.npz")
    logits = torch.from_numpy(z["logits"]).to(DEV)
    offsets = z["offsets"].tolist()
    trees = []
    for r in range(len(offsets) - 1):
        lo, hi = offsets[r], offsets[r + 1]
        trees.append(SimpleNamespace(
            token_ids=torch.from_numpy(z["token_ids"][lo:hi]).to(DEV),
            parent_indices=torch.from_numpy(z["parents"][lo:hi]).to(DEV),
            depth=torch.from_numpy(z["depths"][lo:hi]).to(DEV), num_nodes=hi - lo))
    results = jb.accept_batch(logits, trees, offsets, int(z["max_depth"]))
    assert results[0]["path"] == [0, 2, 4]
    for r, res in enumerate(results):
        assert res["accepted_length"] == int(z["accepted_length"][r])
        assert res["correction"] == int(z["correction"][r])
    bad = trees[0].depth.clone()
    bad[2] = 5
    trees[0] = SimpleNamespace(token_ids=trees[0].token_ids, parent_indices=trees[0].parent_indices,
                               depth=bad, num_nodes=trees[0].num_nodes)
    with pytest.raises(RuntimeError, match="canonical tail"):
        jb.accept_batch(logits, trees, offsets, int(z["max_depth"]))


@pytest.mark.parametrize("vocab,offset", [(151936, 0), (151937, 1), (1000, 3)])
def test_large_vocabulary_planted_paths(vocab, offset):
    """Qwen3-sized vocabulary, odd sizes and rows that do not start on 16 bytes."""
    rng = np.random.default_rng(vocab + offset)
    sizes = [1, 7, 33, 64]
    tokens, parents, offsets = [], [], [0]
    for n in sizes:
        par = [-1] + [int(rng.integers(max(0, i - 3), i)) for i in range(1, n)]
        tokens += [int(t) for t in rng.integers(0, 50, size=n)]
        parents += par
        offsets.append(offsets[-1] + n)
    q = offsets[-1]
    gen = torch.Generator(device=DEV).manual_seed(5)
    backing = torch.randn(q, vocab + offset, generator=gen, device=DEV).bfloat16()
    logits = backing[:, offset:]
    tok = np.array(tokens)
    for r, n in enumerate(sizes):  # plant root -> first child -> ... chains
        lo = offsets[r]
        node = 0
        for _ in range(6):
            kids = [j for j in range(n) if parents[lo + j] == node]
            if not kids:
                break
            child = kids[-1]
            logits[lo + node, int(tok[lo + child])] = 40.0
            node = child
    logits[0, vocab - 1] = float("nan")  # NaN ranks highest (torch.argmax)
    depth = []
    for r, n in enumerate(sizes):
        d = [0] * n
        for i in range(1, n):
            d[i] = d[parents[offsets[r] + i]] + 1
        depth += d
    expected = accept_oracle.accept_batch(logits.float().cpu().numpy(), tokens, parents, depth,
                                          offsets, 8)
    assert expected[0]["correction"] == vocab - 1
    out = jb.accept_walk(logits, torch.tensor(tokens, device=DEV), torch.tensor(parents, device=DEV),
                         torch.tensor(offsets, device=DEV, dtype=torch.int32), 8)
    _check(expected, *out)


def test_depth_zero_returns_root_and_its_greedy_token():
    z = load_npz("accept.npz")
    logits, tokens, parents, offsets, _ = _device_case(z, torch.float32)
    path, accepted, correction, outputs = jb.accept_walk(logits, tokens, parents, offsets, 0)
    greedy = logits.argmax(-1).cpu()
    assert (path[:, 0] == 0).all() and (accepted == 0).all()
    assert correction.cpu().tolist() == greedy[torch.from_numpy(z["offsets"][:-1]).long()].tolist()
    assert outputs[:, 0].cpu().tolist() == correction.cpu().tolist()


def test_offsets_outside_the_nodes_are_skipped_and_flagged():
    """A request whose offsets reach past the node arrays reads nothing beyond them."""
    z = load_npz("accept.npz")
    logits, tokens, parents, offsets, _ = _device_case(z, torch.float32)
    jb.read_device_errors()
    bad = torch.tensor([0, 5, logits.shape[0] + 10], dtype=torch.int32, device=DEV)
    path, accepted, correction, _ = jb.accept_walk(logits, tokens, parents, bad, 4)
    torch.cuda.synchronize()
    assert int(accepted[1]) == -1 and (path[1] == -1).all()
    assert int(accepted[0]) == int(z["accepted_length"][0])
    assert jb.read_device_errors() & 1
