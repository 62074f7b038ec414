"""Packed ragged tree-verification metadata: the attention kernel's input contract.

Mirrors ``PackedTreeMetadata`` of the reference
(nanovllm/speculative/jetspec/packed_metadata.py:16-237): the same device fields with the
same dtypes and layouts, the same host tuples, and the same validation rules, so that
objects of either class can be passed to the kernels here.  Only tree nodes are packed:
each request keeps its own prefix page table, node slots and ancestor matrix.

Device fields (R requests, Q = sum of node counts):
  cu_seqlens_q i32[R+1], query_to_request i32[Q], query_local_row i32[Q],
  prefix_lens i32[R], block_tables i32[R, W] padded with -1 (W >= 1),
  tree_slots i64[Q], qq_bias f32[sum T_r^2] (0 visible / -inf hidden, row-major per
  request), qq_bias_offsets i64[R+1], node_counts i32[R].
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch


def ancestor_mask_from_parents(parents: Sequence[int]) -> np.ndarray:
    """Boolean [T, T] matrix: row j marks node j and every ancestor of j.

    ``parents[0]`` must be -1 (the root) and every other parent must precede its
    child, which is the topological order the kernels rely on.
    """
    count = len(parents)
    if count < 1 or int(parents[0]) != -1:
        raise ValueError("a tree needs a root at index 0 with parent -1")
    mask = np.zeros((count, count), dtype=bool)
    mask[0, 0] = True
    for node in range(1, count):
        parent = int(parents[node])
        if not 0 <= parent < node:
            raise ValueError("tree parents must precede their children")
        mask[node] = mask[parent]
        mask[node, node] = True
    return mask


def _bias_rows(mask: np.ndarray) -> np.ndarray:
    return np.where(mask, np.float32(0.0), np.float32(-np.inf)).astype(np.float32).reshape(-1)


@dataclass(frozen=True)
class StagedTopology:
    """Compact round topology for the device metadata build (PackedTreeMetadata
    .stage_topology): ``host`` is the int32 buffer to upload; the rest is what the host keeps
    (per-request node counts, prefix lengths, tables, the arena pages, request IDs)."""
    host: np.ndarray
    counts: tuple
    prefixes: tuple
    tables: tuple
    pages: tuple
    ids: tuple
    width: int
    block_size: int
    query_offsets: tuple   # cu_seqlens_q on the host
    bias_offsets: tuple    # qq_bias_offsets on the host
    slot_ids: tuple        # node j's scratch slot: the j-th slot of the arena pages


@dataclass(frozen=True)
class PackedTreeMetadata:
    cu_seqlens_q: torch.Tensor
    query_to_request: torch.Tensor
    query_local_row: torch.Tensor
    prefix_lens: torch.Tensor
    block_tables: torch.Tensor
    tree_slots: torch.Tensor
    qq_bias: torch.Tensor
    qq_bias_offsets: torch.Tensor
    node_counts: torch.Tensor
    block_size: int
    prefix_lengths: tuple[int, ...]
    query_offsets: tuple[int, ...]
    node_counts_host: tuple[int, ...]
    block_tables_host: tuple[tuple[int, ...], ...]
    tree_slot_ids: tuple[int, ...]
    request_ids: tuple

    # ---- construction -------------------------------------------------------------------
    @classmethod
    def build(cls, prefix_lens, block_tables, tree_slots, ancestor_masks, block_size, *,
              request_ids=None) -> "PackedTreeMetadata":
        """Validate host-side once and build the compact device buffers.

        Follows PackedTreeMetadata.build (packed_metadata.py:35-126): rejects
        non-tight page tables, malformed or non-causal ancestor masks, negative or
        overlapping scratch slots and scratch pages shared with a live prefix.
        Outputs live on the device of ``tree_slots[0]``.
        """
        prefixes = tuple(int(v) for v in prefix_lens)
        count = len(prefixes)
        if count < 1 or not (len(block_tables) == len(tree_slots) == len(ancestor_masks) == count):
            raise ValueError("packed metadata requires equally sized nonempty request lists")
        block_size = int(block_size)
        if block_size <= 0 or any(v < 0 for v in prefixes):
            raise ValueError("invalid packed prefix length or page geometry")
        ids = tuple(range(count)) if request_ids is None else tuple(request_ids)
        if len(ids) != count or len(set(ids)) != count:
            raise ValueError("request IDs must be unique and match the request count")
        device = tree_slots[0].device
        tables, slot_lists, masks = [], [], []
        for prefix, table, slots, ancestors in zip(prefixes, block_tables, tree_slots,
                                                   ancestor_masks):
            pages = tuple(int(v) for v in table)
            if (len(pages) != -(-prefix // block_size) or len(set(pages)) != len(pages)
                    or any(v < 0 for v in pages)):
                raise ValueError("prefix block table must be a tight canonical page table")
            if (slots.ndim != 1 or slots.dtype not in (torch.int32, torch.int64)
                    or slots.device != device):
                raise ValueError("tree slots must be integer vectors on one common device")
            nodes = int(slots.numel())
            if (nodes < 1 or tuple(ancestors.shape) != (nodes, nodes)
                    or ancestors.dtype != torch.bool or ancestors.device != device):
                raise ValueError("ancestor masks must be request-local boolean [nodes,nodes] matrices")
            mask = ancestors.detach().cpu().numpy()
            if not mask.diagonal().all() or np.triu(mask, 1).any():
                raise ValueError("ancestor mask must include self and be causal in local flat order")
            ids_here = [int(v) for v in slots.detach().cpu().tolist()]
            if any(v < 0 for v in ids_here):
                raise ValueError("scratch slot IDs cannot be negative")
            tables.append(pages)
            slot_lists.append(ids_here)
            masks.append(mask)
        return cls._assemble(prefixes, tables, slot_lists, masks, block_size, ids, device)

    @classmethod
    def from_host_trees(cls, prefix_lens, block_tables, trees, arena_blocks, block_size, *,
                        device, request_ids) -> "PackedTreeMetadata":
        """Serving builder from validated CPU topology and scratch-page ownership.

        Follows PackedTreeMetadata.from_host_trees (packed_metadata.py:128-198): each
        tree provides ``num_nodes``, ``host_ancestor`` (CPU bool [T, T]),
        ``host_parents`` and ``host_depths``; node j's scratch slot is the j-th slot of
        the packed arena pages ``arena_blocks``.
        """
        prefixes = tuple(int(v) for v in prefix_lens)
        tables = tuple(tuple(int(v) for v in table) for table in block_tables)
        ids = tuple(request_ids)
        count = len(prefixes)
        if not count or not (len(tables) == len(trees) == len(ids) == count):
            raise ValueError("packed metadata request lists must align")
        if block_size <= 0 or any(v < 0 for v in prefixes) or len(set(ids)) != count:
            raise ValueError("invalid packed prefix geometry or duplicate request ID")
        masks = []
        for prefix, table, tree in zip(prefixes, tables, trees):
            if (len(table) != -(-prefix // block_size) or len(set(table)) != len(table)
                    or any(v < 0 for v in table)):
                raise ValueError("prefix block table must be a tight canonical page table")
            nodes = int(tree.num_nodes)
            ancestor = tree.host_ancestor
            if (ancestor.device.type != "cpu" or ancestor.dtype != torch.bool
                    or tuple(ancestor.shape) != (nodes, nodes) or nodes < 1):
                raise ValueError("host ancestor must be a nonempty boolean square matrix")
            mask = ancestor.numpy()
            if not mask.diagonal().all() or np.triu(mask, 1).any():
                raise ValueError("ancestor mask must include self and be locally causal")
            parents, depths = tree.host_parents, tree.host_depths
            if len(parents) != nodes or len(depths) != nodes or parents[0] != -1 or depths[0] != 0:
                raise ValueError("invalid root topology")
            for node in range(1, nodes):
                parent = parents[node]
                if not 0 <= parent < node or depths[node] != depths[parent] + 1:
                    raise ValueError("tree parent/depth mismatch")
                expected = mask[parent].copy()
                expected[node] = True
                if not np.array_equal(expected, mask[node]):
                    raise ValueError("ancestor visibility differs from parent topology")
            masks.append(mask)
        pages = tuple(int(v) for v in arena_blocks)
        total = sum(m.shape[0] for m in masks)
        if len(pages) * block_size < total or len(set(pages)) != len(pages) or any(v < 0 for v in pages):
            raise ValueError("invalid or insufficient scratch page ownership")
        if set(pages).intersection(v for table in tables for v in table):
            raise ValueError("scratch pages overlap a live committed prefix")
        flat = [pages[j // block_size] * block_size + j % block_size for j in range(total)]
        slot_lists, cursor = [], 0
        for mask in masks:
            slot_lists.append(flat[cursor:cursor + mask.shape[0]])
            cursor += mask.shape[0]
        return cls._assemble(prefixes, tables, slot_lists, masks, int(block_size), ids,
                             torch.device(device), validate_slots=False)

    @classmethod
    def from_parents_device(cls, prefix_lens, block_tables, parents, arena_blocks, block_size,
                            *, device, request_ids=None) -> "PackedTreeMetadata":
        """from_host_trees' metadata, derived on the device from compact topology.

        Uploads node counts, prefix lengths, block tables, parents and the arena pages
        as one int32 buffer (about 4 bytes per node instead of 4 T^2 bytes of bias per
        request) and builds cu_seqlens_q, query_to_request, query_local_row, tree_slots,
        qq_bias and qq_bias_offsets with one launch of jt_metadata_build_launch; the
        prefix lengths, node counts and block tables are views of the uploaded buffer.
        Node j's scratch slot is the j-th slot of the packed arena pages, as in
        from_host_trees.  Host-side checks: tight canonical tables, parents in
        topological order, enough arena pages, no arena page inside a prefix.

        The two halves are public for callers that stage the upload themselves (pinned
        memory, a copy stream): ``stage_topology`` (host checks and the int32 buffer) and
        ``from_staged_topology`` (the device build from that buffer once it is on the GPU).
        """
        topo = cls.stage_topology(prefix_lens, block_tables, parents, arena_blocks, block_size,
                                  request_ids=request_ids)
        staged = torch.from_numpy(topo.host).to(torch.device(device))   # the one upload
        return cls.from_staged_topology(staged, topo)

    @staticmethod
    def stage_topology(prefix_lens, block_tables, parents, arena_blocks, block_size, *,
                       request_ids=None) -> "StagedTopology":
        """Host half of from_parents_device: the checks and the compact int32 buffer
        (``StagedTopology.host``: node counts, prefix lengths, padded block tables, parents,
        arena pages)."""
        prefixes = tuple(int(v) for v in prefix_lens)
        tables = tuple(tuple(int(v) for v in table) for table in block_tables)
        parent_arrays = [np.asarray(p, dtype=np.int64).reshape(-1) for p in parents]
        count = len(prefixes)
        ids = tuple(range(count)) if request_ids is None else tuple(request_ids)
        if not count or not (len(tables) == len(parent_arrays) == len(ids) == count):
            raise ValueError("packed metadata request lists must align")
        if block_size <= 0 or any(v < 0 for v in prefixes) or len(set(ids)) != count:
            raise ValueError("invalid packed prefix geometry or duplicate request ID")
        for prefix, table in zip(prefixes, tables):
            if (len(table) != (prefix + block_size - 1) // block_size or
                    len(set(table)) != len(table) or any(v < 0 for v in table)):
                raise ValueError("prefix block table must be a tight canonical page table")
        counts = [int(p.size) for p in parent_arrays]
        if min(counts) < 1:
            raise ValueError("tree parents must start at a root (-1) and precede their children")
        if max(counts) > 1024:
            raise ValueError("trees are limited to 1024 nodes")
        total = sum(counts)
        # Vectorised topology check: local index j of every node, its parent p; the root
        # (j = 0) needs p = -1, every other node 0 <= p < j.
        flat_parents = np.concatenate(parent_arrays)
        local = np.arange(total, dtype=np.int64) - np.repeat(
            np.cumsum([0] + counts[:-1], dtype=np.int64), counts)
        root = local == 0
        if (np.any(flat_parents[root] != -1) or
                np.any((flat_parents[~root] < 0) | (flat_parents[~root] >= local[~root]))):
            raise ValueError("tree parents must start at a root (-1) and precede their children")
        pages = tuple(int(v) for v in arena_blocks)
        if (len(pages) * block_size < total or len(set(pages)) != len(pages) or
                any(v < 0 for v in pages)):
            raise ValueError("invalid or insufficient scratch page ownership")
        if set(pages).intersection(v for table in tables for v in table):
            raise ValueError("scratch pages overlap a live committed prefix")
        width = max(1, max(len(t) for t in tables))
        padded = np.full((count, width), -1, dtype=np.int64)
        for row, table in enumerate(tables):
            padded[row, :len(table)] = table
        host = np.concatenate((np.asarray(counts, dtype=np.int64), np.asarray(prefixes, dtype=np.int64),
                               padded.reshape(-1), flat_parents, np.asarray(pages, dtype=np.int64)))
        offsets = np.concatenate(([0], np.cumsum(counts))).astype(np.int64)
        bias_offsets = np.concatenate(([0], np.cumsum(np.asarray(counts, dtype=np.int64) ** 2)))
        node = np.arange(total, dtype=np.int64)
        slots = np.asarray(pages, dtype=np.int64)[node // block_size] * block_size + node % block_size
        return StagedTopology(host=host.astype(np.int32), counts=tuple(counts),
                              prefixes=prefixes, tables=tables, pages=pages, ids=ids,
                              width=width, block_size=int(block_size),
                              query_offsets=tuple(offsets.tolist()),
                              bias_offsets=tuple(bias_offsets.tolist()),
                              slot_ids=tuple(slots.tolist()))

    @classmethod
    def from_staged_topology(cls, staged: torch.Tensor, topo: "StagedTopology"
                             ) -> "PackedTreeMetadata":
        """Device half of from_parents_device: ``staged`` is ``topo.host`` on the GPU (int32,
        contiguous); one jt_metadata_build_launch on the current stream builds the rest."""
        from . import _launch, _lib

        if (staged.dtype != torch.int32 or staged.ndim != 1 or not staged.is_cuda
                or staged.numel() != topo.host.size or not staged.is_contiguous()):
            raise ValueError("staged topology must be the int32 buffer of stage_topology on a GPU")
        device = staged.device
        counts, pages, block_size = topo.counts, topo.pages, topo.block_size
        count, width, total = len(counts), topo.width, sum(counts)
        cursor = 0

        def take(n):
            nonlocal cursor
            view = staged[cursor:cursor + n]
            cursor += n
            return view

        node_counts, prefix_lens_d = take(count), take(count)
        block_tables_d, parents_d, pages_d = take(count * width), take(total), take(len(pages))
        bias_offsets = topo.bias_offsets
        out = dict(
            cu_seqlens_q=torch.empty(count + 1, dtype=torch.int32, device=device),
            query_to_request=torch.empty(total, dtype=torch.int32, device=device),
            query_local_row=torch.empty(total, dtype=torch.int32, device=device),
            tree_slots=torch.empty(total, dtype=torch.int64, device=device),
            qq_bias=torch.empty(bias_offsets[-1], dtype=torch.float32, device=device),
            qq_bias_offsets=torch.empty(count + 1, dtype=torch.int64, device=device))
        p = _lib.JtMetadataBuildParams()
        p.node_counts, p.parents, p.arena_pages = (node_counts.data_ptr(), parents_d.data_ptr(),
                                                   pages_d.data_ptr())
        for name, tensor in out.items():
            setattr(p, name, tensor.data_ptr())
        p.num_requests, p.block_size, p.max_nodes = count, int(block_size), max(counts)
        p.num_nodes, p.num_pages = total, len(pages)
        lib = _lib.load_library()
        _lib.check(lib.jt_metadata_build_launch(ctypes.byref(p), _launch.stream_handle(device)))
        return cls(
            cu_seqlens_q=out["cu_seqlens_q"], query_to_request=out["query_to_request"],
            query_local_row=out["query_local_row"], prefix_lens=prefix_lens_d,
            block_tables=block_tables_d.view(count, width), tree_slots=out["tree_slots"],
            qq_bias=out["qq_bias"], qq_bias_offsets=out["qq_bias_offsets"],
            node_counts=node_counts, block_size=int(block_size), prefix_lengths=topo.prefixes,
            query_offsets=topo.query_offsets, node_counts_host=tuple(counts),
            block_tables_host=topo.tables, tree_slot_ids=topo.slot_ids, request_ids=topo.ids)

    @classmethod
    def from_parents(cls, prefix_lens, block_tables, parents, tree_slots, block_size, *,
                     device, request_ids=None) -> "PackedTreeMetadata":
        """Convenience builder from per-request parent lists and integer slot lists."""
        prefixes = tuple(int(v) for v in prefix_lens)
        if not (len(prefixes) == len(block_tables) == len(parents) == len(tree_slots)) or not prefixes:
            raise ValueError("packed metadata requires equally sized nonempty request lists")
        ids = tuple(range(len(prefixes))) if request_ids is None else tuple(request_ids)
        tables = []
        for prefix, table in zip(prefixes, block_tables):
            pages = tuple(int(v) for v in table)
            if (len(pages) != -(-prefix // int(block_size)) or len(set(pages)) != len(pages)
                    or any(v < 0 for v in pages)):
                raise ValueError("prefix block table must be a tight canonical page table")
            tables.append(pages)
        masks = [ancestor_mask_from_parents(p) for p in parents]
        slot_lists = [[int(v) for v in slots] for slots in tree_slots]
        for mask, slots in zip(masks, slot_lists):
            if len(slots) != mask.shape[0]:
                raise ValueError("one scratch slot per tree node is required")
            if any(v < 0 for v in slots):
                raise ValueError("scratch slot IDs cannot be negative")
        return cls._assemble(prefixes, tables, slot_lists, masks, int(block_size), ids,
                             torch.device(device))

    @classmethod
    def _assemble(cls, prefixes, tables, slot_lists, masks, block_size, ids, device, *,
                  validate_slots=True):
        counts = [m.shape[0] for m in masks]
        all_slots = [v for slots in slot_lists for v in slots]
        if validate_slots:
            if len(set(all_slots)) != len(all_slots):
                raise ValueError("packed requests have overlapping scratch slot ranges")
            live = {v for table in tables for v in table}
            if any(v // block_size in live for v in all_slots):
                raise ValueError("scratch pages overlap a live committed prefix")
        offsets = np.concatenate(([0], np.cumsum(counts))).astype(np.int64)
        bias_sizes = np.asarray([c * c for c in counts], dtype=np.int64)
        bias_offsets = np.concatenate(([0], np.cumsum(bias_sizes))).astype(np.int64)
        width = max(1, max(len(t) for t in tables))
        padded = np.full((len(tables), width), -1, dtype=np.int32)
        for row, table in enumerate(tables):
            padded[row, :len(table)] = table
        q_req = np.repeat(np.arange(len(counts), dtype=np.int32), counts)
        q_row = np.concatenate([np.arange(c, dtype=np.int32) for c in counts])
        bias = np.concatenate([_bias_rows(m) for m in masks])

        def dev(array, dtype):
            return torch.from_numpy(np.ascontiguousarray(array)).to(dtype=dtype).to(device)

        return cls(
            cu_seqlens_q=dev(offsets, torch.int32),
            query_to_request=dev(q_req, torch.int32),
            query_local_row=dev(q_row, torch.int32),
            prefix_lens=dev(np.asarray(prefixes, dtype=np.int64), torch.int32),
            block_tables=dev(padded, torch.int32),
            tree_slots=dev(np.asarray(all_slots, dtype=np.int64), torch.int64),
            qq_bias=dev(bias, torch.float32),
            qq_bias_offsets=dev(bias_offsets, torch.int64),
            node_counts=dev(np.asarray(counts, dtype=np.int64), torch.int32),
            block_size=block_size,
            prefix_lengths=tuple(prefixes),
            query_offsets=tuple(int(v) for v in offsets),
            node_counts_host=tuple(counts),
            block_tables_host=tuple(tuple(t) for t in tables),
            tree_slot_ids=tuple(all_slots),
            request_ids=tuple(ids),
        )

    # ---- queries ------------------------------------------------------------------------
    @property
    def num_requests(self) -> int:
        return len(self.prefix_lengths)

    @property
    def total_queries(self) -> int:
        return self.query_offsets[-1]

    @property
    def mask_elements(self) -> int:
        return int(self.qq_bias.numel())

    def request_slice(self, index: int) -> slice:
        if index < 0 or index >= self.num_requests:
            raise IndexError("packed request index is out of range")
        return slice(self.query_offsets[index], self.query_offsets[index + 1])

    def validate_pool_geometry(self, kv_pool: torch.Tensor) -> None:
        """Host-only bounds check of tables and slots against a 6-D KV pool."""
        if kv_pool.ndim != 6 or kv_pool.shape[0] != 2 or kv_pool.shape[3] != self.block_size:
            raise ValueError("packed metadata and KV pool page geometry differ")
        if kv_pool.device != self.tree_slots.device:
            raise ValueError("packed metadata and KV pool must be on the same device")
        pages = int(kv_pool.shape[2])
        if any(page >= pages for table in self.block_tables_host for page in table):
            raise ValueError("prefix page lies outside the KV pool")
        if any(slot >= pages * self.block_size for slot in self.tree_slot_ids):
            raise ValueError("tree slot lies outside the KV pool")

    def report(self) -> dict:
        tensors = (self.cu_seqlens_q, self.query_to_request, self.query_local_row,
                   self.prefix_lens, self.block_tables, self.tree_slots, self.qq_bias,
                   self.qq_bias_offsets, self.node_counts)
        return {"requests": self.num_requests, "total_queries": self.total_queries,
                "cu_seqlens_q": list(self.query_offsets),
                "prefix_lengths": list(self.prefix_lengths),
                "node_counts": list(self.node_counts_host), "mask_elements": self.mask_elements,
                "total_query_square_not_allocated": self.total_queries ** 2,
                "device_metadata_bytes": sum(t.numel() * t.element_size() for t in tensors),
                "block_size": self.block_size,
                "numerical_contract": "fp32_online_softmax_tile64"}
