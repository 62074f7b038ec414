"""Row-parallel linear with its all-reduce fused into one sm_100a kernel per GPU.

``RowParallelLinear`` keeps the reference's layer (nanovllm/layers/linear.py:131-156):
constructor ``(input_size, output_size, bias=False)``, a ``weight`` of
``[output_size, input_size / tp_size]`` loaded by ``weight_loader`` (which narrows the
checkpoint's input dimension to this rank's shard, :139-147) and ``forward(x)`` returning
the all-reduced ``F.linear`` output with the bias added once (rank 0's).  The reference
runs a cuBLAS GEMM and then ``dist.all_reduce``; here ``jt_row_linear_launch`` computes the
partial tiles with tcgen05 and exchanges them with the other ranks' GPUs through peer
memory while the GEMM still runs (every rank must call forward with the same shapes, as
with the reference's collective).

The exchange needs one workspace per rank, reachable from every rank's GPU:
``RowLinearGroup`` allocates it (``jt_device_alloc_zeroed``), all-gathers the CUDA IPC
handles over the process group and opens the peers' ones.  This is collective and
happens on the first forward and whenever a larger batch arrives.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
from torch import nn

from . import _launch, _lib

_DTYPES = {torch.bfloat16: _lib.JT_BF16, torch.float16: _lib.JT_F16}


class RowLinearGroup:
    """Exchange workspaces of one tensor-parallel group, seen from this rank."""

    def __init__(self, group=None, device: torch.device | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.capacity = (0, 0)
        self._own = None
        self._peers: list[int] = []
        self._array = None

    def _release(self):
        lib = _lib.load_library()
        for r, ptr in enumerate(self._peers):
            if r != self.rank and ptr:
                _lib.check(lib.jt_ipc_close_handle(ctypes.c_void_p(ptr)))
        if self._own:
            _lib.check(lib.jt_device_free(ctypes.c_void_p(self._own)))
        self._own, self._peers, self._array = None, [], None

    def ensure(self, m: int, n: int) -> None:
        """Collective: (re)build the workspaces when [m, n] outgrows them."""
        if self.world == 1 or (m <= self.capacity[0] and n == self.capacity[1]):
            return
        lib = _lib.load_library()
        rows = max(m, 2 * self.capacity[0] if n == self.capacity[1] else 0)
        nbytes = int(lib.jt_row_linear_workspace_size(rows, n, self.world))
        if nbytes <= 0:
            raise ValueError(f"row_linear: invalid output shape [{m}, {n}]")
        if self._own:
            # No rank may still read the old workspaces (a previous call's exchange).
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self._release()
        own = ctypes.c_void_p()
        _lib.check(lib.jt_device_alloc_zeroed(nbytes, ctypes.byref(own)))
        handle = (ctypes.c_char * 64)()
        _lib.check(lib.jt_ipc_get_handle(own, handle))
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        peers = []
        for r, h in enumerate(handles):
            if r == self.rank:
                peers.append(own.value)
                continue
            ptr = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(h, 64)
            _lib.check(lib.jt_ipc_open_handle(buf, ctypes.byref(ptr)))
            peers.append(ptr.value)
        self._own, self._peers = own.value, peers
        self._array = (ctypes.c_void_p * self.world)(*peers)
        self.capacity = (rows, n)
        # Every rank's zeroed workspace exists before any rank's first exchange.
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def workspaces(self):
        return self._array

    def next_epoch(self) -> int:
        """0: the kernel takes each call's epoch from the counter in this rank's workspace
        (advanced on the device, so captured launches replay correctly)."""
        return 0

    def close(self) -> None:
        if self._own:
            torch.cuda.synchronize(self.device)
            self._release()


_GROUPS: dict = {}


def group_state_for(device: torch.device, group=None) -> RowLinearGroup:
    """The exchange workspaces shared by every layer of this rank on ``device``: launches
    on one stream are ordered, and each call finishes reading them before the next starts."""
    key = (device.index, id(group))
    state = _GROUPS.get(key)
    if state is None:
        state = _GROUPS[key] = RowLinearGroup(group, device)
    return state


def _params(x, weight, bias, out, rank, world, workspaces, epoch):
    p = _lib.JtRowLinearParams()
    p.x, p.weight, p.out = x.data_ptr(), weight.data_ptr(), out.data_ptr()
    p.bias = bias.data_ptr() if bias is not None else None
    p.m, p.k = x.shape
    p.n = weight.shape[0]
    p.x_stride, p.w_stride = x.stride(0), weight.stride(0)
    p.dtype = _DTYPES[x.dtype]
    p.rank, p.world = rank, world
    p.workspaces = workspaces
    p.epoch = epoch
    p.wait_limit_cycles = 0
    return p


def _check_operands(x, weight, bias):
    if x.dtype not in _DTYPES or weight.dtype != x.dtype or (bias is not None and
                                                             bias.dtype != x.dtype):
        raise ValueError("row_parallel_linear: x, weight and bias must share bf16 or f16")
    if not (x.is_cuda and weight.is_cuda and x.device == weight.device):
        raise ValueError("row_parallel_linear: CUDA tensors on one device required")
    if weight.ndim != 2 or x.shape[-1] != weight.shape[1]:
        raise ValueError("row_parallel_linear: x [..., k] and weight [n, k] required")
    if bias is not None and bias.shape != (weight.shape[0],):
        raise ValueError("row_parallel_linear: bias must be [n]")


def row_parallel_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                        group_state: RowLinearGroup | None = None) -> torch.Tensor:
    """F.linear(x, weight, bias on rank 0) all-reduced over the group, in one launch."""
    _check_operands(x, weight, bias)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if weight.stride(-1) != 1:
        weight = weight.contiguous()
    bias = bias.contiguous() if bias is not None else None
    m, n = x2.shape[0], weight.shape[0]
    out = torch.empty((m, n), dtype=x.dtype, device=x.device)
    if m == 0:
        return out.reshape(*lead, n)
    state = group_state
    world, rank, ws, epoch = 1, 0, None, 0
    if state is not None and state.world > 1:
        state.ensure(m, n)
        world, rank, ws, epoch = state.world, state.rank, state.workspaces(), state.next_epoch()
    p = _params(x2, weight, bias, out, rank, world, ws, epoch)
    lib = _lib.load_library()
    _lib.check(lib.jt_row_linear_launch(ctypes.byref(p), _launch.stream_handle(x.device)))
    return out.reshape(*lead, n)


def row_parallel_linear_emulated(xs, weights, bias=None, *, workspaces=None):
    """Test form on one GPU: every rank of a group in one launch.

    xs[r] / weights[r] are rank r's input and weight shards (all on the current device);
    returns each rank's all-reduced output.  ``workspaces`` ([world] uint8 tensors of
    jt_row_linear_workspace_size bytes, zeroed before their first use, with their epoch)
    may be passed as ``(tensors, epoch)`` to reuse them across calls.
    """
    world = len(xs)
    lib = _lib.load_library()
    m, n = xs[0].shape[0], weights[0].shape[0]
    if workspaces is None:
        nbytes = int(lib.jt_row_linear_workspace_size(m, n, world))
        tensors = [torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=xs[0].device)
                   for _ in range(world)] if world > 1 else []
        epoch = 1
    else:
        tensors, epoch = workspaces
    array = (ctypes.c_void_p * world)(*[t.data_ptr() for t in tensors]) if world > 1 else None
    outs, params = [], (_lib.JtRowLinearParams * world)()
    for r in range(world):
        _check_operands(xs[r], weights[r], bias)
        out = torch.empty((m, n), dtype=xs[r].dtype, device=xs[r].device)
        outs.append(out)
        params[r] = _params(xs[r], weights[r], bias, out, r, world, array, epoch)
    _lib.check(lib.jt_row_linear_emulate(params, world, _launch.stream_handle(xs[0].device)))
    return outs


class RowParallelLinear(nn.Module):
    """The reference's RowParallelLinear (nanovllm/layers/linear.py:131-156) on the fused
    GEMM + all-reduce kernel.  tp rank / size come from torch.distributed (a single rank
    when no process group is initialised)."""

    def __init__(self, input_size: int, output_size: int, bias: bool = False):
        super().__init__()
        self.tp_size = dist.get_world_size() if dist.is_initialized() else 1
        self.tp_rank = dist.get_rank() if dist.is_initialized() else 0
        if input_size % self.tp_size:
            raise ValueError(f"{input_size} is not divisible by {self.tp_size}")
        self.tp_dim = 1
        self.weight = nn.Parameter(torch.empty(output_size, input_size // self.tp_size))
        self.weight.weight_loader = self.weight_loader
        if bias:
            self.bias = nn.Parameter(torch.empty(output_size))
            self.bias.weight_loader = self.weight_loader
        else:
            self.register_parameter("bias", None)

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        param_data = param.data
        if param_data.ndim == 1:
            param_data.copy_(loaded_weight)
            return
        shard_size = param_data.size(self.tp_dim)
        start_idx = self.tp_rank * shard_size
        param_data.copy_(loaded_weight.narrow(self.tp_dim, start_idx, shard_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        state = group_state_for(x.device) if self.tp_size > 1 else None
        return row_parallel_linear(x, self.weight, self.bias, state)
