"""ctypes binding of the C ABI in include/jetspec_b200.h.

The shared library is the only compute path: if it is missing or fails to load, every
public operator raises ``LibraryMissingError``.  There is no fallback of any kind.
"""
from __future__ import annotations

import ctypes
from pathlib import Path
import threading

LIBRARY_PATH = Path(__file__).resolve().parent / "libjetspec_b200.so"
ABI_VERSION = 1

JT_OK = 0
JT_ERR_INVALID = -1
JT_ERR_WORKSPACE = -2
JT_ERR_CUDA = -3
JT_ERR_UNSUPPORTED = -4

JT_BF16, JT_F16, JT_F32 = 0, 1, 2
JT_FLAG_FP32_PROBABILITY = 1
JT_FLAG_PORTABLE_CORE = 2

EXPORTED_SYMBOLS = (
    "jt_tree_attn_workspace_size",
    "jt_tree_attn_launch",
    "jt_tree_attn_launch_noalloc",
    "jt_kv_store_launch",
    "jt_kv_commit_launch",
    "jt_rope_scatter_launch",
    "jt_accept_walk_launch",
    "jt_selftest_bounded_wait",
    "jt_metadata_build_launch",
    "jt_row_linear_launch",
    "jt_row_linear_workspace_size",
    "jt_row_linear_emulate",
    "jt_device_alloc_zeroed",
    "jt_device_free",
    "jt_ipc_get_handle",
    "jt_ipc_open_handle",
    "jt_ipc_close_handle",
    "jt_kv_commit_max_slots",
    "jt_abi_version",
    "jt_last_error",
    "jt_read_device_errors",
)


class LibraryMissingError(RuntimeError):
    """The sm_100a kernel library is not built or cannot be loaded."""


class KernelLaunchError(RuntimeError):
    """The C ABI rejected or failed a launch; the message comes from jt_last_error()."""


c_void_p = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_u32 = ctypes.c_uint32
c_i64 = ctypes.c_int64


class JtTreeAttnParams(ctypes.Structure):
    _fields_ = [
        ("out", c_void_p), ("q", c_void_p), ("k_pool", c_void_p), ("v_pool", c_void_p),
        ("cu_seqlens_q", c_void_p), ("query_to_request", c_void_p),
        ("query_local_row", c_void_p), ("prefix_lens", c_void_p), ("node_counts", c_void_p),
        ("block_tables", c_void_p), ("tree_slots", c_void_p), ("qq_bias", c_void_p),
        ("qq_bias_offsets", c_void_p),
        ("num_requests", c_i32), ("total_queries", c_i32), ("num_kv_heads", c_i32),
        ("groups", c_i32), ("head_dim", c_i32), ("block_size", c_i32), ("table_width", c_i32),
        ("dtype", c_i32), ("out_dtype", c_i32), ("flags", c_u32),
        ("num_blocks", c_i64),
        ("q_stride0", c_i64), ("q_stride1", c_i64), ("out_stride0", c_i64),
        ("out_stride1", c_i64), ("table_stride0", c_i64),
        ("k_stride0", c_i64), ("k_stride1", c_i64), ("k_stride2", c_i64),
        ("v_stride0", c_i64), ("v_stride1", c_i64), ("v_stride2", c_i64),
        ("scale", ctypes.c_float), ("split_keys", c_i32),
        ("workspace", c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


class JtKvStoreParams(ctypes.Structure):
    _fields_ = [
        ("key", c_void_p), ("value", c_void_p), ("k_cache", c_void_p), ("v_cache", c_void_p),
        ("slot_mapping", c_void_p), ("slot_is_int64", c_i32), ("num_tokens", c_i32),
        ("num_kv_heads", c_i32), ("head_dim", c_i32), ("elem_bytes", c_i32),
        ("block_size", c_i32), ("num_blocks", c_i64),
        ("key_stride0", c_i64), ("key_stride1", c_i64),
        ("value_stride0", c_i64), ("value_stride1", c_i64),
        ("k_stride0", c_i64), ("k_stride1", c_i64), ("k_stride2", c_i64),
        ("v_stride0", c_i64), ("v_stride1", c_i64), ("v_stride2", c_i64),
    ]


class JtKvCommitParams(ctypes.Structure):
    _fields_ = [
        ("kv_pool", c_void_p), ("source_slots", c_void_p), ("destination_slots", c_void_p),
        ("slot_is_int64", c_i32), ("num_slots", c_i32), ("num_layers", c_i32),
        ("num_kv_heads", c_i32), ("head_dim", c_i32), ("elem_bytes", c_i32),
        ("block_size", c_i32), ("num_blocks", c_i64),
        ("stride_axis", c_i64), ("stride_layer", c_i64), ("stride_block", c_i64),
        ("stride_offset", c_i64), ("stride_head", c_i64),
    ]


class JtRopeScatterParams(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("positions", c_void_p),
        ("cos_sin_cache", c_void_p), ("node_slots", c_void_p), ("out", c_void_p),
        ("k_pool", c_void_p), ("v_pool", c_void_p),
        ("dtype", c_i32), ("cache_dtype", c_i32), ("positions_is_int64", c_i32),
        ("slots_is_int64", c_i32), ("rows", c_i32), ("q_heads", c_i32), ("kv_heads", c_i32),
        ("head_dim", c_i32), ("page_size", c_i32), ("num_pages", c_i64),
        ("q_stride0", c_i64), ("q_stride1", c_i64), ("q_stride2", c_i64),
        ("k_stride0", c_i64), ("k_stride1", c_i64), ("k_stride2", c_i64),
        ("v_stride0", c_i64), ("v_stride1", c_i64), ("v_stride2", c_i64),
        ("positions_stride", c_i64), ("slots_stride", c_i64), ("cache_stride0", c_i64),
        ("cache_stride_last", c_i64),
        ("out_stride0", c_i64), ("out_stride1", c_i64), ("out_stride2", c_i64),
        ("kp_stride0", c_i64), ("kp_stride1", c_i64), ("kp_stride2", c_i64), ("kp_stride3", c_i64),
        ("vp_stride0", c_i64), ("vp_stride1", c_i64), ("vp_stride2", c_i64), ("vp_stride3", c_i64),
    ]


class JtAcceptWalkParams(ctypes.Structure):
    _fields_ = [
        ("logits", c_void_p), ("token_ids", c_void_p), ("parent_indices", c_void_p),
        ("depths", c_void_p), ("offsets", c_void_p), ("path", c_void_p),
        ("accepted_length", c_void_p), ("correction", c_void_p), ("outputs", c_void_p),
        ("logits_stride0", c_i64), ("logits_dtype", c_i32), ("vocab", c_i32),
        ("num_requests", c_i32), ("max_depth", c_i32), ("path_stride", c_i32),
        ("num_nodes", c_i32),
    ]


class JtMetadataBuildParams(ctypes.Structure):
    _fields_ = [
        ("node_counts", c_void_p), ("parents", c_void_p), ("arena_pages", c_void_p),
        ("cu_seqlens_q", c_void_p), ("query_to_request", c_void_p),
        ("query_local_row", c_void_p), ("tree_slots", c_void_p), ("qq_bias", c_void_p),
        ("qq_bias_offsets", c_void_p), ("num_requests", c_i32), ("block_size", c_i32),
        ("max_nodes", c_i32), ("num_nodes", c_i32), ("num_pages", c_i32),
    ]


class JtRowLinearParams(ctypes.Structure):
    _fields_ = [
        ("x", c_void_p), ("weight", c_void_p), ("bias", c_void_p), ("out", c_void_p),
        ("m", c_i64), ("n", c_i64), ("k", c_i64), ("x_stride", c_i64), ("w_stride", c_i64),
        ("dtype", c_i32), ("rank", c_i32), ("world", c_i32),
        ("workspaces", ctypes.POINTER(c_void_p)), ("epoch", c_u32),
        ("wait_limit_cycles", c_i64),
    ]


_lock = threading.Lock()
_lib = None


def _declare(lib):
    P = ctypes.POINTER
    lib.jt_tree_attn_workspace_size.argtypes = [c_i32, c_i32, c_i32, c_i32, c_i32,
                                                P(ctypes.c_size_t)]
    lib.jt_tree_attn_workspace_size.restype = ctypes.c_int
    lib.jt_tree_attn_launch.argtypes = [P(JtTreeAttnParams), c_void_p]
    lib.jt_tree_attn_launch.restype = ctypes.c_int
    lib.jt_tree_attn_launch_noalloc.argtypes = [P(JtTreeAttnParams), c_void_p]
    lib.jt_tree_attn_launch_noalloc.restype = ctypes.c_int
    lib.jt_kv_store_launch.argtypes = [P(JtKvStoreParams), c_void_p]
    lib.jt_kv_store_launch.restype = ctypes.c_int
    lib.jt_kv_commit_launch.argtypes = [P(JtKvCommitParams), c_void_p]
    lib.jt_kv_commit_launch.restype = ctypes.c_int
    lib.jt_rope_scatter_launch.argtypes = [P(JtRopeScatterParams), c_void_p]
    lib.jt_rope_scatter_launch.restype = ctypes.c_int
    lib.jt_accept_walk_launch.argtypes = [P(JtAcceptWalkParams), c_void_p]
    lib.jt_accept_walk_launch.restype = ctypes.c_int
    lib.jt_selftest_bounded_wait.argtypes = [c_i64, P(c_i32)]
    lib.jt_selftest_bounded_wait.restype = ctypes.c_int
    lib.jt_metadata_build_launch.argtypes = [P(JtMetadataBuildParams), c_void_p]
    lib.jt_metadata_build_launch.restype = ctypes.c_int
    lib.jt_row_linear_launch.argtypes = [P(JtRowLinearParams), c_void_p]
    lib.jt_row_linear_launch.restype = ctypes.c_int
    lib.jt_row_linear_emulate.argtypes = [P(JtRowLinearParams), c_i32, c_void_p]
    lib.jt_row_linear_emulate.restype = ctypes.c_int
    lib.jt_row_linear_workspace_size.argtypes = [c_i64, c_i64, c_i32]
    lib.jt_row_linear_workspace_size.restype = c_i64
    lib.jt_device_alloc_zeroed.argtypes = [c_i64, P(c_void_p)]
    lib.jt_device_alloc_zeroed.restype = ctypes.c_int
    lib.jt_device_free.argtypes = [c_void_p]
    lib.jt_device_free.restype = ctypes.c_int
    lib.jt_ipc_get_handle.argtypes = [c_void_p, c_void_p]
    lib.jt_ipc_get_handle.restype = ctypes.c_int
    lib.jt_ipc_open_handle.argtypes = [c_void_p, P(c_void_p)]
    lib.jt_ipc_open_handle.restype = ctypes.c_int
    lib.jt_ipc_close_handle.argtypes = [c_void_p]
    lib.jt_ipc_close_handle.restype = ctypes.c_int
    lib.jt_kv_commit_max_slots.argtypes = []
    lib.jt_kv_commit_max_slots.restype = c_i32
    lib.jt_abi_version.argtypes = []
    lib.jt_abi_version.restype = c_i32
    lib.jt_last_error.argtypes = []
    lib.jt_last_error.restype = ctypes.c_char_p
    lib.jt_read_device_errors.argtypes = [P(c_u32)]
    lib.jt_read_device_errors.restype = ctypes.c_int


def load_library(path: Path | None = None):
    """Load (once) and return the ctypes handle of libjetspec_b200.so."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        target = Path(path) if path is not None else LIBRARY_PATH
        if not target.exists():
            raise LibraryMissingError(
                f"{target.name} is not built; run `python -c \"import __graft_entry__ as g; "
                f"g.build()\"` from the repository root (needs nvcc for sm_100a)")
        try:
            lib = ctypes.CDLL(str(target))
        except OSError as error:
            raise LibraryMissingError(f"cannot load {target}: {error}") from error
        missing = [name for name in EXPORTED_SYMBOLS if not hasattr(lib, name)]
        if missing:
            raise LibraryMissingError(f"{target.name} lacks symbols {missing}")
        _declare(lib)
        if lib.jt_abi_version() != ABI_VERSION:
            raise LibraryMissingError(
                f"{target.name} ABI {lib.jt_abi_version()} != expected {ABI_VERSION}")
        if path is None:
            _lib = lib
        return lib


def check(status: int) -> None:
    if status == JT_OK:
        return
    message = load_library().jt_last_error().decode(errors="replace")
    if status in (JT_ERR_INVALID, JT_ERR_UNSUPPORTED):
        raise ValueError(message)
    raise KernelLaunchError(f"status {status}: {message}")


def read_device_errors() -> int:
    """Read and clear the device error words (synchronises; diagnostics only)."""
    lib = load_library()
    bits = c_u32(0)
    check(lib.jt_read_device_errors(ctypes.byref(bits)))
    return int(bits.value)


def selftest_bounded_wait(limit_cycles: int) -> tuple[int, int, int]:
    """Run the bounded-wait self-test (synchronous): (claimed completion, abort flag, cycles)."""
    lib = load_library()
    out = (c_i32 * 3)()
    check(lib.jt_selftest_bounded_wait(int(limit_cycles), out))
    return int(out[0]), int(out[1]), int(out[2])
