"""ctypes binding of the C ABI in ``include/infercache.h``.

The shared library is built in-tree (``python -m infercache_b200.build``) and
loaded from ``infercache_b200/lib/libinfercache_b200.so``.  There is no
fallback: if the library is missing or no sm_100 device is current, the
calls that need it raise.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, c_char_p, c_float, c_int, c_int32, c_int64, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libinfercache_b200.so"

# ---- enums (infercache.h) ----------------------------------------------------
IC_OK = 0
IC_ERR_INVALID_ARG = -1
IC_ERR_UNSUPPORTED = -2
IC_ERR_OUT_OF_PAGES = -3
IC_ERR_SESSION_CAP = -4
IC_ERR_CORRUPT_TABLE = -5
IC_ERR_LAUNCH = -6
IC_ERR_DEVICE_TIMEOUT = -7
IC_ERR_CUDA = -8
IC_ERR_NO_DEVICE = -9

IC_F32, IC_F16, IC_BF16 = 0, 1, 2
IC_CTRL_SINK_FILL, IC_CTRL_RECENT_FILL, IC_CTRL_RECENT_PTR, IC_CTRL_IMPORTANT_FILL = 0, 1, 2, 3
IC_CTRL_WORDS = 8
IC_CNT_TOKENS_SEEN, IC_CNT_EVICTIONS, IC_CNT_STEPS, IC_CNT_PROMOTIONS, IC_CNT_NEAR_TIES = 0, 1, 2, 3, 4
IC_SUMMARY_STATIC_MASS_MAX = 4194304  # floats of ic_summary_score_static's static scratch
IC_COUNTER_WORDS = 8
IC_EV_NONE, IC_EV_DROP, IC_EV_FILL, IC_EV_EVICT, IC_EV_REJECT = 0, 1, 2, 3, 4
IC_DEVFLAG_TIMEOUT, IC_DEVFLAG_BAD_ROW = 1, 2
IC_DECODE_AUTO, IC_DECODE_CUDA_CORES, IC_DECODE_TENSOR_CORES, IC_DECODE_TENSOR_STREAM = 0, 1, 2, 3
IC_DECODE_TENSOR_LEAN = 4
IC_DECODE_TENSOR_SPLIT = 5

DTYPE_CODE = {torch.float32: IC_F32, torch.float16: IC_F16, torch.bfloat16: IC_BF16}


# ---- exceptions -----------------------------------------------------------------
class InferCacheError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class InvalidArgument(InferCacheError, ValueError):
    pass


class Unsupported(InferCacheError, NotImplementedError):
    pass


# ---- structs (field order and types exactly as in infercache.h) ---------------------
class ic_pool(Structure):
    _fields_ = [("k", c_void_p), ("v", c_void_p), ("pool_tokens", c_int64), ("num_layers", c_int32),
                ("num_kv_heads", c_int32), ("head_dim", c_int32), ("dtype", c_int32)]


class ic_tiers(Structure):
    _fields_ = [("sink_size", c_int32), ("recent_size", c_int32), ("important_size", c_int32),
                ("budget", c_int32)]


class ic_sessions(Structure):
    _fields_ = [("num_sessions", c_int32), ("_pad", c_int32), ("slot_table", c_void_p),
                ("positions", c_void_p), ("importance", c_void_p), ("occupied", c_void_p),
                ("ctrl", c_void_p), ("counters", c_void_p), ("dev_status", c_void_p)]


class ic_decode_args(Structure):
    _fields_ = [("pool", ic_pool), ("tiers", ic_tiers), ("sess", ic_sessions), ("layer", c_int32),
                ("num_q_heads", c_int32), ("q", c_void_p), ("k_new", c_void_p), ("v_new", c_void_p),
                ("out", c_void_p), ("out_dtype", c_int32), ("inputs_ready", c_int32), ("mass", c_void_p),
                ("scale", c_float), ("cluster_size", c_int32), ("kernel_variant", c_int32), ("pdl", c_int32)]


class ic_evict_args(Structure):
    _fields_ = [("tiers", ic_tiers), ("sess", ic_sessions), ("mass", c_void_p), ("mass_heads", c_int32),
                ("mass_layers", c_int32), ("mass_div", c_float), ("decay", c_float), ("pdl", c_int32),
                ("advance_pos", c_int32), ("new_pos", c_void_p), ("events", c_void_p)]


class ic_graph_state(Structure):
    _fields_ = [("k", c_void_p), ("v", c_void_p), ("positions", c_void_p), ("scores", c_void_p),
                ("centroid", c_void_p), ("cl_fill", c_void_p), ("c_count", c_void_p), ("ctrl", c_void_p),
                ("num_layers", c_int32), ("num_kv_heads", c_int32), ("head_dim", c_int32), ("dtype", c_int32),
                ("sink_size", c_int32), ("recent_size", c_int32), ("n_clusters", c_int32),
                ("cluster_capacity", c_int32), ("sim_threshold", c_float), ("_pad", c_int32)]


class ic_graph_push_args(Structure):
    _fields_ = [("g", ic_graph_state), ("k_src", c_void_p), ("v_src", c_void_p), ("stride_l", c_int64),
                ("stride_h", c_int64), ("stride_t", c_int64), ("positions", c_void_p), ("scores", c_void_p),
                ("slot_src", c_void_p), ("T", c_int32), ("reset", c_int32)]


class ic_graph_select_args(Structure):
    _fields_ = [("g", ic_graph_state), ("query", c_void_p), ("threshold", c_float), ("top_n", c_int32),
                ("selected", c_void_p), ("slots", c_void_p), ("count", c_void_p)]


class ic_step_args(Structure):
    _fields_ = [("layer0", ic_decode_args), ("q_layer_stride", c_int64), ("kv_layer_stride", c_int64),
                ("out_layer_stride", c_int64), ("evict", ic_evict_args)]


class ic_append_args(Structure):
    _fields_ = [("pool", ic_pool), ("tiers", ic_tiers), ("sess", ic_sessions), ("k", c_void_p),
                ("v", c_void_p), ("stride_s", c_int64), ("stride_l", c_int64), ("stride_h", c_int64)]


class ic_sort_args(Structure):
    _fields_ = [("tiers", ic_tiers), ("sess", ic_sessions), ("sorted_slots", c_void_p), ("fill", c_void_p)]


class ic_boost_args(Structure):
    _fields_ = [("tiers", ic_tiers), ("num_sessions", c_int32), ("L", c_int32), ("H", c_int32),
                ("Q", c_int32), ("width", c_int32), ("weights", c_void_p), ("sorted_slots", c_void_p),
                ("fill", c_void_p), ("mass_out", c_void_p)]


class ic_gather_args(Structure):
    _fields_ = [("pool", ic_pool), ("tiers", ic_tiers), ("sess", ic_sessions), ("session", c_int32),
                ("n", c_int32), ("slots", c_void_p), ("layer_begin", c_int32), ("layer_end", c_int32),
                ("k_out", c_void_p), ("v_out", c_void_p)]


class ic_tier_fill_args(Structure):
    _fields_ = [("tiers", ic_tiers), ("sess", ic_sessions), ("session0", c_int32), ("n", c_int32),
                ("T", c_int32), ("_pad", c_int32), ("scores", c_void_p), ("positions", c_void_p),
                ("slot_token", c_void_p)]


class ic_load_layer_args(Structure):
    _fields_ = [("pool", ic_pool), ("tiers", ic_tiers), ("sess", ic_sessions), ("session", c_int32),
                ("layer", c_int32), ("slot_token", c_void_p), ("k_src", c_void_p), ("v_src", c_void_p),
                ("stride_h", c_int64), ("stride_t", c_int64), ("src_dtype", c_int32), ("T", c_int32)]


class ic_reset_args(Structure):
    _fields_ = [("pool", ic_pool), ("tiers", ic_tiers), ("sess", ic_sessions), ("session0", c_int32),
                ("n", c_int32), ("zero_kv", c_int32)]


class ic_page_rows_args(Structure):
    _fields_ = [("pool", ic_pool), ("page_ids", c_void_p), ("n_page_ids", c_int32),
                ("layer_begin", c_int32), ("layer_end", c_int32), ("_pad", c_int32),
                ("start_token", c_int64), ("n_tokens", c_int64), ("k_buf", c_void_p), ("v_buf", c_void_p),
                ("stride_l", c_int64), ("stride_h", c_int64), ("stride_t", c_int64)]


class ic_summary_args(Structure):
    _fields_ = [("q", c_void_p), ("k", c_void_p), ("v", c_void_p), ("out", c_void_p), ("lse", c_void_p),
                ("head_mass", c_void_p), ("colsum", c_void_p), ("importance", c_void_p),
                ("batch", c_int32), ("num_q_heads", c_int32), ("num_kv_heads", c_int32), ("seq_len", c_int32),
                ("head_dim", c_int32), ("dtype", c_int32), ("accumulate", c_int32), ("scale", c_float),
                ("dev_status", c_void_p)]


class ic_index_rows_args(Structure):
    _fields_ = [("src", c_void_p), ("out", c_void_p), ("idx", c_void_p), ("stride_h", c_int64),
                ("stride_n", c_int64), ("H", c_int32), ("N", c_int32), ("F", c_int32), ("D", c_int32),
                ("dtype", c_int32), ("_pad", c_int32)]


class ic_scatter_mass_args(Structure):
    _fields_ = [("weights", c_void_p), ("slots", c_void_p), ("importance", c_void_p), ("rows", c_int32),
                ("width", c_int32), ("n_slots", c_int32), ("budget", c_int32)]


class ic_argmin_args(Structure):
    _fields_ = [("x", c_void_p), ("start", c_int32), ("n", c_int32), ("out_idx", c_void_p), ("out_val", c_void_p)]


class ic_compact_attn_args(Structure):
    _fields_ = [("q", c_void_p), ("k_buf", c_void_p), ("v_buf", c_void_p), ("slots", c_void_p), ("out", c_void_p),
                ("k_stride_h", c_int64), ("k_stride_n", c_int64), ("v_stride_h", c_int64),
                ("v_stride_n", c_int64), ("B", c_int32), ("H", c_int32), ("F", c_int32), ("D", c_int32),
                ("budget", c_int32), ("dtype", c_int32), ("scale", c_float), ("_pad", c_int32)]


# entry point name -> argument struct (None for the library-information calls)
ENTRY_POINTS = {
    "ic_decode_layer": ic_decode_args,
    "ic_evict_update": ic_evict_args,
    "ic_decode_step": ic_step_args,
    "ic_append_staging": ic_append_args,
    "ic_sort_slots": ic_sort_args,
    "ic_boost_sorted": ic_boost_args,
    "ic_gather_slots": ic_gather_args,
    "ic_tier_fill": ic_tier_fill_args,
    "ic_load_layer": ic_load_layer_args,
    "ic_reset_sessions": ic_reset_args,
    "ic_page_gather": ic_page_rows_args,
    "ic_page_write": ic_page_rows_args,
    "ic_summary_score": ic_summary_args,
    "ic_summary_score_static": ic_summary_args,
    "ic_index_rows": ic_index_rows_args,
    "ic_scatter_mass": ic_scatter_mass_args,
    "ic_argmin_range": ic_argmin_args,
    "ic_compact_attention": ic_compact_attn_args,
    "ic_graph_push": ic_graph_push_args,
    "ic_graph_select": ic_graph_select_args,
}
# entry points over an array of argument structs: (const args*, int32 count, stream)
BATCH_ENTRY_POINTS = {
    "ic_page_gather_batch": ic_page_rows_args,
    "ic_page_write_batch": ic_page_rows_args,
}
IC_PAGE_BATCH_MAX = 32
INFO_ENTRY_POINTS = ["ic_status_str", "ic_abi_version", "ic_device_check", "ic_last_error"]
HOST_ENTRY_POINTS = ["ic_host_device_pointer", "ic_wait_probe", "ic_graph_replay"]

_LIB = None


def load(path: Path = LIB_PATH):
    """Load the library (once) and declare every entry point's signature."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not Path(path).exists():
        raise ImportError(f"{path} is missing: run `python -m infercache_b200.build` "
                          "(the CUDA library is required; there is no CPU path)")
    lib = ctypes.CDLL(str(path), mode=os.RTLD_LOCAL)
    for name, st in ENTRY_POINTS.items():
        fn = getattr(lib, name)
        fn.argtypes = [POINTER(st), c_void_p]
        fn.restype = c_int
    for name, st in BATCH_ENTRY_POINTS.items():
        fn = getattr(lib, name)
        fn.argtypes = [POINTER(st), c_int32, c_void_p]
        fn.restype = c_int
    lib.ic_status_str.argtypes = [c_int]
    lib.ic_status_str.restype = c_char_p
    lib.ic_abi_version.argtypes = []
    lib.ic_abi_version.restype = c_int
    lib.ic_device_check.argtypes = []
    lib.ic_device_check.restype = c_int
    lib.ic_last_error.argtypes = []
    lib.ic_last_error.restype = c_char_p
    lib.ic_host_device_pointer.argtypes = [c_void_p, POINTER(c_void_p)]
    lib.ic_host_device_pointer.restype = c_int
    lib.ic_wait_probe.argtypes = [c_void_p, c_int64, c_void_p]
    lib.ic_wait_probe.restype = c_int
    lib.ic_graph_replay.argtypes = [POINTER(c_void_p), POINTER(c_void_p), c_int32, c_int32]
    lib.ic_graph_replay.restype = c_int
    _LIB = lib
    return lib


def raise_for(status: int, what: str = "") -> None:
    if status == IC_OK:
        return
    lib = load()
    msg = f"{what}: {lib.ic_status_str(status).decode()} ({lib.ic_last_error().decode()})"
    if status == IC_ERR_INVALID_ARG:
        raise InvalidArgument(status, msg)
    if status == IC_ERR_UNSUPPORTED:
        raise Unsupported(status, msg)
    raise InferCacheError(status, msg)


def call(name: str, args) -> None:
    """Call entry point `name` with a struct on torch's current CUDA stream."""
    lib = load()
    stream = torch.cuda.current_stream().cuda_stream
    raise_for(getattr(lib, name)(ctypes.byref(args), c_void_p(stream)), name)


def call_batch(name: str, args) -> None:
    """Call batch entry point `name` with a list of structs (at most
    IC_PAGE_BATCH_MAX) on torch's current CUDA stream."""
    lib = load()
    stream = torch.cuda.current_stream().cuda_stream
    st = BATCH_ENTRY_POINTS[name]
    arr = (st * len(args))(*args)
    raise_for(getattr(lib, name)(arr, len(args), c_void_p(stream)), name)


_DEVICE_OK = {}


def require_device(device: torch.device) -> None:
    """Fail loudly unless `device` is an sm_100 GPU and the library loads."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError(f"infercache_b200 runs on CUDA devices only, got {device}")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx in _DEVICE_OK:
        return
    lib = load()
    with torch.cuda.device(idx):
        rc = lib.ic_device_check()
    raise_for(rc, "device check")
    _DEVICE_OK[idx] = True


def host_device_pointer(t: torch.Tensor) -> int:
    """Device address of a pinned (page-locked, mapped) host tensor's data
    (``ic_host_device_pointer``), for kernels that read or write it over PCIe."""
    if t.device.type != "cpu" or not t.is_pinned():
        raise ValueError("host_device_pointer needs a pinned host tensor")
    lib = load()
    out = c_void_p()
    raise_for(lib.ic_host_device_pointer(c_void_p(t.data_ptr()), ctypes.byref(out)), "ic_host_device_pointer")
    return int(out.value)


def ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise ValueError(f"unsupported dtype {dt}; use float32, float16 or bfloat16") from None
