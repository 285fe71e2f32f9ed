"""ctypes binding of the C ABI in include/ttjam_b200.h.

The shared library is built in-tree (`build.py`). Loading fails loudly when it
is missing: there is no CPU or eager-PyTorch fallback for the forward pass.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

TT_ABI_VERSION = 2

TT_OK = 0
TT_ERR_INVALID_CONFIG = -1
TT_ERR_INVALID_ARGUMENT = -2
TT_ERR_UNSUPPORTED = -3
TT_ERR_WORKSPACE = -4
TT_ERR_CUDA = -5
TT_ERR_DEVICE_TIMEOUT = -6
TT_ERR_DEVICE_FAULT = -7
TT_ERR_DEVICE_RANGE = -8

# tt_config.flags: the automatic plan never picks the fp16-split schedule.
TT_FLAG_FP32_ONLY = 1
# Largest finite fp16 value; tt_fp16_operand_bound must stay below it for the
# split-precision schedule.
TT_FP16_MAX = 65504.0

# Size of the library's fixed scratch array behind tt_forward_noalloc.
TT_NOALLOC_SCRATCH_BYTES = 16 << 20

PLAN_NAMES = {1: "cluster", 2: "ops_ffma", 3: "ops_tc", 4: "tile"}
PLAN_IDS = {"auto": 0, **{v: k for k, v in PLAN_NAMES.items()}}

# Every entry point include/ttjam_b200.h declares.
EXPORTED = (
    "tt_abi_version", "tt_validate_config", "tt_image_bytes", "tt_pack_image",
    "tt_workspace_bytes", "tt_forward", "tt_forward_plan", "tt_forward_launch_count",
    "tt_read_status", "tt_last_error", "tt_forward_noalloc", "tt_fp16_operand_bound",
    "tt_launch_probe_start", "tt_launch_probe_read", "tt_test_arm_wait_timeout",
    "tt_pack_image_typed", "tt_typed_workspace_bytes", "tt_forward_typed",
    "tt_host_workspace_bytes", "tt_forward_host", "tt_test_gelu",
)

# Element types of the typed entry points (TT_DTYPE_*), by torch dtype name.
TT_DTYPE_F32 = 0
TT_DTYPE_F16 = 1
TT_DTYPE_BF16 = 2
DTYPE_CODES = {"float32": TT_DTYPE_F32, "float16": TT_DTYPE_F16, "bfloat16": TT_DTYPE_BF16}

# TT_KERNEL_* launch kinds reported by tt_launch_probe_read.
KERNEL_KINDS = {1: "layernorm", 2: "qkv", 3: "attention", 4: "out_proj", 5: "ffn_in",
                6: "ffn_out", 7: "final_norm", 8: "whole_forward", 9: "row_scan", 10: "convert"}


class TTConfig(ctypes.Structure):
    _fields_ = [("d_model", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("ffn_dim", ctypes.c_int32), ("num_layers", ctypes.c_int32),
                ("causal", ctypes.c_int32), ("plan", ctypes.c_int32),
                ("flags", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class TTLayerParams(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "norm1_weight", "norm1_bias", "q_weight", "q_bias", "k_weight", "k_bias",
        "v_weight", "v_bias", "out_weight", "out_bias", "norm2_weight", "norm2_bias",
        "ffn_in_weight", "ffn_in_bias", "ffn_out_weight", "ffn_out_bias")]


_lock = threading.Lock()
_lib = None


def lib_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load (building first if needed and allowed) the sm_100a library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(f"CUDA extension not built: {path} is missing "
                                   "(run python -m ttjam_gottagofast_b200.build)")
            _build.build()
        lib = ctypes.CDLL(path)
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
        cfgp = ctypes.POINTER(TTConfig)
        lib.tt_abi_version.restype = ctypes.c_int
        lib.tt_abi_version.argtypes = []
        lib.tt_validate_config.restype = ctypes.c_int
        lib.tt_validate_config.argtypes = [cfgp]
        lib.tt_image_bytes.restype = sz
        lib.tt_image_bytes.argtypes = [cfgp]
        lib.tt_pack_image.restype = ctypes.c_int
        lib.tt_pack_image.argtypes = [cfgp, ctypes.POINTER(TTLayerParams), vp, vp, vp, sz, vp]
        lib.tt_pack_image_typed.restype = ctypes.c_int
        lib.tt_pack_image_typed.argtypes = [cfgp, ctypes.c_int, ctypes.POINTER(TTLayerParams),
                                            vp, vp, vp, sz, vp]
        lib.tt_typed_workspace_bytes.restype = sz
        lib.tt_typed_workspace_bytes.argtypes = [cfgp, ctypes.c_int, i64, i64]
        lib.tt_forward_typed.restype = ctypes.c_int
        lib.tt_forward_typed.argtypes = [cfgp, vp, ctypes.c_int, vp, vp, i64, i64, vp, vp, sz, vp]
        lib.tt_host_workspace_bytes.restype = sz
        lib.tt_host_workspace_bytes.argtypes = [cfgp, i64, i64]
        lib.tt_forward_host.restype = ctypes.c_int
        lib.tt_forward_host.argtypes = [cfgp, vp, vp, vp, i64, i64, vp, vp, sz, vp]
        lib.tt_workspace_bytes.restype = sz
        lib.tt_workspace_bytes.argtypes = [cfgp, i64, i64]
        lib.tt_forward.restype = ctypes.c_int
        lib.tt_forward.argtypes = [cfgp, vp, vp, vp, i64, i64, vp, vp, sz, vp]
        lib.tt_forward_plan.restype = ctypes.c_int
        lib.tt_forward_plan.argtypes = [cfgp, i64, i64]
        lib.tt_forward_launch_count.restype = ctypes.c_int
        lib.tt_forward_launch_count.argtypes = [cfgp, i64, i64]
        lib.tt_forward_noalloc.restype = ctypes.c_int
        lib.tt_forward_noalloc.argtypes = [cfgp, vp, vp, vp, i64, i64, vp, vp]
        lib.tt_fp16_operand_bound.restype = ctypes.c_int
        lib.tt_fp16_operand_bound.argtypes = [cfgp, vp, ctypes.POINTER(ctypes.c_float), vp]
        lib.tt_read_status.restype = ctypes.c_int
        lib.tt_read_status.argtypes = [cfgp, vp, ctypes.POINTER(i32), ctypes.POINTER(i32), vp]
        lib.tt_last_error.restype = ctypes.c_int
        lib.tt_last_error.argtypes = [ctypes.c_char_p, sz]
        lib.tt_launch_probe_start.restype = ctypes.c_int
        lib.tt_launch_probe_start.argtypes = [ctypes.c_int]
        lib.tt_launch_probe_read.restype = ctypes.c_int
        lib.tt_launch_probe_read.argtypes = [ctypes.POINTER(ctypes.c_float),
                                             ctypes.POINTER(i32), ctypes.c_int]
        lib.tt_test_gelu.restype = ctypes.c_int
        lib.tt_test_gelu.argtypes = [vp, vp, i64, vp]
        lib.tt_test_arm_wait_timeout.restype = ctypes.c_int
        lib.tt_test_arm_wait_timeout.argtypes = [ctypes.c_int]
        if lib.tt_abi_version() != TT_ABI_VERSION:
            raise RuntimeError("libttjam_b200.so ABI version mismatch; rebuild it")
        _lib = lib
        return lib


def last_error(lib=None) -> str:
    lib = lib or load()
    buf = ctypes.create_string_buffer(1024)
    lib.tt_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, what: str, lib=None) -> None:
    """Map a negative tt_status to the Python exception the reference raises
    for the same condition (ValueError for config errors)."""
    if rc == TT_OK:
        return
    msg = f"{what}: {last_error(lib)} (status {rc})"
    if rc == TT_ERR_INVALID_CONFIG:
        raise ValueError(msg)
    if rc in (TT_ERR_INVALID_ARGUMENT, TT_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def make_config(cfg, plan: str = "auto", flags: int = 0) -> TTConfig:
    """A tt_config from any object with TransformerConfig's fields."""
    c = TTConfig()
    c.plan = PLAN_IDS[plan]
    c.flags = flags
    c.d_model = int(cfg.d_model)
    c.num_heads = int(cfg.num_heads)
    c.ffn_dim = int(cfg.ffn_dim)
    c.num_layers = int(cfg.num_layers)
    c.causal = 1 if cfg.causal else 0
    return c
