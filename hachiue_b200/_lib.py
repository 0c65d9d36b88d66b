"""ctypes binding of libhachiue_cuda.so (the C ABI in include/hachiue_cuda.h).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libhachiue_cuda.so")

HCU_OK, HCU_EINVAL, HCU_ECUDA, HCU_ENCCL, HCU_ETIMEDOUT, HCU_ENOMEM, HCU_EUNSUPPORTED = range(7)
KV_F32, KV_F16, KV_BF16, KV_Q8_0, KV_Q8_0_WGSL = 0, 1, 2, 3, 4
OPT_ATTN_CUDA_CORES, OPT_ATTN_CHUNK, OPT_GDN_SCRATCH_MB, OPT_SWA_CTAS, OPT_GDN_CHAIN_COLS = 1, 2, 3, 4, 5
COMM_ID_BYTES = 128
DT_F32, DT_BF16 = 0, 2

STATUS_NAMES = {
    HCU_OK: "HCU_OK", HCU_EINVAL: "HCU_EINVAL", HCU_ECUDA: "HCU_ECUDA", HCU_ENCCL: "HCU_ENCCL",
    HCU_ETIMEDOUT: "HCU_ETIMEDOUT", HCU_ENOMEM: "HCU_ENOMEM", HCU_EUNSUPPORTED: "HCU_EUNSUPPORTED",
}

# Every symbol include/hachiue_cuda.h declares (checked by the CPU tests).
EXPORTS = (
    "hcu_version", "hcu_last_error", "hcu_create", "hcu_destroy", "hcu_set_stream", "hcu_get_stream",
    "hcu_stream_sync", "hcu_alloc", "hcu_free", "hcu_memset", "hcu_copy_to_device", "hcu_copy_to_host",
    "hcu_device_status", "hcu_inject_failure", "hcu_selftest_wait_timeout", "hcu_comm_create", "hcu_comm_destroy",
    "hcu_allgather", "hcu_dispatch", "hcu_attention", "hcu_attention_noalloc", "hcu_kv_append", "hcu_kv_append_rows",
    "hcu_deltanet_gbeta", "hcu_deltanet_recur", "hcu_deltanet_decode", "hcu_swa_prefill",
    "hcu_deltanet_chunked_prefill", "hcu_deltanet_chunked_prefill_snap", "hcu_conv1d_causal", "hcu_deltanet_norm_gate", "hcu_gdn_layer_step",
    "hcu_rmsnorm", "hcu_rope", "hcu_split_q_gate", "hcu_sigmoid_gate", "hcu_attn_prologue",
    "hcu_selftest_dirty_tickets", "hcu_attention_noalloc_status", "hcu_set_q8_convention", "hcu_set_option",
    "hcu_comm_unique_id", "hcu_comm_init_rank", "hcu_kv_append_rows_kv",
)


class HachiueError(RuntimeError):
    """A failed C-ABI call; ``status`` is the HCU_* code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class hcu_kv_cache(ctypes.Structure):
    _fields_ = [("format", ctypes.c_uint32), ("rows", ctypes.c_uint32), ("k", ctypes.c_void_p),
                ("v", ctypes.c_void_p), ("k_scale", ctypes.c_void_p), ("v_scale", ctypes.c_void_p)]


class hcu_attention_params(ctypes.Structure):
    _fields_ = [("S", ctypes.c_uint32), ("H", ctypes.c_uint32), ("KV", ctypes.c_uint32), ("Dh", ctypes.c_uint32),
                ("posBase", ctypes.c_uint32), ("windowSize", ctypes.c_uint32), ("batch", ctypes.c_uint32),
                ("max_context", ctypes.c_uint32), ("pos_base", ctypes.c_void_p),
                ("kv_row_offset", ctypes.c_void_p), ("seq_row_stride", ctypes.c_uint64), ("gate", ctypes.c_void_p)]


class hcu_attn_prologue_params(ctypes.Structure):
    _fields_ = [("S", ctypes.c_uint32), ("H", ctypes.c_uint32), ("KV", ctypes.c_uint32), ("Dh", ctypes.c_uint32),
                ("rotaryDim", ctypes.c_uint32), ("posBase", ctypes.c_uint32), ("batch", ctypes.c_uint32),
                ("split_gate", ctypes.c_uint32), ("eps", ctypes.c_float), ("pos_base", ctypes.c_void_p),
                ("kv_row_offset", ctypes.c_void_p), ("seq_row_stride", ctypes.c_uint64)]


class hcu_deltanet_params(ctypes.Structure):
    _fields_ = [("S", ctypes.c_uint32), ("H", ctypes.c_uint32), ("DK", ctypes.c_uint32), ("DV", ctypes.c_uint32),
                ("HK", ctypes.c_uint32), ("loadState", ctypes.c_uint32), ("batch", ctypes.c_uint32),
                ("qkv_seq_stride", ctypes.c_uint64), ("gbeta_seq_stride", ctypes.c_uint64),
                ("state_seq_stride", ctypes.c_uint64), ("core_seq_stride", ctypes.c_uint64)]


class hcu_conv1d_params(ctypes.Structure):
    _fields_ = [("S", ctypes.c_uint32), ("C", ctypes.c_uint32), ("K", ctypes.c_uint32), ("loadState", ctypes.c_uint32),
                ("batch", ctypes.c_uint32), ("x_seq_stride", ctypes.c_uint64), ("y_seq_stride", ctypes.c_uint64),
                ("state_seq_stride", ctypes.c_uint64)]


class hcu_gdn_step_params(ctypes.Structure):
    _fields_ = [("H", ctypes.c_uint32), ("HK", ctypes.c_uint32), ("DK", ctypes.c_uint32), ("DV", ctypes.c_uint32),
                ("K", ctypes.c_uint32), ("loadState", ctypes.c_uint32), ("batch", ctypes.c_uint32),
                ("eps", ctypes.c_float), ("qkv_seq_stride", ctypes.c_uint64), ("conv_seq_stride", ctypes.c_uint64),
                ("ab_seq_stride", ctypes.c_uint64), ("z_seq_stride", ctypes.c_uint64),
                ("state_seq_stride", ctypes.c_uint64), ("out_seq_stride", ctypes.c_uint64)]


class hcu_swa_params(ctypes.Structure):
    _fields_ = [("B", ctypes.c_uint32), ("T", ctypes.c_uint32), ("H", ctypes.c_uint32), ("KV", ctypes.c_uint32),
                ("D", ctypes.c_uint32), ("window", ctypes.c_uint32), ("out_dtype", ctypes.c_uint32)]


class hcu_gdn_prefill_params(ctypes.Structure):
    _fields_ = [("B", ctypes.c_uint32), ("T", ctypes.c_uint32), ("NK", ctypes.c_uint32), ("NV", ctypes.c_uint32),
                ("D", ctypes.c_uint32), ("load_state", ctypes.c_uint32),
                ("q_row_stride", ctypes.c_uint64), ("k_row_stride", ctypes.c_uint64),
                ("v_row_stride", ctypes.c_uint64), ("q_seq_stride", ctypes.c_uint64),
                ("k_seq_stride", ctypes.c_uint64), ("v_seq_stride", ctypes.c_uint64),
                ("gb_row_stride", ctypes.c_uint64), ("gb_seq_stride", ctypes.c_uint64)]


_lock = threading.Lock()
_lib = None


def load(path: str | None = None):
    """Load (once) and return the ctypes library.  Raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise ImportError(
                f"hachiue: CUDA library {p} is not built; run `python -m hachiue_b200.build` "
                "(there is no CPU fallback)")
        L = ctypes.CDLL(p)
        vp, u32, i32, sz = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_size_t
        sig = {
            "hcu_version": ([], i32),
            "hcu_last_error": ([], ctypes.c_char_p),
            "hcu_create": ([i32, sz, ctypes.POINTER(vp)], i32),
            "hcu_destroy": ([vp], i32),
            "hcu_set_stream": ([vp, vp], i32),
            "hcu_get_stream": ([vp], vp),
            "hcu_stream_sync": ([vp], i32),
            "hcu_alloc": ([vp, sz, ctypes.POINTER(vp)], i32),
            "hcu_free": ([vp, vp], i32),
            "hcu_memset": ([vp, vp, i32, sz], i32),
            "hcu_copy_to_device": ([vp, vp, vp, sz], i32),
            "hcu_copy_to_host": ([vp, vp, vp, sz], i32),
            "hcu_device_status": ([vp, ctypes.POINTER(u32), i32], i32),
            "hcu_inject_failure": ([vp, i32, i32], i32),
            "hcu_selftest_wait_timeout": ([vp], i32),
            "hcu_comm_create": ([i32, ctypes.POINTER(i32), ctypes.POINTER(vp)], i32),
            "hcu_comm_destroy": ([vp], i32),
            "hcu_allgather": ([vp, ctypes.POINTER(vp), ctypes.POINTER(vp), sz, ctypes.POINTER(vp)], i32),
            "hcu_dispatch": ([vp, ctypes.c_char_p, ctypes.POINTER(u32), ctypes.POINTER(vp), i32], i32),
            "hcu_attention": ([vp, ctypes.POINTER(hcu_attention_params), vp, ctypes.POINTER(hcu_kv_cache), vp], i32),
            "hcu_attention_noalloc": ([ctypes.POINTER(hcu_attention_params), vp, ctypes.POINTER(hcu_kv_cache), vp,
                                       vp], i32),
            "hcu_kv_append": ([vp, u32, u32, u32, u32, u32, vp, vp, vp], i32),
            "hcu_kv_append_rows": ([vp, u32, u32, u32, u32, vp, vp, vp, vp], i32),
            "hcu_deltanet_gbeta": ([vp, u32, u32, vp, vp, vp, vp, vp], i32),
            "hcu_deltanet_recur": ([vp, ctypes.POINTER(hcu_deltanet_params), vp, vp, vp, vp, vp], i32),
            "hcu_deltanet_decode": ([vp, ctypes.POINTER(hcu_deltanet_params), vp, vp, vp, vp, vp, vp, vp, vp], i32),
            "hcu_swa_prefill": ([vp, ctypes.POINTER(hcu_swa_params), vp, vp, vp, vp], i32),
            "hcu_deltanet_chunked_prefill": ([vp, ctypes.POINTER(hcu_gdn_prefill_params), vp, vp, vp, vp, vp, vp,
                                              vp, vp], i32),
            "hcu_deltanet_chunked_prefill_snap": ([vp, ctypes.POINTER(hcu_gdn_prefill_params), vp, vp, vp, vp, vp,
                                                   vp, vp, vp, u32, vp], i32),
            "hcu_conv1d_causal": ([vp, ctypes.POINTER(hcu_conv1d_params), vp, vp, vp, vp, vp], i32),
            "hcu_deltanet_norm_gate": ([vp, u32, u32, ctypes.c_float, vp, vp, vp, vp], i32),
            "hcu_gdn_layer_step": ([vp, ctypes.POINTER(hcu_gdn_step_params)] + [vp] * 13, i32),
            "hcu_rmsnorm": ([vp, u32, u32, ctypes.c_float, u32, vp, vp, vp], i32),
            "hcu_rope": ([vp, u32, u32, u32, u32, u32, vp, vp, vp], i32),
            "hcu_split_q_gate": ([vp, u32, u32, u32, vp, vp, vp], i32),
            "hcu_sigmoid_gate": ([vp, ctypes.c_uint64, vp, vp], i32),
            "hcu_attn_prologue": ([vp, ctypes.POINTER(hcu_attn_prologue_params)] + [vp] * 9
                                  + [ctypes.POINTER(hcu_kv_cache)], i32),
            "hcu_selftest_dirty_tickets": ([vp], i32),
            "hcu_attention_noalloc_status": ([ctypes.POINTER(u32), i32, vp], i32),
            "hcu_set_q8_convention": ([vp, u32], i32),
            "hcu_set_option": ([vp, i32, ctypes.c_int64], i32),
            "hcu_comm_unique_id": ([ctypes.POINTER(ctypes.c_uint8)], i32),
            "hcu_comm_init_rank": ([i32, i32, ctypes.POINTER(ctypes.c_uint8), i32, i32, ctypes.POINTER(vp)], i32),
            "hcu_kv_append_rows_kv": ([vp, u32, u32, u32, vp, vp, vp, ctypes.POINTER(hcu_kv_cache)], i32),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
        return L


def check(status: int) -> None:
    """Raise HachiueError for a non-zero status, with hcu_last_error()."""
    if status != HCU_OK:
        msg = load().hcu_last_error().decode(errors="replace")
        raise HachiueError(status, f"{STATUS_NAMES.get(status, status)}: {msg}")
