"""ctypes binding of libshardlm_cuda.so (the C ABI declared in include/shardlm_cuda.h).

There is no fallback: if the library cannot be loaded (or built with nvcc when it is missing or
older than its sources), every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

P = C.c_void_p
I32 = C.c_int
I64 = C.c_int64
U64 = C.c_uint64
F32 = C.c_float
PP = C.POINTER(C.c_void_p)

SHD_OK = 0
SHD_ERR_ARG = -1
SHD_ERR_CUDA = -2
SHD_ERR_NCCL = -3
SHD_ERR_TIMEOUT = -4
SHD_ERR_UNSUPPORTED = -5
SHD_ERR_NUMERIC = -6

NL_APPROX, NL_GPU, NL_MPC = 0, 1, 2
ROWS_PLAIN, ROWS_QKV, ROWS_GATEUP = 0, 1, 2

_ERR_NAMES = {
    SHD_ERR_ARG: "SHD_ERR_ARG",
    SHD_ERR_CUDA: "SHD_ERR_CUDA",
    SHD_ERR_NCCL: "SHD_ERR_NCCL",
    SHD_ERR_TIMEOUT: "SHD_ERR_TIMEOUT",
    SHD_ERR_UNSUPPORTED: "SHD_ERR_UNSUPPORTED",
    SHD_ERR_NUMERIC: "SHD_ERR_NUMERIC",
}

# name -> (restype, argtypes); mirrors include/shardlm_cuda.h
SIGNATURES: dict[str, tuple] = {
    "shd_init": (I32, [I32, PP]),
    "shd_destroy": (I32, [P]),
    "shd_set_stream": (I32, [P, P]),
    "shd_last_error": (C.c_char_p, [P]),
    "shd_sync": (I32, [P]),
    "shd_launch_count": (I64, [P]),
    "shd_wait_selftest": (I32, [P, I32]),
    "shd_weight_upload_f32_as_bf16": (I32, [P, P, I32, I32, PP]),
    "shd_weight_from_bf16": (I32, [P, P, P, I32, I32, I32, I32, PP]),
    "shd_weight_upload_i32": (I32, [P, P, P, I32, I32, PP]),
    "shd_weight_destroy": (I32, [P]),
    "shd_weight_device_bytes": (I64, [P]),
    "shd_linear_dual_f32": (I32, [P, P, P, P, P, P, P, I32, P, P]),
    "shd_linear_dual_ring": (I32, [P, P, P, P, P, P, P, I32, I32]),
    "shd_linear_dual_f32_noalloc": (I32, [P, P, P, P, P, P, I32, P, P, P]),
    "shd_reconstruct_f32": (I32, [P, P, P, P, I64]),
    "shd_reshare_f32": (I32, [P, P, P, P, P, I64]),
    "shd_add_shares": (I32, [P, P, P, P, P, P, P, I64]),
    "shd_beaver_mul_f32": (I32, [P] + [P] * 14 + [I64]),
    "shd_beaver_mul_ring": (I32, [P] + [P] * 14 + [I64, I32]),
    "shd_beaver_triples_f32": (I32, [P, U64, U64, I64] + [P] * 9),
    "shd_beaver_triples_ring": (I32, [P, U64, U64, I64] + [P] * 6),
    "shd_fill_uniform_f32": (I32, [P, U64, U64, F32, F32, P, I64]),
    "shd_rmsnorm_reshare": (I32, [P, P, P, P, F32, I32, P, P, P, I32, I32]),
    "shd_swiglu_reshare": (I32, [P, P, P, P, P, I32, P, P, P, I64]),
    "shd_silu_reshare": (I32, [P, P, P, I32, P, P, P, I64]),
    "shd_rope_init": (I32, [P, I32, I32, F32]),
    "shd_rope_shares": (I32, [P, P, P, I32, I32, I32, I32]),
    "shd_attn_decode": (I32, [P, P, P, P, I32, I32, I32, I32, P, I32, I32, P, P, P]),
    "shd_embed_shares": (I32, [P, P, I32, I32, P, I32, U64, U64, P, P]),
    "shd_attn_prefill": (I32, [P, P, P, P, I32, I32, I32, I32, I32, I32, I32, P, P, P]),
    "shd_model_prefill_hidden": (I32, [P, I32, P, P, I32, P, P, P, P, P]),
    "shd_model_read_kv": (I32, [P, I32, I32, I32, P, P]),
    "shd_model_forward_host_hidden": (I32, [P, I32, P, P, P, P, P, P]),
    "shd_bincode_prefill": (I32, [P, I32, P, C.c_size_t, I32, P, C.c_size_t, P]),
    "shd_bincode_decode": (I32, [P, I32, P, C.c_size_t, P, C.c_size_t, P]),
    "shd_ot_standard_tables": (I32, [P, I32, P]),
    "shd_ot_process_query": (I32, [P, P, U64, P, C.c_size_t, P, C.c_size_t, I32, P, C.c_size_t, P]),
    "shd_embed_shares_session": (I32, [P, P, I32, I32, P, I32, P, P, P]),
    "shd_fixed_from_f64": (I32, [P, P, I64, I32, P]),
    "shd_ring_share_seeded": (I32, [P, P, I64, U64, P, P]),
    "shd_argmax_reconstruct": (I32, [P, P, P, I32, I32, P]),
    "shd_tp_unique_id": (I32, [P]),
    "shd_tp_init": (I32, [P, I32, I32, P]),
    "shd_tp_destroy": (I32, [P]),
    "shd_tp_peer_path": (I32, [P]),
    "shd_allreduce_shares": (I32, [P, P, C.c_size_t, I32]),
    "shd_model_create": (I32, [P, P, PP]),
    "shd_model_destroy": (I32, [P]),
    "shd_model_shard_info": (I32, [P, P]),
    "shd_tp_plan": (I32, [P, P]),
    "shd_model_set_layer": (I32, [P, I32] + [P] * 12),
    "shd_model_set_embedding": (I32, [P, P]),
    "shd_model_set_head": (I32, [P, P, P]),
    "shd_model_set_masks": (I32, [P, P, I64]),
    "shd_model_reset": (I32, [P]),
    "shd_model_prefill": (I32, [P, I32, P, I32, P]),
    "shd_model_decode_async": (I32, [P, I32]),
    "shd_model_read_tokens": (I32, [P, I32, P]),
    "shd_model_forward_host": (I32, [P, I32, P, P, P, P]),
    "shd_model_forward_host_rows": (I32, [P, I32, P, P, P, P, P]),
    "shd_model_seq_len": (I32, [P, I32]),
    "shd_model_step_launches": (I64, [P]),
    "shd_model_set_profiling": (I32, [P, I32]),
    "shd_model_linear_times": (I32, [P, P, P]),
    "shd_model_timeline": (I32, [P, I32, P, P, P]),
}


class ModelConfigC(C.Structure):
    """shd_model_config of include/shardlm_cuda.h."""
    _fields_ = [
        ("hidden", I32), ("n_layers", I32), ("n_heads", I32), ("n_kv_heads", I32),
        ("head_dim", I32), ("intermediate", I32), ("vocab", I32),
        ("rope_theta", F32), ("rms_eps", F32),
        ("max_seq", I32), ("max_batch", I32),
        ("variant_decode", I32), ("variant_prefill", I32), ("variant_attn", I32),
        ("share_seed", U64),
        ("tp_rank", I32), ("tp_world", I32),
    ]


class ShardInfoC(C.Structure):
    """shd_shard_info of include/shardlm_cuda.h."""
    _fields_ = [
        ("q_head_begin", I32), ("q_head_count", I32),
        ("kv_head_begin", I32), ("kv_head_count", I32),
        ("inter_begin", I32), ("inter_count", I32),
        ("vocab_begin", I32), ("vocab_count", I32),
    ]

_lib = None
_lock = threading.Lock()


class ShdError(RuntimeError):
    def __init__(self, code: int, message: str):
        self.code = code
        super().__init__(f"{_ERR_NAMES.get(code, code)}: {message}")


def lib() -> C.CDLL:
    """Load libshardlm_cuda.so, building it first when missing or stale."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if _build.library_stale() and os.environ.get("SHD_NO_BUILD") != "1":
            _build.build_library()
        if not _build.LIB.exists():
            raise RuntimeError(f"libshardlm_cuda.so missing at {_build.LIB}")
        handle = C.CDLL(str(_build.LIB), mode=C.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, ctx_ptr=None) -> None:
    if rc != SHD_OK:
        msg = ""
        if ctx_ptr:
            raw = lib().shd_last_error(ctx_ptr)
            msg = raw.decode() if raw else ""
        raise ShdError(rc, msg)
