"""ctypes binding of the C ABI in ``include/eesd.h`` (``thesis_b200/_lib/libeesd.so``).

There is no fallback: if the extension is missing or a call fails, the error is raised.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libeesd.so"

OK, ERR_ARG, ERR_CUDA, ERR_DEVICE = 0, 1, 2, 3
BF16, F32 = 0, 1
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2
OPT_MMA_N, OPT_SPLITS, OPT_STAGES, OPT_PAIR, OPT_HEAD_TWO_TILES, OPT_SPIN_LIMIT, OPT_MMA_SPLIT = 1, 2, 3, 4, 5, 6, 7
PROF_KINDS = 9
PROF_NAMES = ["norm", "gemm_qkv", "rope_kv", "attn", "gemm_o", "gemm_w13", "gemm_w2", "head", "misc"]

vp, i32, i64, f32, sz = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t
i32p = C.POINTER(C.c_int32)


class ModelDesc(C.Structure):
    _fields_ = [
        ("dtype", i32), ("n_layers", i32), ("dim", i32), ("n_heads", i32), ("n_kv_heads", i32), ("head_dim", i32),
        ("intermediate", i32), ("vocab", i32), ("norm_eps", f32), ("max_batch", i32), ("max_seq", i32),
        ("max_tokens", i32), ("weights_packed", i32), ("wqkv", C.POINTER(vp)), ("wo", C.POINTER(vp)), ("w13", C.POINTER(vp)),
        ("w2", C.POINTER(vp)), ("attn_norm", C.POINTER(vp)), ("ffn_norm", C.POINTER(vp)), ("final_norm", vp),
        ("lm_head", vp), ("embed", vp), ("rope_cos", vp), ("rope_sin", vp), ("k_cache", vp), ("v_cache", vp),
        ("workspace", vp), ("workspace_bytes", sz),
    ]


class Batch(C.Structure):
    _fields_ = [("n_tokens", i32), ("n_blocks", i32), ("n_items", i32), ("max_ctx", i32), ("tok_pos", vp),
                ("tok_row", vp), ("blk", vp), ("items", vp)]


# name -> (restype, argtypes); every symbol declared in include/eesd.h
SIGNATURES = {
    "eesd_version": (C.c_int, []),
    "eesd_last_error": (C.c_char_p, []),
    "eesd_attn_item_tokens": (C.c_int, [C.c_int, C.c_int]),
    "eesd_packed_weight_bytes": (sz, [C.c_int, C.c_int]),
    "eesd_pack_weight": (C.c_int, [vp, C.c_int, C.c_int, vp, vp]),
    "eesd_model_workspace_bytes": (sz, [C.POINTER(ModelDesc)]),
    "eesd_model_create": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(vp)]),
    "eesd_model_destroy": (C.c_int, [vp]),
    "eesd_forward_layers": (C.c_int, [vp, vp, C.POINTER(Batch), C.c_int, C.c_int, vp]),
    "eesd_head_argmax": (C.c_int, [vp, vp, vp, C.c_int, vp, vp, vp]),
    "eesd_embed": (C.c_int, [vp, vp, C.c_int, vp, vp]),
    "eesd_model_check": (C.c_int, [vp, C.POINTER(C.c_int), vp]),
    "eesd_model_profile": (C.c_int, [vp, C.c_int]),
    "eesd_model_profile_read": (C.c_int, [vp, C.POINTER(C.c_double), C.POINTER(i64)]),
    "eesd_model_profile_records": (C.c_int, [vp, vp, vp, vp, C.c_int]),
    "eesd_model_launch_count": (i64, [vp]),
    "eesd_copy_rows": (C.c_int, [C.c_int, vp, vp, vp, vp, C.c_int, C.c_int, vp]),
    "eesd_gather_ids": (C.c_int, [vp, vp, vp, C.c_int, vp]),
    "eesd_scatter_ids": (C.c_int, [vp, vp, vp, C.c_int, vp]),
    "eesd_greedy_accept": (C.c_int, [vp, vp, C.c_int, vp, C.c_int, vp, vp]),
    "eesd_round_meta_ints": (sz, [C.c_int, C.c_int, C.c_int]),
    "eesd_round_meta": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, vp, vp]),
    "eesd_round_advance": (C.c_int, [vp, C.c_int, vp, vp, C.c_int, vp]),
    "eesd_rmsnorm": (C.c_int, [C.c_int, vp, vp, vp, vp, C.c_int, C.c_int, C.c_float, vp]),
    "eesd_gemm_workspace_bytes": (sz, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "eesd_gemm": (C.c_int, [C.c_int, C.c_int, vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, sz, vp]),
    "eesd_set_option": (C.c_int, [C.c_int, C.c_int]),
    "eesd_status_read": (C.c_int, [vp, C.POINTER(C.c_int), vp]),
    "eesd_head_argmax_static": (C.c_int, [vp, C.c_int, vp, C.c_int, C.c_int, C.c_int, vp, vp, C.c_float, vp, vp, vp]),
    "eesd_attn_varlen_gqa": (C.c_int, [C.c_int, vp, C.c_int, C.c_int, C.c_int, vp, vp, C.c_int, C.c_int,
                                       C.POINTER(Batch), C.c_int, vp, vp, vp, vp, vp]),
    "eesd_rope_kv_append": (C.c_int, [C.c_int, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_int, vp, vp, vp, vp,
                                      C.c_int, C.c_int, vp, vp]),
}

_lib = None


class EesdError(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load the extension once.  Raises when it is missing: there is no other backend."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise EesdError(f"{LIB_PATH} is missing: build it with `python -m thesis_b200.build`")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str = "") -> None:
    if rc != OK:
        msg = load().eesd_last_error().decode(errors="replace")
        raise EesdError(f"{what or 'eesd call'} failed with status {rc}: {msg}")


# entry points that launch exactly one kernel (counted for the bench's launch total)
KERNEL_CALLS = {"eesd_pack_weight", "eesd_copy_rows", "eesd_gather_ids", "eesd_scatter_ids", "eesd_greedy_accept",
                "eesd_round_meta", "eesd_round_advance", "eesd_rmsnorm",
                "eesd_gemm", "eesd_attn_varlen_gqa", "eesd_rope_kv_append"}
direct_launches = 0


def call(name: str, *args):
    global direct_launches
    rc = getattr(load(), name)(*args)
    check(rc, name)
    if name in KERNEL_CALLS:
        direct_launches += 1
    return rc


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor, None for None."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
