"""ctypes binding of ``libpkv.so``, the C ABI declared in ``include/pkv.h``.

The library is built in-tree (``python mini_inference_b200/build.py``). There is
no fallback: if it is missing or fails to load, importing this module raises,
and every op of the package is unusable.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libpkv.so"

PKV_OK = 0
PKV_ERR_INVALID_ARGUMENT = 1
PKV_ERR_OUT_OF_RANGE = 2
PKV_ERR_WORKSPACE = 3
PKV_ERR_CUDA = 4
PKV_ERR_NO_BLOCKS = 5
PKV_ERR_DOUBLE_FREE = 6
PKV_ERR_UNKNOWN_SLOT = 7
PKV_ERR_UNSUPPORTED = 8
PKV_ERR_TIMEOUT = 9
PKV_ERR_EMPTY_PROMPT = 10
PKV_ERR_PROMPT_TOO_LONG = 11

PKV_SEQ_WAITING, PKV_SEQ_RUNNING, PKV_SEQ_FINISHED = 0, 1, 2

PKV_F16 = 0
PKV_BF16 = 1

PKV_DECODE_INPUTS_READY = 1
PKV_LM_WEIGHT_READY = 1
PKV_DECODE_STATIC_SCRATCH_BYTES = 16 * 1024 * 1024


class PkvPool(ctypes.Structure):
    _fields_ = [("k", c_void_p), ("v", c_void_p), ("num_layers", c_int32), ("num_blocks_total", c_int32),
                ("num_kv_heads", c_int32), ("block_size", c_int32), ("head_dim", c_int32), ("dtype", c_int32)]


class PkvTables(ctypes.Structure):
    _fields_ = [("block_tables", c_void_p), ("stride", c_int64), ("rows", c_int32), ("cols", c_int32),
                ("seq_rows", c_void_p)]


class PkvSchedStep(ctypes.Structure):
    _fields_ = [("capacity", c_int32), ("prefill_ids", c_void_p), ("prefill_slots", c_void_p),
                ("prefill_cached_tokens", c_void_p), ("decode_ids", c_void_p), ("decode_slots", c_void_p),
                ("preempted_ids", c_void_p), ("n_prefills", c_int32), ("n_decodes", c_int32),
                ("n_preempted", c_int32), ("prefill_new_tokens", c_void_p), ("decode_last_tokens", c_void_p)]


P_POOL = POINTER(PkvPool)
P_TABLES = POINTER(PkvTables)
P_I32 = POINTER(c_int32)
P_I64 = POINTER(c_int64)

# name -> (restype, argtypes); must match include/pkv.h
SIGNATURES: dict[str, tuple] = {
    "pkv_status_string": (c_char_p, [c_int32]),
    "pkv_last_cuda_error": (c_char_p, []),
    "pkv_version": (c_int32, []),
    "pkv_kv_append": (c_int32, [P_POOL, c_int32, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                                c_void_p]),
    "pkv_rope_append": (c_int32, [P_POOL, c_int32, c_void_p, c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p,
                                  c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p,
                                  c_void_p]),
    "pkv_lm_head_argmax_workspace_bytes": (c_int64, [c_int32]),
    "pkv_lm_head_argmax": (c_int32, [c_void_p, c_int64, c_int32, c_void_p, c_int64, c_int32, c_int32, c_int32,
                                     c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_void_p, c_void_p]),
    "pkv_add_rms_norm": (c_int32, [c_int32, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                                   c_void_p, c_int64, c_int64, c_int32, c_float, c_void_p]),
    "pkv_add_rms_norm_partials": (c_int32, [c_int32, c_void_p, c_int64, c_int32, c_int64, c_void_p, c_int64,
                                            c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_float,
                                            c_void_p]),
    "pkv_silu_mul": (c_int32, [c_int32, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_int32, c_void_p]),
    "pkv_decode_attention": (c_int32, [P_POOL, c_int32, P_TABLES, c_int32, c_int32, c_void_p, c_int64, c_int64,
                                       c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                       c_void_p, c_float, c_int32, c_void_p, c_int64, c_void_p, c_void_p]),
    "pkv_decode_attention_rope": (c_int32, [P_POOL, c_int32, P_TABLES, c_int32, c_int32, c_void_p, c_int64, c_int64,
                                            c_void_p, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_float,
                                            c_int32, c_void_p, c_int64, c_void_p, c_void_p]),
    "pkv_decode_workspace_bytes": (c_int64, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32]),
    "pkv_decode_reset_workspace": (c_int32, [c_void_p, c_int64, c_void_p]),
    "pkv_decode_static_reset": (c_int32, [c_void_p]),
    "pkv_decode_static_scratch": (c_int32, [POINTER(c_void_p), P_I64, c_void_p]),
    "pkv_decode_attention_static": (c_int32, [P_POOL, c_int32, P_TABLES, c_int32, c_int32, c_void_p, c_int64,
                                              c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                              c_int64, c_void_p, c_void_p, c_float, c_int32, c_void_p, c_void_p]),
    "pkv_prefill_attention": (c_int32, [P_POOL, c_int32, P_TABLES, c_int32, c_void_p, c_void_p, c_int32, c_int32,
                                        c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_float, c_void_p,
                                        c_void_p]),
    "pkv_build_decode_metadata": (c_int32, [P_TABLES, c_int32, c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                                            c_void_p, c_void_p, c_void_p]),
    "pkv_build_prefill_metadata": (c_int32, [P_TABLES, c_int32, c_void_p, c_void_p, c_int32, c_int64, c_void_p,
                                             c_void_p, c_void_p, c_void_p]),
    "pkv_commit_decode": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p]),
    "pkv_update_tables": (c_int32, [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_void_p]),
    "pkv_copy_blocks": (c_int32, [P_POOL, c_void_p, c_void_p, c_int32, c_void_p, c_void_p]),
    "pkv_sched_create": (c_int32, [c_void_p, c_int32, c_int64, c_int64, c_int32, c_void_p, c_int32,
                                   POINTER(c_void_p)]),
    "pkv_sched_destroy": (None, [c_void_p]),
    "pkv_sched_add": (c_int32, [c_void_p, c_int64, c_void_p, c_int64, c_int32, c_int32]),
    "pkv_sched_schedule": (c_int32, [c_void_p, POINTER(PkvSchedStep)]),
    "pkv_sched_set_chunked_prefill": (c_int32, [c_void_p, c_int32]),
    "pkv_sched_append_tokens": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32, c_void_p]),
    "pkv_sched_abort": (c_int32, [c_void_p, c_int64, P_I32]),
    "pkv_sched_counts": (c_int32, [c_void_p, P_I32, P_I32, P_I64]),
    "pkv_sched_queues": (c_int32, [c_void_p, c_void_p, c_void_p, c_int32]),
    "pkv_bm_create": (c_int32, [c_int32, c_int32, c_int32, c_int32, c_int32, POINTER(c_void_p)]),
    "pkv_bm_destroy": (None, [c_void_p]),
    "pkv_bm_can_allocate": (c_int32, [c_void_p, c_int64, P_I32]),
    "pkv_bm_allocate": (c_int32, [c_void_p, c_int64, c_void_p, c_int64, P_I32]),
    "pkv_bm_register_prefix": (c_int32, [c_void_p, c_int32, c_void_p, c_int64]),
    "pkv_bm_ensure_capacity": (c_int32, [c_void_p, c_int32, c_int64, P_I32]),
    "pkv_bm_free": (c_int32, [c_void_p, c_int32]),
    "pkv_bm_fork": (c_int32, [c_void_p, c_int32, P_I32]),
    "pkv_bm_prepare_write": (c_int32, [c_void_p, c_int32, c_int64, c_int64, c_void_p, c_int32, P_I32]),
    "pkv_bm_decode_positions": (c_int32, [c_void_p, c_void_p, c_int32, c_void_p]),
    "pkv_bm_commit_decode": (c_int32, [c_void_p, c_void_p, c_int32]),
    "pkv_bm_get_length": (c_int32, [c_void_p, c_int32, P_I64]),
    "pkv_bm_set_length": (c_int32, [c_void_p, c_int32, c_int64]),
    "pkv_bm_get_table": (c_int32, [c_void_p, c_int32, c_void_p, c_int32, P_I32]),
    "pkv_bm_live_slots": (c_int32, [c_void_p, c_void_p, c_int32, P_I32]),
    "pkv_bm_num_free_blocks": (c_int32, [c_void_p, P_I32]),
    "pkv_bm_num_free_slots": (c_int32, [c_void_p, P_I32]),
    "pkv_bm_prefix_hit_tokens": (c_int32, [c_void_p, P_I64]),
    "pkv_bm_free_order": (c_int32, [c_void_p, c_void_p, c_int32, P_I32]),
    "pkv_bm_ref_counts": (c_int32, [c_void_p, c_void_p, c_int32]),
    "pkv_bm_cached_blocks": (c_int32, [c_void_p, c_void_p, c_int32, P_I32]),
    "pkv_bm_set_journal": (c_int32, [c_void_p, c_int32]),
    "pkv_bm_drain_table_edits": (c_int32, [c_void_p, c_void_p, c_int32, P_I32, P_I32]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH.name} is not built; run `python mini_inference_b200/build.py` "
                          "(the paged-KV path has no fallback without it)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class PkvError(RuntimeError):
    """A status other than PKV_OK from libpkv, with the library's own message."""

    def __init__(self, status: int, what: str) -> None:
        msg = lib.pkv_status_string(status).decode()
        if status == PKV_ERR_CUDA:
            msg += ": " + lib.pkv_last_cuda_error().decode()
        super().__init__(f"{what}: {msg} (status {status})")
        self.status = status


def check(status: int, what: str) -> None:
    if status != PKV_OK:
        raise PkvError(status, what)


def status_name(status: int) -> str:
    return lib.pkv_status_string(status).decode()
