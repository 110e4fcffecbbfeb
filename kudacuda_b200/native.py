"""ctypes signatures of the C ABI declared in include/kudacuda.h and
include/kudacuda_registry.h, and the loader for the in-tree library.

The library is the product: there is no Python or CPU implementation of any
op behind these symbols.  ``load_library`` fails loudly when the built
``lib/libkudacuda.so`` is missing.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Any

PACKAGE_DIR = Path(__file__).resolve().parent
DEFAULT_LIBRARY = PACKAGE_DIR / "lib" / "libkudacuda.so"

_p = ctypes.c_void_p
_u64 = ctypes.c_uint64
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); the reference-ABI part matches the argtypes of
# the reference bridge (python/kudacuda_sidecar.py:259-419).
SIGNATURES: dict[str, tuple[Any, list[Any]]] = {
    "kudacuda_create": (_p, [_i32]),
    "kudacuda_freeze": (_i32, [_p]),
    "kudacuda_can_dispatch": (_i32, [_p, ctypes.c_char_p, _i64, _i64]),
    "kudacuda_vector_add": (_i32, [_p, _u64, _u64, _u64, _i64, _u64]),
    "kudacuda_rmsnorm": (_i32, [_p, _u64, _u64, _u64, _i64, _i64, _f32, _u64]),
    "kudacuda_fused_rmsnorm_qkv": (_i32, [_p, _u64, _u64, _u64, _u64, _u64, _i64, _i64, _f32, _u64]),
    "kudacuda_qwen2_fused_rmsnorm_qkv_nf4": (_i32, [_p] + [_u64] * 14 + [_i64] * 5 + [_f32, _u64]),
    "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2": (_i32, [_p] + [_u64] * 15 + [_i64] * 5 + [_f32, _u64]),
    "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3": (_i32, [_p] + [_u64] * 15 + [_i64] * 5 + [_f32, _u64]),
    "kudacuda_qwen2_swiglu_nf4": (_i32, [_p] + [_u64] * 7 + [_i64] * 4 + [_f32, _u64]),
    "kudacuda_qwen2_swiglu_nf4_bf16": (_i32, [_p] + [_u64] * 7 + [_i64] * 4 + [_f32, _u64]),
    "kudacuda_qwen2_gqa_decode_workspace_v3": (_i32, [_p] + [_u64] * 6 + [_i64] * 6 + [_f32, _u64]),
    "kudacuda_qwen2_gqa_decode": (_i32, [_p] + [_u64] * 4 + [_i64] * 6 + [_f32, _u64]),
    "kudacuda_qwen2_gqa_decode_graph": (_i32, [_p] + [_u64] * 4 + [_i64] * 6 + [_f32, _u64, _u64]),
    "kudacuda_qwen2_gqa_decode_group_tiled": (_i32, [_p] + [_u64] * 4 + [_i64] * 6 + [_f32, _u64]),
    "kudacuda_qwen2_gqa_decode_vectorized": (_i32, [_p] + [_u64] * 4 + [_i64] * 6 + [_f32, _u64]),
    "kudacuda_begin_capture": (_i32, [_p, _u64]),
    "kudacuda_end_capture": (_i32, [_p, _u64]),
    "kudacuda_replay_graph": (_i32, [_p, _u64]),
    "kudacuda_reset_graph": (_i32, [_p]),
    "kudacuda_last_error": (ctypes.c_char_p, [_p]),
    "kudacuda_destroy": (None, [_p]),
    # sm100 additions
    "kudacuda_sm100_nf4_gemv": (_i32, [_p, _u64, _i32, _u64, _u64, _u64, _u64, _i32, _i64, _i64, _i64, _u64]),
    "kudacuda_sm100_nf4_linear_residual_bf16": (_i32, [_p, _u64, _u64, _u64, _u64, _i64, _i64, _i64, _u64]),
    "kudacuda_sm100_nf4_dequantize": (_i32, [_p, _u64, _u64, _u64, _i32, _i64, _i64, _u64]),
    "kudacuda_sm100_nf4_quantize": (_i32, [_p, _u64, _i32, _u64, _u64, _i64, _i64, _u64]),
    "kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16": (_i32, [_p] + [_u64] * 17 + [_i64] * 7 + [_f32, _u64]),
    "kudacuda_sm100_swiglu_nf4_bf16": (_i32, [_p] + [_u64] * 7 + [_i64] * 3 + [_f32, _u64]),
    "kudacuda_sm100_gqa_decode": (
        _i32,
        [_p, _u64, _u64, _u64, _u64, _u64, _i64, _u64, _u64, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _u64],
    ),
    "kudacuda_sm100_gqa_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "kudacuda_sm100_rmsnorm_nf4_gemv": (_i32, [_p, _u64, _u64, _u64, _u64, _u64, _i32, _i64, _i64, _f32, _u64]),
    "kudacuda_sm100_residual_add_f32": (_i32, [_p, _u64, _u64, _i64, _u64]),
    "kudacuda_sm100_argmax_workspace_bytes": (_i64, []),
    "kudacuda_sm100_argmax_shard_f32": (_i32, [_p, _u64, _i64, _i64, _u64, _i64, _u64, _u64, _u64]),
    "kudacuda_sm100_select_token": (_i32, [_p, _u64, _i64, _u64, _u64]),
    "kudacuda_sm100_nf4_retile_groups": (_i64, [_i32, _i64, _i64, _i64, _i64]),
    "kudacuda_sm100_nf4_retile": (
        _i32, [_p, _i32, _u64, _u64, _i64, _u64, _u64, _i64, _u64, _u64, _i64, _i64, _i64, _u64, _u64, _u64]
    ),
    "kudacuda_sm100_decode_persistent_scratch_bytes": (_i64, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "kudacuda_sm100_decode_layers_persistent": (
        _i32,
        [_p, _u64, _i64, _u64, _u64, _u64, _u64, _i64, _u64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32,
         _u64],
    ),
    "kudacuda_sm100_decode_persistent_tap_elements": (_i64, [_i64] * 6),
    "kudacuda_sm100_decode_layers_persistent_debug": (
        _i32,
        [_p, _u64, _i64, _u64, _u64, _u64, _u64, _i64, _u64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32,
         _u64, _i64, _i64, _i64, _u64],
    ),
    "kudacuda_sm100_nf4_retile16_tiles": (_i64, [_i32, _i64, _i64, _i64, _i64]),
    "kudacuda_sm100_nf4_retile16": (
        _i32, [_p, _i32, _u64, _u64, _i64, _u64, _u64, _i64, _u64, _u64, _i64, _i64, _i64, _u64, _i64, _u64]
    ),
    "kudacuda_sm100_decode_rows_scratch_bytes": (_i64, [_p, _i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "kudacuda_sm100_decode_layers_rows": (
        _i32,
        [_p, _u64, _i64, _u64, _u64, _u64, _u64, _i64, _u64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32,
         _u64, _i64, _i64, _i64, _u64],
    ),
    "kudacuda_sm100_decode_layers_rows_tp": (
        _i32,
        [_p, _u64, _i64, _u64, _u64, _u64, _u64, _i64, _u64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32,
         _i64, _i64, _u64, _u64],
    ),
    "kudacuda_sm100_tp_exchange_bytes": (_i64, [_i64, _i64]),
    "kudacuda_sm100_ipc_alloc": (_i32, [_p, _i64, ctypes.POINTER(_u64), _p, _i64]),
    "kudacuda_sm100_ipc_open": (_i32, [_p, _p, _i64, ctypes.POINTER(_u64)]),
    "kudacuda_sm100_ipc_close": (_i32, [_p, _u64, _i32]),
    "kudacuda_sm100_batch_gemm_ksplit": (_i64, [_i64, _i64]),
    "kudacuda_sm100_batch_gemm": (_i32, [_p, _i32, _u64, _u64, _i64, _i64, _u64, _i64, _i64, _u64, _i64, _i64, _u64]),
    "kudacuda_sm100_batch_retile_bytes": (_i64, [_i64, _i64]),
    "kudacuda_sm100_batch_retile": (_i32, [_p, _u64, _u64, _i64, _i64, _u64, _i64, _u64]),
    "kudacuda_sm100_batch_gemm_residual": (
        _i32, [_p, _i32, _u64, _u64, _i64, _i64, _u64, _i64, _i64, _i64, _u64, _i64, _u64, _u64, _u64]
    ),
    "kudacuda_sm100_batch_gemm_swiglu": (
        _i32, [_p, _i32, _u64, _u64, _i64, _i64, _u64, _i64, _i64, _i64, _u64, _i64, _u64, _u64, _u64]
    ),
    "kudacuda_sm100_batch_gemm_qkv_rope": (
        _i32,
        [_p, _i32, _u64, _u64, _i64, _u64, _i64, _i64, _i64, _u64, _i64, _u64, _i64, _i64, _i64] + [_u64] * 5
        + [_i64, _u64, _u64, _u64, _u64, _i64, _i32, _u64],
    ),
    "kudacuda_sm100_batch_rmsnorm": (_i32, [_p, _u64, _u64, _u64, _i64, _i64, _f32, _u64]),
    "kudacuda_sm100_batch_qkv_rope": (
        _i32, [_p, _u64, _i64, _i64, _i64, _i64, _i64, _i64] + [_u64] * 5 + [_i64] + [_u64] * 4 + [_i64, _i32, _u64]
    ),
    "kudacuda_sm100_batch_residual": (_i32, [_p, _u64, _i64, _i64, _i64, _i64, _u64, _u64]),
    "kudacuda_sm100_batch_swiglu": (_i32, [_p, _u64, _i64, _i64, _i64, _i64, _u64, _u64]),
    "kudacuda_sm100_batch_argmax_workspace_bytes": (_i64, [_i64]),
    "kudacuda_sm100_batch_argmax_advance": (
        _i32, [_p, _u64, _i64, _i64, _i64, _i64, _u64, _i64, _u64, _u64, _i64, _u64]
    ),
    "kudacuda_sm100_batch_embedding": (_i32, [_p, _u64, _u64, _u64, _i64, _i64, _i64, _u64]),
    "kudacuda_sm100_batch_state_views": (_i32, [_p, _u64, _i64, _u64, _u64, _u64]),
    "kudacuda_sm100_batch_split_sum": (_i32, [_p, _u64, _i64, _i64, _i64, _u64, _u64]),
    "kudacuda_sm100_batch_argmax_pairs": (_i32, [_p, _u64, _i64, _i64, _i64, _i64, _u64, _i64, _i64, _u64, _u64]),
    "kudacuda_sm100_batch_select_advance": (_i32, [_p, _u64, _i64, _i64, _u64, _u64, _i64, _u64]),
    "kudacuda_sm100_gqa_batch_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "kudacuda_sm100_gqa_decode_batch": (
        _i32, [_p, _u64, _u64, _u64, _u64, _u64, _i64, _u64, _u64, _i64, _i64, _i64, _i64, _i64, _f32, _i32, _u64]
    ),
    "kudacuda_sm100_gqa_decode_static": (
        _i32, [_p, _u64, _u64, _u64, _u64, _u64, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _u64]
    ),
    "kudacuda_sm100_lm_head_argmax_bf16": (
        _i32,
        [_p, _u64, _u64, _u64, _u64, _u64, _u64, _i64, _u64, _i64, _i64, _f32, _u64],
    ),
    "kudacuda_sm100_lm_head_workspace_bytes": (_i64, []),
    "kudacuda_sm100_embedding_bf16": (_i32, [_p, _u64, _u64, _u64, _i64, _i64, _u64]),
    "kudacuda_sm100_decode_advance": (_i32, [_p, _u64, _u64, _u64, _i64, _u64]),
    "kudacuda_sm100_graph_step_host": (_i32, [_p, _p, _u64, _i64, _p, _u64, _i64, _u64]),
    "kudacuda_sm100_error_word": (_i32, [_p, ctypes.POINTER(ctypes.c_int), _i32]),
    "kudacuda_sm100_target_arch": (ctypes.c_char_p, []),
    # include/kudacuda_registry.h
    "kudacuda_tactic_count": (_i32, []),
    "kudacuda_tactic_info": (
        _i32,
        [_i32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i64), ctypes.POINTER(_i64)],
    ),
}

DTYPE_CODES = {"float32": 0, "float16": 1, "bfloat16": 2}


def configure(lib: Any) -> Any:
    """Attach restype/argtypes for every known symbol the library exports."""

    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = restype
        fn.argtypes = argtypes
    return lib


def load_library(path: str | Path | None = None) -> ctypes.CDLL:
    lib_path = Path(path) if path is not None else DEFAULT_LIBRARY
    if not lib_path.exists():
        raise FileNotFoundError(
            f"KudaCuda sm_100a library not found at {lib_path}; build it with `python -m kudacuda_b200.build`"
        )
    return configure(ctypes.CDLL(str(lib_path)))


def tactic_table(lib: Any) -> list[dict[str, Any]]:
    """Read the built-in tactic table through kudacuda_tactic_info."""

    rows = []
    for i in range(int(lib.kudacuda_tactic_count())):
        name = ctypes.c_char_p()
        symbol = ctypes.c_char_p()
        max_batch = ctypes.c_int64()
        seq_len = ctypes.c_int64()
        if lib.kudacuda_tactic_info(i, ctypes.byref(name), ctypes.byref(symbol), ctypes.byref(max_batch), ctypes.byref(seq_len)):
            break
        rows.append(
            {
                "name": name.value.decode(),
                "symbol": symbol.value.decode(),
                "max_batch": int(max_batch.value),
                "seq_len": int(seq_len.value),
            }
        )
    return rows
