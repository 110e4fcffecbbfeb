"""Python access to the CPU oracle (oracle/kc_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, as the checker.  The
product path (kudacuda_b200) never imports this module.

Each wrapper names the reference file:line its C function restates.  Arrays
are numpy; bf16 and f16 tensors travel as uint16 bit patterns.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "build" / "libkc_oracle.so"

F32, F16, BF16 = 0, 1, 2

_lib = None


def build() -> Path:
    src = ORACLE_DIR / "kc_oracle.c"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.kc_f32_to_bf16.restype = ctypes.c_uint16
        _lib.kc_f32_to_bf16.argtypes = [ctypes.c_float]
        _lib.kc_f32_to_f16.restype = ctypes.c_uint16
        _lib.kc_f32_to_f16.argtypes = [ctypes.c_float]
        _lib.kc_bf16_to_f32.restype = ctypes.c_float
        _lib.kc_bf16_to_f32.argtypes = [ctypes.c_uint16]
        _lib.kc_f16_to_f32.restype = ctypes.c_float
        _lib.kc_f16_to_f32.argtypes = [ctypes.c_uint16]
        _lib.kc_nf4_codebook.restype = ctypes.c_float
        _lib.kc_nf4_codebook.argtypes = [ctypes.c_int]
        _lib.kc_nf4_quantize_value.restype = ctypes.c_int
        _lib.kc_nf4_quantize_value.argtypes = [ctypes.c_float]
        _lib.kc_lm_head_argmax.restype = ctypes.c_int64
        _lib.kc_num_threads.restype = ctypes.c_int
    return _lib


def _ptr(a: np.ndarray | None) -> ctypes.c_void_p:
    if a is None:
        return ctypes.c_void_p(0)
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def set_threads(n: int) -> None:
    lib().kc_set_num_threads(ctypes.c_int(int(n)))


def num_threads() -> int:
    return int(lib().kc_num_threads())


# ---------------------------------------------------------------- formats
def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""

    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f16_bits(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_to_f32(b: np.ndarray) -> np.ndarray:
    return np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32)


# ---------------------------------------------------------------- NF4
def codebook() -> np.ndarray:
    """kernels/common/nf4_device.cuh:10-27."""

    return np.array([lib().kc_nf4_codebook(i) for i in range(16)], dtype=np.float32)


def midpoints() -> np.ndarray:
    out = np.zeros(15, dtype=np.float32)
    lib().kc_nf4_midpoints(_ptr(out))
    return out


def nf4_quantize(w: np.ndarray, blocksize: int = 64) -> tuple[np.ndarray, np.ndarray]:
    """bitsandbytes 0.50.1 blockwise NF4 (restated; parity unpinned)."""

    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    n = w.size
    packed = np.zeros((n + 1) // 2, dtype=np.uint8)
    absmax = np.zeros((n + blocksize - 1) // blocksize, dtype=np.float32)
    lib().kc_nf4_quantize(_ptr(w), ctypes.c_int64(n), ctypes.c_int64(blocksize), _ptr(packed), _ptr(absmax))
    return packed, absmax


def nf4_dequant(packed: np.ndarray, absmax: np.ndarray, n: int, blocksize: int = 64) -> np.ndarray:
    """kernels/common/nf4_device.cuh:29-40 (bit-exact)."""

    out = np.zeros(n, dtype=np.float32)
    lib().kc_nf4_dequant(
        _ptr(np.ascontiguousarray(packed, dtype=np.uint8)),
        _ptr(np.ascontiguousarray(absmax, dtype=np.float32)),
        ctypes.c_int64(n),
        ctypes.c_int64(blocksize),
        _ptr(out),
    )
    return out


def nf4_gemv(x: np.ndarray, packed: np.ndarray, absmax: np.ndarray, rows: int, k: int, blocksize: int = 64) -> np.ndarray:
    """fp32 y = x . W^T in index order (tests/nf4_tiled_gemv_smoke.cu:86-94)."""

    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(rows, dtype=np.float32)
    lib().kc_nf4_gemv_f32(
        _ptr(x), _ptr(packed), _ptr(absmax), ctypes.c_int64(rows), ctypes.c_int64(k), ctypes.c_int64(blocksize), _ptr(y)
    )
    return y


# ---------------------------------------------------------------- norms
def rmsnorm_ref(x: np.ndarray, w: np.ndarray, dtype: int, eps: float) -> np.ndarray:
    """kernels/common/nf4_tiled_gemv.cuh:61-100 (fp32 normalised)."""

    out = np.zeros(x.size, dtype=np.float32)
    lib().kc_rmsnorm_ref(_ptr(x), _ptr(w), ctypes.c_int(dtype), ctypes.c_int64(x.size), ctypes.c_float(eps), _ptr(out))
    return out


def rmsnorm_f64(rows: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """harness/reference.py:9-31."""

    rows = np.ascontiguousarray(rows, dtype=np.float64)
    w = np.ascontiguousarray(w, dtype=np.float64)
    out = np.zeros_like(rows)
    lib().kc_rmsnorm_f64(
        _ptr(rows), _ptr(w), ctypes.c_int64(rows.shape[0]), ctypes.c_int64(rows.shape[1]), ctypes.c_double(eps), _ptr(out)
    )
    return out


def rmsnorm_hf_bf16(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    out = np.zeros(x.size, dtype=np.uint16)
    lib().kc_rmsnorm_hf_bf16(_ptr(x), _ptr(w), ctypes.c_int64(x.size), ctypes.c_float(eps), _ptr(out))
    return out


# ---------------------------------------------------------------- fused reference ops
def qkv_nf4_ref(x, norm_w, dtype, eps, q, k, v, blocksize=64):
    """tests/nf4_tiled_gemv_smoke.cu:77-103.  q/k/v = (packed, absmax, bias, rows)."""

    hidden = x.size
    qo = np.zeros(q[3], dtype=np.uint16)
    ko = np.zeros(k[3], dtype=np.uint16)
    vo = np.zeros(v[3], dtype=np.uint16)
    norm = np.zeros(hidden, dtype=np.float32)
    lib().kc_qkv_nf4_ref(
        _ptr(x), _ptr(norm_w), ctypes.c_int(dtype), ctypes.c_int64(hidden), ctypes.c_float(eps),
        _ptr(q[0]), _ptr(q[1]), _ptr(q[2]), ctypes.c_int64(q[3]),
        _ptr(k[0]), _ptr(k[1]), _ptr(k[2]),
        _ptr(v[0]), _ptr(v[1]), _ptr(v[2]), ctypes.c_int64(k[3]),
        ctypes.c_int64(blocksize), _ptr(qo), _ptr(ko), _ptr(vo), _ptr(norm),
    )
    return qo, ko, vo, norm


def swiglu_nf4_ref(x, norm_w, dtype, eps, gate, up, inter, blocksize=64):
    """tests/nf4_swiglu_bf16_smoke.cu:61-84.  gate/up = (packed, absmax)."""

    out = np.zeros(inter, dtype=np.uint16)
    lib().kc_swiglu_nf4_ref(
        _ptr(x), _ptr(norm_w), ctypes.c_int(dtype), ctypes.c_int64(x.size), ctypes.c_float(eps),
        _ptr(gate[0]), _ptr(gate[1]), _ptr(up[0]), _ptr(up[1]), ctypes.c_int64(inter), ctypes.c_int64(blocksize), _ptr(out),
    )
    return out


def gqa_decode(q, kcache, vcache, dtype, q_heads, kv_heads, head_dim, kv_len, kv_stride, scale):
    """tests/qwen2_gqa_smoke.cu:65-93; q/k/v as uint16 bit patterns (f16/bf16) or f32."""

    out = np.zeros(q_heads * head_dim, dtype=np.float32 if dtype == F32 else np.uint16)
    lib().kc_gqa_decode(
        _ptr(q), _ptr(kcache), _ptr(vcache), ctypes.c_int(dtype), ctypes.c_int64(q_heads), ctypes.c_int64(kv_heads),
        ctypes.c_int64(head_dim), ctypes.c_int64(kv_len), ctypes.c_int64(kv_stride), ctypes.c_float(scale), _ptr(out),
    )
    return out


def rope_hf_bf16(x: np.ndarray, heads: int, head_dim: int, cos_row: np.ndarray, sin_row: np.ndarray) -> np.ndarray:
    out = np.ascontiguousarray(x, dtype=np.uint16).copy()
    lib().kc_rope_hf_bf16(_ptr(out), ctypes.c_int64(heads), ctypes.c_int64(head_dim), _ptr(cos_row), _ptr(sin_row))
    return out


# ---------------------------------------------------------------- layer / model
class _Layer(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int64),
        ("q_heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("inter", ctypes.c_int64),
        ("blocksize", ctypes.c_int64),
        ("eps", ctypes.c_float),
        ("in_norm", ctypes.c_void_p),
        ("post_norm", ctypes.c_void_p),
        ("qw", ctypes.c_void_p),
        ("kw", ctypes.c_void_p),
        ("vw", ctypes.c_void_p),
        ("ow", ctypes.c_void_p),
        ("gw", ctypes.c_void_p),
        ("uw", ctypes.c_void_p),
        ("dw", ctypes.c_void_p),
        ("qa", ctypes.c_void_p),
        ("ka", ctypes.c_void_p),
        ("va", ctypes.c_void_p),
        ("oa", ctypes.c_void_p),
        ("ga", ctypes.c_void_p),
        ("ua", ctypes.c_void_p),
        ("da", ctypes.c_void_p),
        ("qb", ctypes.c_void_p),
        ("kb", ctypes.c_void_p),
        ("vb", ctypes.c_void_p),
    ]


def layer_step_hf(layer: dict, cfg: dict, x: np.ndarray, kcache: np.ndarray, vcache: np.ndarray, cap: int, pos: int,
                  cos_row: np.ndarray, sin_row: np.ndarray) -> None:
    """One Qwen2 decoder layer in Transformers' bf16 order (in place on x and caches).

    layer: numpy arrays {in_norm, post_norm, q/k/v/o/gate/up/down: (packed, absmax), q_b/k_b/v_b}.
    """

    def v(a):
        return None if a is None else ctypes.c_void_p(a.ctypes.data)

    L = _Layer(
        cfg["hidden"], cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["inter"], 64, cfg["eps"],
        v(layer["in_norm"]), v(layer["post_norm"]),
        v(layer["q"][0]), v(layer["k"][0]), v(layer["v"][0]), v(layer["o"][0]), v(layer["gate"][0]), v(layer["up"][0]),
        v(layer["down"][0]),
        v(layer["q"][1]), v(layer["k"][1]), v(layer["v"][1]), v(layer["o"][1]), v(layer["gate"][1]), v(layer["up"][1]),
        v(layer["down"][1]),
        v(layer.get("q_b")), v(layer.get("k_b")), v(layer.get("v_b")),
    )
    lib().kc_layer_step_hf(
        ctypes.byref(L), _ptr(x), _ptr(kcache), _ptr(vcache), ctypes.c_int64(cap), ctypes.c_int64(pos), _ptr(cos_row), _ptr(sin_row)
    )


def lm_head_argmax(x: np.ndarray, final_norm: np.ndarray, emb: np.ndarray, eps: float, want_logits: bool = False):
    vocab, hidden = emb.shape
    logits = np.zeros(vocab, dtype=np.uint16) if want_logits else None
    tok = lib().kc_lm_head_argmax(
        _ptr(x), _ptr(final_norm), _ptr(emb), ctypes.c_int64(vocab), ctypes.c_int64(hidden), ctypes.c_float(eps), _ptr(logits)
    )
    return int(tok), logits
