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
    """fp32 -> f16 bit patterns, round to nearest even; beyond the f16 range -> inf (IEEE, as torch)."""

    with np.errstate(over="ignore"):
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


# ---------------------------------------------------------------- persistent-decode weight layout
# The "group tile" stream layout consumed by kudacuda_sm100_decode_layers_persistent
# (no reference counterpart: a load-time re-layout of the bitsandbytes NF4
# storage, kernels/common/nf4_device.cuh:29-40, that keeps every code byte and
# absmax value bit-exact and only moves them).  Restated here in numpy as the
# checker of the device re-tile kernel.
RETILE_PLAIN, RETILE_SWIGLU, RETILE_QKV_ROPE = 0, 1, 2


def retile_rows(mode: int, rows: tuple[int, int, int], head_dim: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(matrix index, source row) of every group row, each shaped [groups, 64].

    plain: group g rows 64g .. 64g+63 of matrix 0; SwiGLU: rows 0..31 are gate
    rows 32g.., rows 32..63 the matching up rows; q/k/v: each q head then each
    k head in groups of 32 RoPE pairs (row r < 32 is element 32m + r of the
    head's first half, row r + 32 its partner in the second half), then plain
    64-row groups of v."""

    rr = np.arange(64)
    if mode == RETILE_PLAIN:
        groups = rows[0] // 64
        m = np.zeros((groups, 64), dtype=np.int64)
        r = np.arange(groups)[:, None] * 64 + rr[None, :]
        return m, r
    if mode == RETILE_SWIGLU:
        groups = rows[0] // 32
        m = np.broadcast_to((rr >= 32).astype(np.int64), (groups, 64)).copy()
        r = np.arange(groups)[:, None] * 32 + (rr & 31)[None, :]
        return m, r
    if mode == RETILE_QKV_ROPE:
        hd = head_dim
        gph = hd // 64
        qg, kg, vg = rows[0] // hd * gph, rows[1] // hd * gph, rows[2] // 64
        ms, rs = [], []
        for grp in range(qg + kg + vg):
            if grp < qg + kg:
                mat = 0 if grp < qg else 1
                u = grp if grp < qg else grp - qg
                head, mm = divmod(u, gph)
                ms.append(np.full(64, mat))
                rs.append(head * hd + 32 * mm + (rr & 31) + np.where(rr >= 32, hd // 2, 0))
            else:
                ms.append(np.full(64, 2))
                rs.append(64 * (grp - qg - kg) + rr)
        return np.stack(ms).astype(np.int64), np.stack(rs).astype(np.int64)
    raise ValueError(f"unknown re-tile mode {mode}")


def retile_nf4(mode: int, mats: list[tuple[np.ndarray, np.ndarray, int]], k: int, head_dim: int = 0):
    """bitsandbytes (packed [rows*k/2] u8, absmax [rows*k/64] f32, rows) matrices ->
    (codes u8 [groups * (k/64) * 2048], absmax f32 [groups * (k/64) * 64]).

    Chunk (group, block b): 4 tiles x 32 lanes x 16 bytes, lane 4g + t holding
    bytes [32b + 8t, +8) of group rows 16*tile + g then 16*tile + 8 + g; then 64
    absmax ordered [half][g][tile] (row 16*tile + 8*half + g)."""

    rows = tuple(m[2] for m in mats) + (0,) * (3 - len(mats))
    msel, rsel = retile_rows(mode, rows, head_dim)
    groups, nbpt = msel.shape[0], k // 64
    packed = [np.asarray(p, dtype=np.uint8).reshape(n, k // 2) for p, _, n in mats]
    absm = [np.asarray(a, dtype=np.float32).reshape(n, nbpt) for _, a, n in mats]
    data = np.zeros((64, groups, k // 2), dtype=np.uint8)
    amax = np.zeros((64, groups, nbpt), dtype=np.float32)
    for gr in range(64):
        for mi in range(len(mats)):
            sel = msel[:, gr] == mi
            data[gr, sel] = packed[mi][rsel[sel, gr]]
            amax[gr, sel] = absm[mi][rsel[sel, gr]]
    data = data.reshape(64, groups, nbpt, 4, 8)  # [group row][group][block][t][8 bytes]
    ia = (16 * np.arange(4)[:, None] + np.arange(8)[None, :])  # [tile, g] -> group row of lane (g, t)'s row A
    codes = np.empty((groups, nbpt, 4, 8, 4, 16), dtype=np.uint8)  # [group][block][tile][g][t][16]
    codes[..., :8] = data[ia].transpose(2, 3, 0, 1, 4, 5)
    codes[..., 8:] = data[ia + 8].transpose(2, 3, 0, 1, 4, 5)
    ab = np.empty((groups, nbpt, 2, 8, 4), dtype=np.float32)  # [group][block][half][g][tile]
    for h in range(2):
        ab[:, :, h] = amax[(16 * np.arange(4)[None, :] + 8 * h + np.arange(8)[:, None])].transpose(2, 3, 0, 1)
    return codes.reshape(-1), ab.reshape(-1)


def tile16_rows(mode: int, rows: tuple[int, int, int], head_dim: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """(matrix index, source row) of every row of every 16-row tile, shaped
    [tiles, 16] -- the row-complete layout of the persistent decode kernel.

    plain: tile t rows 16t .. 16t+15; SwiGLU: rows 0..7 are gate rows 8t..8t+7,
    rows 8..15 the matching up rows; q/k/v: each q head, then each k head, in
    tiles of 8 RoPE pairs (row r < 8 is element 8m + r of the head's first
    half, row r + 8 its partner in the second half), then tiles of 16
    consecutive v rows."""

    r16 = np.arange(16)
    if mode == RETILE_PLAIN:
        t = rows[0] // 16
        return np.zeros((t, 16), dtype=np.int64), np.arange(t)[:, None] * 16 + r16[None, :]
    if mode == RETILE_SWIGLU:
        t = rows[0] // 8
        m = np.broadcast_to((r16 >= 8).astype(np.int64), (t, 16)).copy()
        return m, np.arange(t)[:, None] * 8 + (r16 & 7)[None, :]
    if mode == RETILE_QKV_ROPE:
        hd = head_dim
        per = hd // 16  # tiles per head: hd/2 first-half elements, 8 per tile
        qt, kt, vt = rows[0] // hd * per, rows[1] // hd * per, rows[2] // 16
        ms, rs = [], []
        for tile in range(qt + kt + vt):
            if tile < qt + kt:
                mat = 0 if tile < qt else 1
                u = tile if tile < qt else tile - qt
                head, mm = divmod(u, per)
                ms.append(np.full(16, mat))
                rs.append(head * hd + 8 * mm + (r16 & 7) + np.where(r16 >= 8, hd // 2, 0))
            else:
                ms.append(np.full(16, 2))
                rs.append(16 * (tile - qt - kt) + r16)
        return np.stack(ms).astype(np.int64), np.stack(rs).astype(np.int64)
    raise ValueError(f"unknown re-tile mode {mode}")


def retile_tiles16(mode: int, mats: list[tuple[np.ndarray, np.ndarray, int]], k: int, head_dim: int = 0) -> np.ndarray:
    """bitsandbytes matrices -> units u8 [tiles * (k/64) * 576], tile-major.

    Unit (tile, block b): 512 code bytes, lane 4g + t holding bytes
    [32b + 8t, +8) of tile row g then of tile row g + 8 (its m16n8k16 A
    fragments), then the 16 rows' fp32 absmax of block b as (row g, row g + 8)
    pairs for g = 0..7 (rows 0, 8, 1, 9, ...: lane g's two scales together)."""

    rows = tuple(m[2] for m in mats) + (0,) * (3 - len(mats))
    msel, rsel = tile16_rows(mode, rows, head_dim)
    tiles, nbpt = msel.shape[0], k // 64
    packed = [np.asarray(pk, dtype=np.uint8).reshape(n, k // 2) for pk, _, n in mats]
    absm = [np.asarray(a, dtype=np.float32).reshape(n, nbpt) for _, a, n in mats]
    data = np.zeros((tiles, 16, k // 2), dtype=np.uint8)
    amax = np.zeros((tiles, 16, nbpt), dtype=np.float32)
    for mi in range(len(mats)):
        sel = msel == mi
        data[sel] = packed[mi][rsel[sel]]
        amax[sel] = absm[mi][rsel[sel]]
    d = data.reshape(tiles, 16, nbpt, 4, 8)  # [tile][row][block][t][8 bytes]
    codes = np.empty((tiles, nbpt, 8, 4, 16), dtype=np.uint8)  # [tile][block][g][t][16]
    codes[..., :8] = d[:, :8].transpose(0, 2, 1, 3, 4)
    codes[..., 8:] = d[:, 8:].transpose(0, 2, 1, 3, 4)
    units = np.empty((tiles, nbpt, 576), dtype=np.uint8)
    units[:, :, :512] = codes.reshape(tiles, nbpt, 512)
    pairs = [r for g in range(8) for r in (g, g + 8)]
    units[:, :, 512:] = np.ascontiguousarray(amax.transpose(0, 2, 1)[:, :, pairs]).view(np.uint8).reshape(tiles, nbpt, 64)
    return units.reshape(-1)


# ---------------------------------------------------------------- batched decode GEMM
def batch_gemm_ref(packed: np.ndarray, absmax: np.ndarray | None, rows: int, k: int, x_bits: np.ndarray,
                   weight_type: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """Batched projection as Transformers runs it on bitsandbytes NF4 weights
    for a batch (the reference itself projects one token at a time,
    tests/nf4_tiled_gemv_smoke.cu:86-94): W is dequantised to bf16
    (kernels/common/nf4_device.cuh:29-40 in fp32, rounded once), then
    y[r][b] = sum_k W[r][k] * x[b][k], here exactly in float64.

    weight_type 0: packed NF4 + absmax; 1: packed holds bf16 bits [rows][k].
    x_bits: bf16 bits [n][k].  Returns (y [rows][n] float64, the sum of
    |W[r][k] * x[b][k]| [rows][n], the scale an fp32-accumulation error bound
    is relative to)."""

    if weight_type == 0:
        w = bf16_to_f32(bf16_bits(nf4_dequant(packed, absmax, rows * k))).reshape(rows, k).astype(np.float64)
    else:
        w = bf16_to_f32(np.asarray(packed, dtype=np.uint16)).reshape(rows, k).astype(np.float64)
    x = bf16_to_f32(np.asarray(x_bits, dtype=np.uint16)).reshape(-1, k).astype(np.float64)
    return w @ x.T, np.abs(w) @ np.abs(x).T


def batch_retile(packed: np.ndarray, absmax: np.ndarray, rows: int, k: int) -> np.ndarray:
    """The batched GEMM's streaming form of an NF4 matrix (a load-time move of
    the bitsandbytes storage, kernels/common/nf4_device.cuh:29-40, no value
    changed): per 128-row tile t and 64-element K block kb one 4,608-byte
    record = codes of rows 128t..128t+127, bytes 32kb..32kb+31 ([128][32]),
    then those rows' absmax of block kb (128 fp32); rows past the matrix zero."""

    nblk = k // 64
    tiles = (rows + 127) // 128
    codes = np.zeros((tiles * 128, k // 2), dtype=np.uint8)
    codes[:rows] = np.asarray(packed, dtype=np.uint8).reshape(rows, k // 2)
    am = np.zeros((tiles * 128, nblk), dtype=np.float32)
    am[:rows] = np.asarray(absmax, dtype=np.float32).reshape(rows, nblk)
    c = codes.reshape(tiles, 128, nblk, 32).transpose(0, 2, 1, 3).reshape(tiles, nblk, 4096)
    a = am.reshape(tiles, 128, nblk).transpose(0, 2, 1).copy().view(np.uint8).reshape(tiles, nblk, 512)
    return np.concatenate([c, a], axis=2).reshape(-1)
