"""GPU parity of every sm_100a kernel, called through the C ABI, against the
CPU oracle on identical bytes.

Tolerances: NF4 dequant and quantisation are bit-exact; GEMV / layer outputs
must satisfy |gpu - oracle| <= 2e-3 + 1e-2 * |oracle| (
bf16); attention uses the reference's atol = rtol = 3.5e-3
(tools/correctness/run_qwen2_gqa_check.py, tests/qwen2_gqa_smoke.cu:39).
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from tests import fixtures as F
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
GQA_TOL = 3.5e-3


def _torch():
    import torch

    return torch


# Every device tensor a test creates stays referenced until the test ends:
# ctypes calls take raw pointers, and a temporary freed before the launch
# would hand its memory to the next allocation.
_LIVE: list = []


@pytest.fixture(autouse=True)
def _keep_device_tensors_alive():
    yield
    _torch().cuda.synchronize()
    _LIVE.clear()


def dev(a: np.ndarray):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(a).copy()).cuda()
    _LIVE.append(t)
    return t


def host(t) -> np.ndarray:
    torch = _torch()
    torch.cuda.synchronize()
    return t.cpu().numpy()


def stream() -> int:
    return int(_torch().cuda.current_stream().cuda_stream)


def ok(lib, h, status):
    assert status == 0, lib.kudacuda_last_error(h)


def close(actual: np.ndarray, expected: np.ndarray, atol=ATOL, rtol=RTOL):
    err = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    bound = atol + rtol * np.abs(expected.astype(np.float64))
    bad = int(np.sum(~(err <= bound)))
    assert bad == 0, f"{bad} mismatches, max abs err {err.max():.3e}"


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """bf16 unit in the last place at |v| (7 stored mantissa bits)."""

    v = np.maximum(np.abs(v.astype(np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(v)) - 7)


def close_chain(actual: np.ndarray, expected: np.ndarray, intermediates: tuple = (), max_ulps: int = 2,
                max_frac_outside: float = 1e-2):
    """Output of a chain of bf16 roundings (Transformers order).  The GPU and
    the oracle accumulate in different orders (~1e-4 relative, f16 codebook
    levels), so a rounded intermediate can land one bf16 ulp apart and the
    final rounding can add one more.  Bound per element: max_ulps ulps of the
    output + one ulp of every rounded intermediate (oracle magnitudes) + atol;
    and all but a max_frac_outside fraction within the single-rounding
    tolerance 1e-2 rel / 2e-3 abs."""

    err = np.abs(actual.astype(np.float64) - expected.astype(np.float64))
    bound = max_ulps * bf16_ulp(expected) + ATOL
    for inter in intermediates:
        bound = bound + bf16_ulp(np.asarray(inter, dtype=np.float64))
    assert np.all(err <= bound), f"max abs err {err.max():.3e} ({int(np.sum(err > bound))} over the chain bound)"
    outside = np.mean(~(err <= ATOL + RTOL * np.abs(expected.astype(np.float64))))
    assert outside <= max_frac_outside, f"{outside:.2e} of elements outside 1e-2/2e-3"


def err_word(lib, h) -> int:
    import ctypes

    w = ctypes.c_int(0)
    assert lib.kudacuda_sm100_error_word(h, ctypes.byref(w), 1) == 0
    return int(w.value)


# ------------------------------------------------------------------ NF4 dequant / quantise
def test_nf4_dequant_bit_exact(kc_lib, kc_handle):
    g = F.rng(1)
    n = 11008 * 2048
    packed = g.integers(0, 256, n // 2, dtype=np.uint8)
    absmax = g.random(n // 64, dtype=np.float32) * np.float32(0.1)
    out = dev(np.zeros(n, dtype=np.float32))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_nf4_dequantize(
        kc_handle, dev(packed).data_ptr(), dev(absmax).data_ptr(), out.data_ptr(), 0, n, 64, stream()))
    np.testing.assert_array_equal(host(out).view(np.uint32), O.nf4_dequant(packed, absmax, n).view(np.uint32))


def test_nf4_dequant_odd_length_and_bf16(kc_lib, kc_handle):
    g = F.rng(2)
    n = 64 * 5 + 33
    packed = g.integers(0, 256, (n + 1) // 2, dtype=np.uint8)
    absmax = g.random((n + 63) // 64, dtype=np.float32)
    out = dev(np.zeros(n, dtype=np.uint16))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_nf4_dequantize(
        kc_handle, dev(packed).data_ptr(), dev(absmax).data_ptr(), out.data_ptr(), 2, n, 64, stream()))
    np.testing.assert_array_equal(host(out), O.bf16_bits(O.nf4_dequant(packed, absmax, n)))


@pytest.mark.parametrize("in_dtype", [0, 2])
def test_nf4_quantize_bit_exact(kc_lib, kc_handle, in_dtype):
    g = F.rng(3)
    n = 2048 * 256 + 64 * 3
    w = (g.standard_normal(n, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    w[:64] = 0.0  # an all-zero block
    w[64:128] *= 1e-30  # tiny block
    if in_dtype == 2:
        bits = O.bf16_bits(w)
        src = dev(bits)
        w_ref = O.bf16_to_f32(bits)
    else:
        src = dev(w)
        w_ref = w
    packed = dev(np.zeros(n // 2, dtype=np.uint8))
    absmax = dev(np.zeros(n // 64, dtype=np.float32))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_nf4_quantize(
        kc_handle, src.data_ptr(), in_dtype, packed.data_ptr(), absmax.data_ptr(), n, 64, stream()))
    ref_p, ref_a = O.nf4_quantize(w_ref)
    np.testing.assert_array_equal(host(absmax).view(np.uint32), ref_a.view(np.uint32))
    np.testing.assert_array_equal(host(packed), ref_p)


# ------------------------------------------------------------------ GEMV (config 1)
@pytest.mark.parametrize("rows,k", [(11008, 2048), (2048, 11008), (256, 2048), (130, 64), (1, 128)])
def test_nf4_gemv_bf16_matches_oracle(kc_lib, kc_handle, rows, k):
    g = F.rng(10 + rows % 7)
    packed, absmax = F.nf4_weight(g, rows, k)
    x = F.bf16_normal(g, k)
    y = dev(np.zeros(rows, dtype=np.uint16))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_nf4_gemv(
        kc_handle, dev(x).data_ptr(), 2, dev(packed).data_ptr(), dev(absmax).data_ptr(), 0, y.data_ptr(), 2,
        rows, k, 64, stream()))
    ref = O.nf4_gemv(O.bf16_to_f32(x), packed, absmax, rows, k)
    close(O.bf16_to_f32(host(y)), O.bf16_to_f32(O.bf16_bits(ref)))
    assert err_word(kc_lib, kc_handle) == 0


def test_nf4_gemv_f32_out_with_bias(kc_lib, kc_handle):
    g = F.rng(20)
    rows, k = 2048, 2048
    packed, absmax = F.nf4_weight(g, rows, k)
    x = (g.standard_normal(k, dtype=np.float32)).astype(np.float32)
    bias = (g.standard_normal(rows, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    y = dev(np.zeros(rows, dtype=np.float32))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_nf4_gemv(
        kc_handle, dev(x).data_ptr(), 0, dev(packed).data_ptr(), dev(absmax).data_ptr(), dev(bias).data_ptr(),
        y.data_ptr(), 0, rows, k, 64, stream()))
    # f32 input is staged as f16 for the mixed FMA: compare against the
    # oracle fed with the same f16-rounded activations
    ref = O.nf4_gemv(O.f16_to_f32(O.f16_bits(x)), packed, absmax, rows, k) + bias
    close(host(y), ref, atol=1e-3, rtol=1e-3)


def test_gemv_rejects_bad_shapes(kc_lib, kc_handle):
    st = kc_lib.kudacuda_sm100_nf4_gemv(kc_handle, 1 << 20, 2, 1 << 20, 1 << 20, 0, 1 << 20, 2, 16, 100, 64, stream())
    assert st == 1
    assert b"k a multiple of 64" in kc_lib.kudacuda_last_error(kc_handle)


# ------------------------------------------------------------------ reference ABI: fused QKV
@pytest.mark.parametrize("variant", ["", "_v2", "_v3"])
def test_reference_abi_fused_qkv_nf4_smoke_fixture(kc_lib, kc_handle, variant):
    c = F.smoke_qkv_case(O.F16)
    qo_ref, ko_ref, vo_ref, norm_ref = O.qkv_nf4_ref(c["x"], c["nw"], O.F16, c["eps"], c["q"], c["k"], c["v"])
    t = {n: dev(a) for n, a in (("x", c["x"]), ("nw", c["nw"]))}
    q = [dev(a) for a in c["q"][:3]]
    k = [dev(a) for a in c["k"][:3]]
    v = [dev(a) for a in c["v"][:3]]
    qo = dev(np.zeros((1, 2048), dtype=np.uint16))
    ko = dev(np.zeros((1, 256), dtype=np.uint16))
    vo = dev(np.zeros((1, 256), dtype=np.uint16))
    ws = dev(np.zeros((1, 2048), dtype=np.float32))
    args = [kc_handle, t["x"].data_ptr(), t["nw"].data_ptr(), q[0].data_ptr(), q[1].data_ptr(), q[2].data_ptr(),
            k[0].data_ptr(), k[1].data_ptr(), k[2].data_ptr(), v[0].data_ptr(), v[1].data_ptr(), v[2].data_ptr()]
    if variant:
        args.append(ws.data_ptr())
    args += [qo.data_ptr(), ko.data_ptr(), vo.data_ptr(), 1, 2048, 2048, 256, 64, c["eps"], stream()]
    fn = getattr(kc_lib, "kudacuda_qwen2_fused_rmsnorm_qkv_nf4" + variant)
    ok(kc_lib, kc_handle, fn(*args))
    for got, ref in ((qo, qo_ref), (ko, ko_ref), (vo, vo_ref)):
        g = O.f16_to_f32(host(got).reshape(-1))
        r = O.f16_to_f32(ref)
        # tests/nf4_tiled_gemv_smoke.cu:50 -- the reference's own tolerance for this fixture
        # (weights with absmax 0.2-0.4 and fp32-normalised inputs; see the seeded test below
        # for the north_star tolerance on BASELINE-distributed data)
        assert np.max(np.abs(g - r)) <= 0.035
    if variant:
        close(host(ws).reshape(-1), norm_ref, atol=1e-5, rtol=1e-5)


def test_reference_abi_fused_qkv_nf4_seeded_north_star_tolerance(kc_lib, kc_handle):
    """BASELINE data (N(0,0.02) NF4 weights, N(0,1) input): 1e-2 rel / 2e-3 abs."""

    g = F.rng(40)
    x = O.f16_bits(g.standard_normal(2048, dtype=np.float32))
    nw = O.f16_bits((1 + 0.02 * g.standard_normal(2048)).astype(np.float32))
    mats = []
    for rows in (2048, 256, 256):
        p, a = F.nf4_weight(g, rows, 2048)
        mats.append((p, a, O.f16_bits((0.02 * g.standard_normal(rows)).astype(np.float32)), rows))
    qo_ref, ko_ref, vo_ref, _ = O.qkv_nf4_ref(x, nw, O.F16, 1e-6, *mats)
    outs = [dev(np.zeros((1, r), dtype=np.uint16)) for r in (2048, 256, 256)]
    ptrs = [dev(a).data_ptr() for m in mats for a in m[:3]]
    ok(kc_lib, kc_handle, kc_lib.kudacuda_qwen2_fused_rmsnorm_qkv_nf4(
        kc_handle, dev(x).data_ptr(), dev(nw).data_ptr(), *ptrs, *[o.data_ptr() for o in outs],
        1, 2048, 2048, 256, 64, 1e-6, stream()))
    for got, ref in zip(outs, (qo_ref, ko_ref, vo_ref)):
        close(O.f16_to_f32(host(got).reshape(-1)), O.f16_to_f32(ref))


def test_reference_abi_qkv_guard_rejects_shapes(kc_lib, kc_handle):
    st = kc_lib.kudacuda_qwen2_fused_rmsnorm_qkv_nf4(kc_handle, *([1 << 20] * 14), 2, 2048, 2048, 256, 64, 1e-5, stream())
    assert st == 1
    assert b"rows=1, hidden=2048" in kc_lib.kudacuda_last_error(kc_handle)


# ------------------------------------------------------------------ reference ABI: SwiGLU
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_reference_abi_swiglu_nf4_smoke_fixture(kc_lib, kc_handle, dtype):
    c = F.smoke_swiglu_case(dtype)
    ref = O.swiglu_nf4_ref(c["x"], c["nw"], dtype, c["eps"], c["gate"], c["up"], c["inter"])
    out = dev(np.zeros((1, c["inter"]), dtype=np.uint16))
    fn = kc_lib.kudacuda_qwen2_swiglu_nf4 if dtype == O.F16 else kc_lib.kudacuda_qwen2_swiglu_nf4_bf16
    tensors = [dev(c["x"]), dev(c["nw"]), dev(c["gate"][0]), dev(c["gate"][1]), dev(c["up"][0]), dev(c["up"][1])]
    ok(kc_lib, kc_handle, fn(kc_handle, *[t.data_ptr() for t in tensors], out.data_ptr(), 1, 2048, 11008, 64,
                             c["eps"], stream()))
    conv = O.f16_to_f32 if dtype == O.F16 else O.bf16_to_f32
    got, exp = conv(host(out).reshape(-1)), conv(ref)
    tol = 0.045 if dtype == O.F16 else 0.08  # tests/nf4_swiglu_smoke.cu:48, nf4_swiglu_bf16_smoke.cu:48
    assert np.max(np.abs(got - exp)) <= tol


# ------------------------------------------------------------------ reference ABI: GQA
@pytest.mark.parametrize("entry", ["direct", "group_tiled", "vectorized", "graph", "workspace_v3"])
def test_reference_abi_gqa_smoke_fixture(kc_lib, kc_handle, entry):
    kv_len = 37
    c = F.smoke_gqa_case(kv_len, O.F16)
    cap = 512 if entry in ("graph", "workspace_v3") else kv_len
    # caches laid out [kv_heads][cap][128]; rows >= kv_len stay zero
    kc = np.zeros((2, cap, 128), dtype=np.uint16)
    vc = np.zeros((2, cap, 128), dtype=np.uint16)
    kc[:, :kv_len] = c["k"].reshape(2, kv_len, 128)
    vc[:, :kv_len] = c["v"].reshape(2, kv_len, 128)
    ref = O.gqa_decode(c["q"], np.ascontiguousarray(kc), np.ascontiguousarray(vc), O.F16, 16, 2, 128, kv_len, cap,
                       float(c["scale"]))
    q, k, v = dev(c["q"]), dev(kc), dev(vc)
    out = dev(np.zeros(16 * 128, dtype=np.uint16))
    kvl = dev(np.array([kv_len], dtype=np.int32))
    s = stream()
    if entry == "direct":
        st = kc_lib.kudacuda_qwen2_gqa_decode(kc_handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                              1, 1, kv_len, 16, 2, 128, float(c["scale"]), s)
    elif entry == "group_tiled":
        st = kc_lib.kudacuda_qwen2_gqa_decode_group_tiled(kc_handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                          out.data_ptr(), 1, 1, kv_len, 16, 2, 128, float(c["scale"]), s)
    elif entry == "vectorized":
        st = kc_lib.kudacuda_qwen2_gqa_decode_vectorized(kc_handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                         out.data_ptr(), 1, 1, kv_len, 16, 2, 128, float(c["scale"]), s)
    elif entry == "graph":
        st = kc_lib.kudacuda_qwen2_gqa_decode_graph(kc_handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                    out.data_ptr(), 1, 1, cap, 16, 2, 128, float(c["scale"]),
                                                    kvl.data_ptr(), s)
    else:
        ws = dev(np.zeros(16 * 8 * 130, dtype=np.float32))
        st = kc_lib.kudacuda_qwen2_gqa_decode_workspace_v3(kc_handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                           out.data_ptr(), ws.data_ptr(), kvl.data_ptr(), 1, 1, cap,
                                                           16, 2, 128, float(c["scale"]), s)
    ok(kc_lib, kc_handle, st)
    close(O.f16_to_f32(host(out)), O.f16_to_f32(ref), atol=GQA_TOL, rtol=GQA_TOL)


@pytest.mark.parametrize("kv_len", [1, 7, 128, 512, 585, 1024, 2048])
def test_reference_abi_gqa_seeded_lengths(kc_lib, kc_handle, kv_len):
    """tools/correctness/run_qwen2_gqa_check.py: seeded randn, kv in {1,7,128,512,585,1024,2048}."""

    g = F.rng(F.SEED + kv_len)
    q = O.f16_bits(g.standard_normal(16 * 128, dtype=np.float32))
    k = O.f16_bits(g.standard_normal(2 * kv_len * 128, dtype=np.float32))
    v = O.f16_bits(g.standard_normal(2 * kv_len * 128, dtype=np.float32))
    scale = 1.0 / math.sqrt(128)
    ref = O.gqa_decode(q, k, v, O.F16, 16, 2, 128, kv_len, kv_len, scale)
    out = dev(np.zeros(16 * 128, dtype=np.uint16))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_qwen2_gqa_decode(kc_handle, dev(q).data_ptr(), dev(k).data_ptr(),
                                                           dev(v).data_ptr(), out.data_ptr(), 1, 1, kv_len, 16, 2, 128,
                                                           scale, stream()))
    close(O.f16_to_f32(host(out)), O.f16_to_f32(ref), atol=GQA_TOL, rtol=GQA_TOL)


@pytest.mark.parametrize("q_heads,kv_heads,kv_len,cap,batch", [(16, 2, 512, 512, 1), (16, 2, 300, 2048, 1),
                                                               (32, 8, 4096, 4096, 1), (8, 8, 77, 128, 1),
                                                               (16, 8, 33, 64, 1), (16, 2, 100, 512, 4)])
def test_sm100_gqa_bf16_device_length(kc_lib, kc_handle, q_heads, kv_heads, kv_len, cap, batch):
    g = F.rng(kv_len + q_heads)
    d = 128
    q = F.bf16_normal(g, batch * q_heads * d)
    kc = F.bf16_normal(g, batch * kv_heads * cap * d)
    vc = F.bf16_normal(g, batch * kv_heads * cap * d)
    scale = 1.0 / math.sqrt(d)
    nbytes = kc_lib.kudacuda_sm100_gqa_workspace_bytes(batch, q_heads, kv_heads, cap, d)
    ws = dev(np.zeros(nbytes // 4, dtype=np.float32))
    tickets = dev(np.zeros(batch * kv_heads, dtype=np.int32))
    kvl = dev(np.array([kv_len], dtype=np.int32))
    out = dev(np.zeros(batch * q_heads * d, dtype=np.uint16))
    dq, dk, dv = dev(q), dev(kc), dev(vc)
    for _ in range(2):  # second call checks that tickets self-reset
        ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_gqa_decode(
            kc_handle, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), ws.data_ptr(), nbytes,
            tickets.data_ptr(), kvl.data_ptr(), 2, batch, 0, cap, q_heads, kv_heads, d, scale, stream()))
        got = host(out).reshape(batch, -1)
        for b in range(batch):
            ref = O.gqa_decode(q.reshape(batch, -1)[b].copy(), kc.reshape(batch, -1)[b].copy(),
                               vc.reshape(batch, -1)[b].copy(), O.BF16, q_heads, kv_heads, d, kv_len, cap, scale)
            close(O.bf16_to_f32(got[b]), O.bf16_to_f32(ref), atol=GQA_TOL, rtol=GQA_TOL)
    assert int(host(tickets).sum()) == 0


# ------------------------------------------------------------------ sm100 bf16 layer blocks
def _rope(max_pos=4096, d=128, theta=1e6):
    return F.rope_tables(max_pos, d, theta)


def test_sm100_qkv_rope_kv_append(kc_lib, kc_handle):
    g = F.rng(30)
    cfg = dict(hidden=2048, q_heads=16, kv_heads=2, head_dim=128, inter=11008, eps=1e-6)
    layer = F.qwen_layer(g)
    cos, sin = _rope()
    cap, pos = 512, 77
    x = F.bf16_normal(g, 2048)
    kc = np.zeros((2, cap, 128), dtype=np.uint16)
    vc = np.zeros((2, cap, 128), dtype=np.uint16)
    # oracle: norm -> linears -> rope -> append
    xn = O.rmsnorm_hf_bf16(x, layer["in_norm"], 1e-6)
    def lin(wp, bias):
        y = O.bf16_to_f32(O.bf16_bits(O.nf4_gemv(O.bf16_to_f32(xn), wp[0], wp[1], wp[1].size * 64 // 2048, 2048)))
        return O.bf16_bits(O.bf16_to_f32(O.bf16_bits(y + O.bf16_to_f32(bias))))
    q_ref = O.rope_hf_bf16(lin(layer["q"], layer["q_b"]), 16, 128, cos[pos], sin[pos])
    k_ref = O.rope_hf_bf16(lin(layer["k"], layer["k_b"]), 2, 128, cos[pos], sin[pos])
    v_ref = lin(layer["v"], layer["v_b"])

    t = {key: dev(val) for key, val in (("x", x), ("nw", layer["in_norm"]), ("cos", cos), ("sin", sin))}
    W = {n: (dev(layer[n][0]), dev(layer[n][1]), dev(layer[n + "_b"])) for n in ("q", "k", "v")}
    posd = dev(np.array([pos], dtype=np.int32))
    qo = dev(np.zeros(2048, dtype=np.uint16))
    kd, vd = dev(kc), dev(vc)
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16(
        kc_handle, t["x"].data_ptr(), t["nw"].data_ptr(),
        *[p.data_ptr() for n in ("q", "k", "v") for p in W[n]],
        t["cos"].data_ptr(), t["sin"].data_ptr(), posd.data_ptr(), qo.data_ptr(), kd.data_ptr(), vd.data_ptr(),
        2048, 16, 2, 128, cap, 4096, 64, 1e-6, stream()))
    # chain: bf16(acc) -> bf16(+bias) -> RoPE products -> bf16 sum; the
    # pre-rotation values bound the intermediates (both rotation partners)
    def partners(lin_out, heads):
        y = O.bf16_to_f32(lin_out).reshape(heads, 2, 64)
        m = np.maximum(np.abs(y[:, 0]), np.abs(y[:, 1]))
        return np.concatenate([m, m], axis=1).reshape(-1)
    qm = partners(lin(layer["q"], layer["q_b"]), 16)
    km = partners(lin(layer["k"], layer["k_b"]), 2)
    close_chain(O.bf16_to_f32(host(qo)), O.bf16_to_f32(q_ref), intermediates=(qm, qm, qm))
    kh, vh = host(kd), host(vd)
    close_chain(O.bf16_to_f32(kh[:, pos].reshape(-1)), O.bf16_to_f32(k_ref), intermediates=(km, km, km))
    close_chain(O.bf16_to_f32(vh[:, pos].reshape(-1)), O.bf16_to_f32(v_ref))
    kh[:, pos] = 0
    vh[:, pos] = 0
    assert not kh.any() and not vh.any(), "kernel wrote outside the appended position"
    assert err_word(kc_lib, kc_handle) == 0


def test_sm100_swiglu_hf_and_residual(kc_lib, kc_handle):
    g = F.rng(31)
    hidden, inter = 2048, 11008
    gate = F.nf4_weight(g, inter, hidden)
    up = F.nf4_weight(g, inter, hidden)
    down = F.nf4_weight(g, hidden, inter)
    nw = F.bf16_normal(g, hidden, 0.02, 1.0)
    x = F.bf16_normal(g, hidden)
    xn = O.bf16_to_f32(O.rmsnorm_hf_bf16(x, nw, 1e-6))
    gr = O.bf16_to_f32(O.bf16_bits(O.nf4_gemv(xn, gate[0], gate[1], inter, hidden)))
    ur = O.bf16_to_f32(O.bf16_bits(O.nf4_gemv(xn, up[0], up[1], inter, hidden)))
    act = O.bf16_to_f32(O.bf16_bits(gr / (1.0 + np.exp(-gr))))
    h_ref = O.bf16_bits(act * ur)
    h = dev(np.zeros(inter, dtype=np.uint16))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_swiglu_nf4_bf16(
        kc_handle, dev(x).data_ptr(), dev(nw).data_ptr(), dev(gate[0]).data_ptr(), dev(gate[1]).data_ptr(),
        dev(up[0]).data_ptr(), dev(up[1]).data_ptr(), h.data_ptr(), hidden, inter, 64, 1e-6, stream()))
    hg = host(h)
    close_chain(O.bf16_to_f32(hg), O.bf16_to_f32(h_ref), intermediates=(gr, ur, act))
    # down_proj + residual, fed with the oracle's h so the check isolates the GEMV
    resid = dev(x)
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_nf4_linear_residual_bf16(
        kc_handle, dev(h_ref).data_ptr(), dev(down[0]).data_ptr(), dev(down[1]).data_ptr(), resid.data_ptr(),
        hidden, inter, 64, stream()))
    d_ref = O.bf16_to_f32(O.bf16_bits(O.nf4_gemv(O.bf16_to_f32(h_ref), down[0], down[1], hidden, inter)))
    r_ref = O.bf16_to_f32(O.bf16_bits(O.bf16_to_f32(x) + d_ref))
    close_chain(O.bf16_to_f32(host(resid)), r_ref, intermediates=(d_ref,))


def test_sm100_lm_head_argmax(kc_lib, kc_handle):
    g = F.rng(32)
    vocab, hidden = 151936, 2048
    emb = F.bf16_normal(g, vocab * hidden, 0.02).reshape(vocab, hidden)
    fn = F.bf16_normal(g, hidden, 0.02, 1.0)
    x = F.bf16_normal(g, hidden)
    tok_ref, logits_ref = O.lm_head_argmax(x, fn, emb, 1e-6, want_logits=True)
    nbytes = kc_lib.kudacuda_sm100_lm_head_workspace_bytes()
    ws = dev(np.zeros(nbytes // 4, dtype=np.float32))
    ticket = dev(np.zeros(1, dtype=np.int32))
    tok = dev(np.zeros(1, dtype=np.int32))
    logits = dev(np.zeros(vocab, dtype=np.uint16))
    demb = dev(emb)
    for _ in range(2):
        ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_lm_head_argmax_bf16(
            kc_handle, dev(x).data_ptr(), dev(fn).data_ptr(), demb.data_ptr(), logits.data_ptr(), tok.data_ptr(),
            ws.data_ptr(), nbytes, ticket.data_ptr(), vocab, hidden, 1e-6, stream()))
        lg = O.bf16_to_f32(host(logits))
        close(lg, O.bf16_to_f32(logits_ref))
        t = int(host(tok)[0])
        # argmax of the GPU's own logits, lowest index on ties
        assert t == int(np.argmax(lg))
        assert lg[t] >= O.bf16_to_f32(logits_ref)[tok_ref] - 2 * (ATOL + RTOL * abs(O.bf16_to_f32(logits_ref)[tok_ref]))
    assert int(host(ticket)[0]) == 0


def test_sm100_embedding_gather(kc_lib, kc_handle):
    g = F.rng(33)
    emb = F.bf16_normal(g, 1000 * 256).reshape(1000, 256)
    tok = dev(np.array([777], dtype=np.int32))
    out = dev(np.zeros(256, dtype=np.uint16))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_embedding_bf16(kc_handle, dev(emb).data_ptr(), tok.data_ptr(),
                                                               out.data_ptr(), 1000, 256, stream()))
    np.testing.assert_array_equal(host(out), emb[777])


def test_reference_abi_small_ops(kc_lib, kc_handle):
    g = F.rng(34)
    a = g.standard_normal(1000, dtype=np.float32)
    b = g.standard_normal(1000, dtype=np.float32)
    o = dev(np.zeros(1000, dtype=np.float32))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_vector_add(kc_handle, dev(a).data_ptr(), dev(b).data_ptr(), o.data_ptr(),
                                                     1000, stream()))
    np.testing.assert_array_equal(host(o), a + b)
    rows = g.standard_normal((3, 512), dtype=np.float32)
    w = g.standard_normal(512, dtype=np.float32)
    ro = dev(np.zeros((3, 512), dtype=np.float32))
    ok(kc_lib, kc_handle, kc_lib.kudacuda_rmsnorm(kc_handle, dev(rows).data_ptr(), dev(w).data_ptr(), ro.data_ptr(),
                                                  3, 512, 1e-5, stream()))
    close(host(ro), O.rmsnorm_f64(rows, w, 1e-5).astype(np.float32), atol=1e-5, rtol=1e-5)
