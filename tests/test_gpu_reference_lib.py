"""The reference's own CUDA kernels, compiled for sm_100a from its sources
into oracle/_ref/libkudacuda_ref.so, run on the same bytes as the oracle and
this library.

This pins the CPU oracle to the reference implementation itself (not only to
a restatement of its host loops): the reference's fused RMSNorm + NF4 QKV
(v1, v2, v3), NF4 SwiGLU (f16, bf16) and every GQA tactic must agree with the
oracle within the tolerances of the reference's own smoke tests
(tests/nf4_tiled_gemv_smoke.cu:50, tests/nf4_swiglu_smoke.cu:48,
tests/nf4_swiglu_bf16_smoke.cu:48, tests/qwen2_gqa_smoke.cu:39), and this
library's kernels, called through the same ABI entry, must agree with the
reference's output to the same tolerance.

Every call stays inside the reference's guards (rows 1, hidden 2048,
q_out 2048, kv_out 256, intermediate 11008, 16/2/128 heads, kv_len <= 2048
direct and <= 512 for the graph, group-tiled, vectorized and workspace
tactics), which its kernels also re-check on the device.  The module skips
when the reference library was not built (no reference checkout where
build() ran).
"""

from __future__ import annotations

import ctypes
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O
from tests import fixtures as F

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libkudacuda_ref.so"
GQA_TOL = 3.5e-3  # tools/correctness/run_qwen2_gqa_check.py, tests/qwen2_gqa_smoke.cu:39

_LIVE: list = []


@pytest.fixture(autouse=True)
def _keep_alive():
    yield
    import torch

    torch.cuda.synchronize()
    _LIVE.clear()


def dev(a):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a).copy()).cuda()
    _LIVE.append(t)
    return t


def host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def stream() -> int:
    import torch

    return int(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def ref():
    if not REF_LIB.exists():
        pytest.skip("the reference library (oracle/_ref) was not built")
    import torch

    from kudacuda_b200 import native

    torch.cuda.init()
    lib = native.configure(ctypes.CDLL(str(REF_LIB)))
    h = lib.kudacuda_create(0)
    assert h
    assert lib.kudacuda_freeze(h) == 0, lib.kudacuda_last_error(h)
    yield lib, h
    torch.cuda.synchronize()
    lib.kudacuda_destroy(h)


def _both(ref, kc_lib, kc_handle):
    return (("reference", ref[0], ref[1]), ("b200", kc_lib, kc_handle))


# ------------------------------------------------------------------ fused RMSNorm + NF4 QKV
@pytest.mark.parametrize("variant", ["", "_v2", "_v3"])
def test_reference_qkv_kernels_pin_the_oracle(ref, kc_lib, kc_handle, variant):
    c = F.smoke_qkv_case(O.F16)
    qo_ref, ko_ref, vo_ref, _ = O.qkv_nf4_ref(c["x"], c["nw"], O.F16, c["eps"], c["q"], c["k"], c["v"])
    x, nw = dev(c["x"]), dev(c["nw"])
    mats = [dev(a) for m in (c["q"], c["k"], c["v"]) for a in m[:3]]
    outs = {}
    for name, lib, h in _both(ref, kc_lib, kc_handle):
        qo = dev(np.zeros((1, 2048), dtype=np.uint16))
        ko = dev(np.zeros((1, 256), dtype=np.uint16))
        vo = dev(np.zeros((1, 256), dtype=np.uint16))
        ws = dev(np.zeros((1, 2048), dtype=np.float32))
        args = [h, x.data_ptr(), nw.data_ptr(), *[m.data_ptr() for m in mats]]
        if variant:
            args.append(ws.data_ptr())
        args += [qo.data_ptr(), ko.data_ptr(), vo.data_ptr(), 1, 2048, 2048, 256, 64, c["eps"], stream()]
        st = getattr(lib, "kudacuda_qwen2_fused_rmsnorm_qkv_nf4" + variant)(*args)
        assert st == 0, lib.kudacuda_last_error(h)
        outs[name] = [O.f16_to_f32(host(t).reshape(-1)) for t in (qo, ko, vo)]
    for i, exp in enumerate((qo_ref, ko_ref, vo_ref)):
        e = O.f16_to_f32(exp)
        err_ref = np.max(np.abs(outs["reference"][i] - e))
        assert err_ref <= 0.035, f"reference kernel vs oracle: {err_ref:.3e}"
        assert np.max(np.abs(outs["b200"][i] - outs["reference"][i])) <= 0.035


# ------------------------------------------------------------------ NF4 SwiGLU
@pytest.mark.parametrize("dtype", [O.F16, O.BF16])
def test_reference_swiglu_kernels_pin_the_oracle(ref, kc_lib, kc_handle, dtype):
    c = F.smoke_swiglu_case(dtype)
    exp = O.swiglu_nf4_ref(c["x"], c["nw"], dtype, c["eps"], c["gate"], c["up"], c["inter"])
    conv = O.f16_to_f32 if dtype == O.F16 else O.bf16_to_f32
    tol = 0.045 if dtype == O.F16 else 0.08
    tensors = [dev(c["x"]), dev(c["nw"]), dev(c["gate"][0]), dev(c["gate"][1]), dev(c["up"][0]), dev(c["up"][1])]
    outs = {}
    for name, lib, h in _both(ref, kc_lib, kc_handle):
        out = dev(np.zeros((1, c["inter"]), dtype=np.uint16))
        fn = lib.kudacuda_qwen2_swiglu_nf4 if dtype == O.F16 else lib.kudacuda_qwen2_swiglu_nf4_bf16
        st = fn(h, *[t.data_ptr() for t in tensors], out.data_ptr(), 1, 2048, 11008, 64, c["eps"], stream())
        assert st == 0, lib.kudacuda_last_error(h)
        outs[name] = conv(host(out).reshape(-1))
    e = conv(exp)
    err_ref = np.max(np.abs(outs["reference"] - e))
    assert err_ref <= tol, f"reference kernel vs oracle: {err_ref:.3e}"
    assert np.max(np.abs(outs["b200"] - outs["reference"])) <= tol


# ------------------------------------------------------------------ GQA decode
@pytest.mark.parametrize("kv_len", [1, 7, 128, 512, 585, 1024, 2048])
def test_reference_gqa_direct_pins_the_oracle(ref, kc_lib, kc_handle, kv_len):
    """Seeded randn at the reference correctness check's lengths
    (tools/correctness/run_qwen2_gqa_check.py:41,63,79-81)."""

    g = F.rng(F.SEED + kv_len)
    q = O.f16_bits(g.standard_normal(16 * 128, dtype=np.float32))
    k = O.f16_bits(g.standard_normal(2 * kv_len * 128, dtype=np.float32))
    v = O.f16_bits(g.standard_normal(2 * kv_len * 128, dtype=np.float32))
    scale = 1.0 / math.sqrt(128)
    exp = O.f16_to_f32(O.gqa_decode(q, k, v, O.F16, 16, 2, 128, kv_len, kv_len, scale))
    dq, dk, dv = dev(q), dev(k), dev(v)
    outs = {}
    for name, lib, h in _both(ref, kc_lib, kc_handle):
        out = dev(np.zeros(16 * 128, dtype=np.uint16))
        st = lib.kudacuda_qwen2_gqa_decode(h, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), 1, 1,
                                           kv_len, 16, 2, 128, scale, stream())
        assert st == 0, lib.kudacuda_last_error(h)
        outs[name] = O.f16_to_f32(host(out))
    for name in outs:
        err = np.abs(outs[name] - exp)
        assert np.all(err <= GQA_TOL + GQA_TOL * np.abs(exp)), f"{name} vs oracle: max {err.max():.3e}"


@pytest.mark.parametrize("entry", ["group_tiled", "vectorized", "graph", "workspace_v3"])
def test_reference_gqa_tactics_pin_the_oracle(ref, kc_lib, kc_handle, entry):
    kv_len = 37
    c = F.smoke_gqa_case(kv_len, O.F16)
    cap = 512 if entry in ("graph", "workspace_v3") else kv_len
    kc = np.zeros((2, cap, 128), dtype=np.uint16)
    vc = np.zeros((2, cap, 128), dtype=np.uint16)
    kc[:, :kv_len] = c["k"].reshape(2, kv_len, 128)
    vc[:, :kv_len] = c["v"].reshape(2, kv_len, 128)
    exp = O.f16_to_f32(O.gqa_decode(c["q"], np.ascontiguousarray(kc), np.ascontiguousarray(vc), O.F16, 16, 2, 128,
                                    kv_len, cap, float(c["scale"])))
    q, k, v = dev(c["q"]), dev(kc), dev(vc)
    kvl = dev(np.array([kv_len], dtype=np.int32))
    sc = float(c["scale"])
    for name, lib, h in _both(ref, kc_lib, kc_handle):
        out = dev(np.zeros(16 * 128, dtype=np.uint16))
        s = stream()
        if entry == "group_tiled":
            st = lib.kudacuda_qwen2_gqa_decode_group_tiled(h, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                           out.data_ptr(), 1, 1, kv_len, 16, 2, 128, sc, s)
        elif entry == "vectorized":
            st = lib.kudacuda_qwen2_gqa_decode_vectorized(h, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                          out.data_ptr(), 1, 1, kv_len, 16, 2, 128, sc, s)
        elif entry == "graph":
            st = lib.kudacuda_qwen2_gqa_decode_graph(h, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                                     1, 1, cap, 16, 2, 128, sc, kvl.data_ptr(), s)
        else:
            ws = dev(np.zeros(16 * 8 * 130, dtype=np.float32))
            st = lib.kudacuda_qwen2_gqa_decode_workspace_v3(h, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                            out.data_ptr(), ws.data_ptr(), kvl.data_ptr(), 1, 1, cap,
                                                            16, 2, 128, sc, s)
        assert st == 0, lib.kudacuda_last_error(h)
        got = O.f16_to_f32(host(out))
        err = np.abs(got - exp)
        assert np.all(err <= GQA_TOL + GQA_TOL * np.abs(exp)), f"{name} {entry} vs oracle: max {err.max():.3e}"
