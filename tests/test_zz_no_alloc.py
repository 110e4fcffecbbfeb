"""GPU test of the allocation-free GQA entry point, kudacuda_sm100_gqa_decode_static.

It must give the same result as kudacuda_sm100_gqa_decode (caller workspace
and tickets) on two calls in a row: the second call checks that the fixed
scratch's tickets reset themselves.  At 3000 tokens both entry points run the
same split-KV kernel with the same plan, so outputs are bit-identical; at 517
tokens the workspace entry takes the cluster kernel, so the two agree within
the attention tolerance and both match the CPU oracle.  The file name sorts
last so it also runs after every other GPU test (and passes alone).
"""

import math

import numpy as np
import pytest

from tests import fixtures as F

pytestmark = pytest.mark.gpu

_LIVE = []
GQA_TOL = 2e-3  # absolute and relative, bf16 outputs (north-star attention tolerance)


def _dev(a):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")
    _LIVE.append(t)
    return t


def _host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def _stream():
    import torch

    return int(torch.cuda.current_stream().cuda_stream)


def _ok(lib, h, status):
    assert status == 0, lib.kudacuda_last_error(h)


@pytest.mark.parametrize("kv_len", [3000, 517])
def test_static_scratch_gqa_matches_workspace_entry(kc_lib, kc_handle, oracle_mod, kv_len):
    O = oracle_mod
    g = F.rng(900 + kv_len)
    q_heads, kv_heads, d, batch = 16, 2, 128, 1
    kc = F.bf16_normal(g, kv_heads * kv_len * d)
    vc = F.bf16_normal(g, kv_heads * kv_len * d)
    dk, dv = _dev(kc), _dev(vc)
    scale = 1.0 / math.sqrt(d)
    nbytes = kc_lib.kudacuda_sm100_gqa_workspace_bytes(batch, q_heads, kv_heads, kv_len, d)
    ws = _dev(np.zeros(nbytes // 4, dtype=np.float32))
    tickets = _dev(np.zeros(batch * kv_heads, dtype=np.int32))
    for call in range(2):  # two calls in a row, different queries
        q = F.bf16_normal(g, q_heads * d)
        dq = _dev(q)
        out_static = _dev(np.zeros(q_heads * d, dtype=np.uint16))
        out_ws = _dev(np.zeros(q_heads * d, dtype=np.uint16))
        _ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_gqa_decode_static(
            kc_handle, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out_static.data_ptr(), 0, O.BF16, batch,
            kv_len, kv_len, q_heads, kv_heads, d, scale, _stream()))
        _ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_gqa_decode(
            kc_handle, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out_ws.data_ptr(), ws.data_ptr(), nbytes,
            tickets.data_ptr(), 0, O.BF16, batch, kv_len, kv_len, q_heads, kv_heads, d, scale, _stream()))
        got_static, got_ws = _host(out_static), _host(out_ws)
        if kv_len > 2048:
            assert np.array_equal(got_static, got_ws), f"call {call}: static scratch differs from workspace entry"
        ref = O.gqa_decode(q, kc, vc, O.BF16, q_heads, kv_heads, d, kv_len, kv_len, scale)
        a = O.bf16_to_f32(got_static)
        np.testing.assert_allclose(a, O.bf16_to_f32(got_ws), atol=GQA_TOL, rtol=GQA_TOL)
        np.testing.assert_allclose(a, O.bf16_to_f32(ref), atol=GQA_TOL, rtol=GQA_TOL)
    assert int(_host(tickets).sum()) == 0


def test_static_scratch_gqa_device_length_and_batch(kc_lib, kc_handle, oracle_mod):
    """kv_len_device given (the extent is the stride) and batch 2 (one ticket
    per (sequence, KV head)): two calls in a row, each against the workspace
    entry (same split plan: bit-identical) and the oracle per sequence."""

    import torch

    O = oracle_mod
    g = F.rng(4242)
    q_heads, kv_heads, d, batch, stride = 16, 2, 128, 2, 2304
    kc = F.bf16_normal(g, batch * kv_heads * stride * d)
    vc = F.bf16_normal(g, batch * kv_heads * stride * d)
    dk, dv = _dev(kc), _dev(vc)
    scale = 1.0 / math.sqrt(d)
    nbytes = kc_lib.kudacuda_sm100_gqa_workspace_bytes(batch, q_heads, kv_heads, stride, d)
    ws = _dev(np.zeros(nbytes // 4, dtype=np.float32))
    tickets = _dev(np.zeros(batch * kv_heads, dtype=np.int32))
    for call, kv_len in enumerate((2200, 1501)):
        dlen = _dev(np.array([kv_len], dtype=np.int32))
        q = F.bf16_normal(g, batch * q_heads * d)
        dq = _dev(q)
        out_static = _dev(np.zeros(batch * q_heads * d, dtype=np.uint16))
        out_ws = _dev(np.zeros(batch * q_heads * d, dtype=np.uint16))
        _ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_gqa_decode_static(
            kc_handle, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out_static.data_ptr(), dlen.data_ptr(), O.BF16,
            batch, 0, stride, q_heads, kv_heads, d, scale, _stream()))
        # the workspace entry with split-KV forced: the same plan over the stride
        _ok(kc_lib, kc_handle, kc_lib.kudacuda_sm100_gqa_decode(
            kc_handle, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out_ws.data_ptr(), ws.data_ptr(), nbytes,
            tickets.data_ptr(), dlen.data_ptr(), O.BF16, batch, 0, stride, q_heads, kv_heads, d, scale, _stream()))
        got_static, got_ws = _host(out_static), _host(out_ws)
        assert np.array_equal(got_static, got_ws), f"call {call}: static scratch differs from workspace entry"
        qs = q.reshape(batch, q_heads * d)
        kcs = kc.reshape(batch, kv_heads * stride * d)
        vcs = vc.reshape(batch, kv_heads * stride * d)
        for b in range(batch):
            ref = O.gqa_decode(qs[b], kcs[b], vcs[b], O.BF16, q_heads, kv_heads, d, kv_len, stride, scale)
            got = O.bf16_to_f32(got_static.reshape(batch, -1)[b])
            np.testing.assert_allclose(got, O.bf16_to_f32(ref), atol=GQA_TOL, rtol=GQA_TOL)
    torch.cuda.synchronize()
    assert int(_host(tickets).sum()) == 0


def test_static_scratch_gqa_rejects_oversized_requests(kc_lib, kc_handle, oracle_mod):
    # 64 query heads x 8 kv heads x batch 8 needs more partials than the fixed 1 MiB array holds
    O = oracle_mod
    q_heads, kv_heads, d, batch, kv_len = 64, 8, 128, 8, 4096
    q = _dev(np.zeros(batch * q_heads * d, dtype=np.uint16))
    kv = _dev(np.zeros(batch * kv_heads * kv_len * d, dtype=np.uint16))
    out = _dev(np.zeros(batch * q_heads * d, dtype=np.uint16))
    status = kc_lib.kudacuda_sm100_gqa_decode_static(
        kc_handle, q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), 0, O.BF16, batch, kv_len, kv_len,
        q_heads, kv_heads, d, 0.088, _stream())
    assert status == 1
    assert b"fixed scratch" in kc_lib.kudacuda_last_error(kc_handle)
