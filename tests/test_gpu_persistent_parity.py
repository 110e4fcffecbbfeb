"""Parity of the benched path itself -- the persistent all-layers kernel
(kudacuda_sm100_decode_layers_persistent, bench.py's default) -- at the
config-2 KV lengths, through the C ABI's test hooks.

* one Qwen2.5-3B-shaped layer at kv_len in {1, 7, 128, 512, 1024, 2048}
  (cache capacity 2048, random earlier rows; 2048 tokens run the kernel's
  widest attention plan, 32 splits of 64 tokens per KV head): every
  intermediate the kernel forms (RMSNorm, q/k/v after bias and RoPE, the
  attention output, x + o_proj, RMSNorm, SwiGLU, x + down) is read from the
  kernel's tap buffer and checked ELEMENT-WISE against the oracle fed the
  kernel's previous intermediate -- the bf16 chain bound of
  test_gpu_kernels.close_chain (2 ulps + one ulp per rounded intermediate +
  2e-3, and at most 1% of elements outside 1e-2 rel / 2e-3 abs), the
  reference's 3.5e-3 for attention;
* all 36 layers of the config-3 shapes in one launch at kv_len 512 and 2048:
  every layer's output x2 against the oracle's layer fed the kernel's input
  to that layer (norm-wise 1e-2, the composed-output bound), and the
  free-running 36-layer chain reported;
* the bounded-wait path: a dependency wait made unreachable with a short
  poll limit ends the step with bit 4 of the error word set, and the next
  normal step is bit-identical to one that never saw the stall.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import oracle as O
from tests.test_gpu_decode import _b16, _layer_np, norm_close
from tests.test_gpu_kernels import close, close_chain

pytestmark = pytest.mark.gpu

CAP = 2048
KV_LENS = [1, 7, 128, 512, 1024, 2048]


def _plan(layers, seed):
    import torch

    from kudacuda_b200.decode_engine import StaticDecodePlan, random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    torch.cuda.set_device(0)
    cfg = tiny_config(layers=layers, vocab=4096)
    bridge = KudaCudaBridge(device_id=0)
    w = random_weights(bridge, cfg, seed=seed, device="cuda:0")
    plan = StaticDecodePlan(bridge, w, kv_bucket=CAP, max_tokens=CAP, device="cuda:0", persistent=True)
    stream = torch.cuda.Stream()
    return cfg, bridge, w, plan, stream


@pytest.fixture(scope="module")
def one_layer():
    cfg, bridge, w, plan, stream = _plan(1, 20260824)
    yield cfg, bridge, w, plan, stream
    bridge.shutdown()


def _fill_cache(plan, pos, seed):
    """Random N(0,1) bf16 rows before ``pos`` in every layer's K/V cache; host copies."""

    import torch

    rng = np.random.default_rng(seed)
    shape = tuple(plan.buffers.kcache.shape)
    kc = O.bf16_bits(rng.normal(0, 1, shape).astype(np.float32))
    vc = O.bf16_bits(rng.normal(0, 1, shape).astype(np.float32))
    kc[:, :, pos:] = 0
    vc[:, :, pos:] = 0
    plan.buffers.kcache.copy_(torch.from_numpy(kc.view(np.int16)).view(torch.bfloat16).to(plan.device))
    plan.buffers.vcache.copy_(torch.from_numpy(vc.view(np.int16)).view(torch.bfloat16).to(plan.device))
    torch.cuda.synchronize()
    return kc, vc


def _step(plan, bridge, w, stream, token, pos, taps=None, **hooks):
    """Embedding row + one persistent launch at ``pos`` (kv_len = pos + 1)."""

    import torch

    plan.set_state(token, pos, stream)
    sp = int(stream.cuda_stream)
    with torch.cuda.stream(stream):
        bridge.dispatch_embedding(w.embedding, plan.buffers.state[0:1], plan.buffers.x, stream_ptr=sp)
        plan.persistent.record(sp, taps=taps, **hooks)
    stream.synchronize()


def _lin_ref(x_bits, lin_np, rows, k, bias=None):
    y = O.bf16_bits(O.nf4_gemv(O.bf16_to_f32(x_bits), lin_np[0], lin_np[1], rows, k))
    if bias is not None:
        y = O.bf16_bits(O.bf16_to_f32(y) + O.bf16_to_f32(bias))
    return y


@pytest.mark.parametrize("kv_len", KV_LENS)
def test_persistent_layer_stages_elementwise(one_layer, kv_len):
    cfg, bridge, w, plan, stream = one_layer
    pos = kv_len - 1
    kc0, vc0 = _fill_cache(plan, pos, seed=kv_len)
    taps = plan.persistent.new_taps()
    token = 321 + kv_len
    _step(plan, bridge, w, stream, token, pos, taps=taps)
    assert bridge.error_word(clear=True) == 0
    lay = plan.persistent.tap_layout()
    t = _b16(taps)

    def tap(name):
        off, n = lay[name]
        return t[off:off + n].copy()

    d, qh, kvh, H, I = cfg.head_dim, cfg.q_heads, cfg.kv_heads, cfg.hidden, cfg.intermediate
    Lnp = _layer_np(w.layers[0])
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    x0 = _b16(w.embedding[token]).copy()

    xn = tap("xn")
    close_chain(O.bf16_to_f32(xn), O.bf16_to_f32(O.rmsnorm_hf_bf16(x0, Lnp["in_norm"], cfg.eps)))
    q_lin = _lin_ref(xn, Lnp["q"], qh * d, H, Lnp["q_b"])
    k_lin = _lin_ref(xn, Lnp["k"], kvh * d, H, Lnp["k_b"])
    v_lin = _lin_ref(xn, Lnp["v"], kvh * d, H, Lnp["v_b"])
    q_ref = O.rope_hf_bf16(q_lin, qh, d, cos[pos], sin[pos])
    k_ref = O.rope_hf_bf16(k_lin, kvh, d, cos[pos], sin[pos])
    qm = np.abs(O.bf16_to_f32(q_lin)).reshape(qh, 2, 64).max(axis=1).repeat(2, axis=0).reshape(-1)
    km = np.abs(O.bf16_to_f32(k_lin)).reshape(kvh, 2, 64).max(axis=1).repeat(2, axis=0).reshape(-1)
    q, k, v = tap("q"), tap("k"), tap("v")
    close_chain(O.bf16_to_f32(q), O.bf16_to_f32(q_ref), intermediates=(qm, qm, qm))
    close_chain(O.bf16_to_f32(k), O.bf16_to_f32(k_ref), intermediates=(km, km, km))
    close_chain(O.bf16_to_f32(v), O.bf16_to_f32(v_lin))

    # the cache: row pos holds this step's k/v, earlier rows untouched
    kc, vc = _b16(plan.buffers.kcache)[0], _b16(plan.buffers.vcache)[0]
    np.testing.assert_array_equal(kc[:, pos].reshape(-1), k)
    np.testing.assert_array_equal(vc[:, pos].reshape(-1), v)
    np.testing.assert_array_equal(kc[:, :pos], kc0[0][:, :pos])
    np.testing.assert_array_equal(vc[:, :pos], vc0[0][:, :pos])

    att = tap("att")
    att_ref = O.gqa_decode(q, np.ascontiguousarray(kc), np.ascontiguousarray(vc), O.BF16, qh, kvh, d, kv_len, CAP,
                           1.0 / math.sqrt(d))
    close(O.bf16_to_f32(att), O.bf16_to_f32(att_ref), atol=3.5e-3, rtol=3.5e-3)

    x1 = tap("x1")
    o_ref = _lin_ref(att, Lnp["o"], H, qh * d)
    close_chain(O.bf16_to_f32(x1), O.bf16_to_f32(O.bf16_bits(O.bf16_to_f32(x0) + O.bf16_to_f32(o_ref))),
                intermediates=(O.bf16_to_f32(o_ref),))
    xn2 = tap("xn2")
    close_chain(O.bf16_to_f32(xn2), O.bf16_to_f32(O.rmsnorm_hf_bf16(x1, Lnp["post_norm"], cfg.eps)))
    gref = O.bf16_to_f32(_lin_ref(xn2, Lnp["gate"], I, H))
    uref = O.bf16_to_f32(_lin_ref(xn2, Lnp["up"], I, H))
    act = O.bf16_to_f32(O.bf16_bits(gref / (1.0 + np.exp(-gref))))
    h = tap("h")
    close_chain(O.bf16_to_f32(h), O.bf16_to_f32(O.bf16_bits(act * uref)), intermediates=(gref, uref, act))
    x2 = tap("x2")
    d_ref = _lin_ref(h, Lnp["down"], H, I)
    close_chain(O.bf16_to_f32(x2), O.bf16_to_f32(O.bf16_bits(O.bf16_to_f32(x1) + O.bf16_to_f32(d_ref))),
                intermediates=(O.bf16_to_f32(d_ref),))
    np.testing.assert_array_equal(_b16(plan.buffers.x), x2)  # the step's output is the last tap


@pytest.fixture(scope="module")
def full_depth():
    cfg, bridge, w, plan, stream = _plan(36, 20260825)
    yield cfg, bridge, w, plan, stream
    bridge.shutdown()


@pytest.mark.parametrize("kv_len", [512, 2048])
def test_persistent_36_layers_per_layer_norm_wise(full_depth, kv_len):
    cfg, bridge, w, plan, stream = full_depth
    pos = kv_len - 1
    kc0, vc0 = _fill_cache(plan, pos, seed=1000 + kv_len)
    taps = plan.persistent.new_taps()
    token = 77
    _step(plan, bridge, w, stream, token, pos, taps=taps)
    assert bridge.error_word(clear=True) == 0
    lay = plan.persistent.tap_layout()
    stride = lay["stride"][0]
    t = _b16(taps).reshape(cfg.layers, stride)
    x2_off = lay["x2"][0]
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    x_gpu_in = _b16(w.embedding[token]).copy()
    x_free = x_gpu_in.copy()
    worst = 0.0
    for li, L in enumerate(w.layers):
        layer = _layer_np(L)
        # teacher-forced: the oracle layer on the kernel's own input to this layer
        x = x_gpu_in.copy()
        kc, vc = kc0[li].copy(), vc0[li].copy()
        O.layer_step_hf(layer, ocfg, x, kc, vc, CAP, pos, cos[pos], sin[pos])
        got = t[li, x2_off:x2_off + cfg.hidden].copy()
        a, e = O.bf16_to_f32(got), O.bf16_to_f32(x)
        worst = max(worst, float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30)))
        norm_close(a, e)
        # free-running chain (reported)
        kcf, vcf = kc0[li].copy(), vc0[li].copy()
        O.layer_step_hf(layer, ocfg, x_free, kcf, vcf, CAP, pos, cos[pos], sin[pos])
        x_gpu_in = got
    np.testing.assert_array_equal(_b16(plan.buffers.x), x_gpu_in)
    free = float(np.linalg.norm(O.bf16_to_f32(x_gpu_in) - O.bf16_to_f32(x_free)) /
                 np.linalg.norm(O.bf16_to_f32(x_free)))
    print(f"kv {kv_len}: worst per-layer norm-wise error {worst:.3e}; free-running 36-layer chain {free:.3e}")
    assert np.all(np.isfinite(O.bf16_to_f32(x_gpu_in)))


def test_persistent_bounded_wait_runs_out_and_recovers(one_layer):
    cfg, bridge, w, plan, stream = one_layer
    pos = 99
    _fill_cache(plan, pos, seed=5)
    _step(plan, bridge, w, stream, 11, pos)
    assert bridge.error_word(clear=True) == 0
    clean = _b16(plan.buffers.x).copy()
    # the attention -> o_proj wait of layer 0 can never complete: it gives up
    # after 4096 polls, raises the step's abort flag and error bit 4
    _fill_cache(plan, pos, seed=5)
    _step(plan, bridge, w, stream, 11, pos, spin_limit=4096, stall_counter=1)
    assert bridge.error_word(clear=True) & 16
    # the counters and the abort flag reset themselves: the next step is normal
    _fill_cache(plan, pos, seed=5)
    _step(plan, bridge, w, stream, 11, pos)
    assert bridge.error_word(clear=True) == 0
    np.testing.assert_array_equal(_b16(plan.buffers.x), clean)
