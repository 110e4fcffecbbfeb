"""GPU parity of the persistent decode path (kudacuda_sm100_nf4_retile and
kudacuda_sm100_decode_layers_persistent, through the C ABI via the bridge).

* the device re-tile against the oracle's numpy restatement, bit-exact, for
  the plain, SwiGLU and q/k/v (RoPE-pair) layouts;
* whole decoder layers against the oracle's kc_layer_step_hf chain
  (norm-wise tolerance, the same bar as the per-op path);
* graph replay against eager execution and repeated steps: bit-identical
  (the cross-CTA sums have a fixed order);
* greedy decode: teacher-forced top-1 agreement with the oracle, and the
  device error word stays clear (no bounded wait ran out).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.test_gpu_decode import _b16, _layer_np, norm_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny_persistent():
    import torch

    from kudacuda_b200.decode_engine import StaticDecodePlan, random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    torch.cuda.set_device(0)
    cfg = tiny_config(layers=2, vocab=4096)
    bridge = KudaCudaBridge(device_id=0)
    weights = random_weights(bridge, cfg, seed=11, device="cuda:0")
    plan = StaticDecodePlan(bridge, weights, kv_bucket=64, max_tokens=64, device="cuda:0", persistent=True)
    stream = torch.cuda.Stream()
    plan.capture(stream)
    assert plan.launches_per_step == 4
    yield cfg, bridge, weights, plan, stream
    bridge.reset_graph()
    bridge.shutdown()


@pytest.mark.parametrize("which", ["qkv", "o", "gate_up", "down"])
def test_device_retile16_matches_oracle(tiny_persistent, which):
    """The row-split layout (default): 576-byte units, bit-exact."""

    cfg, bridge, w, plan, stream = tiny_persistent
    assert plan.persistent.layout == "rows"
    L = w.layers[1]
    idx = {"qkv": 0, "o": 1, "gate_up": 2, "down": 3}[which]
    (units,) = plan.persistent.tiles[4 + idx]  # layer 1
    mode, lins = {
        "qkv": (O.RETILE_QKV_ROPE, [L.q, L.k, L.v]),
        "o": (O.RETILE_PLAIN, [L.o]),
        "gate_up": (O.RETILE_SWIGLU, [L.gate, L.up]),
        "down": (O.RETILE_PLAIN, [L.down]),
    }[which]
    mats = [(lin.packed.reshape(-1).cpu().numpy(), lin.absmax.cpu().numpy(), lin.rows) for lin in lins]
    np.testing.assert_array_equal(units.cpu().numpy(), O.retile_tiles16(mode, mats, lins[0].k, cfg.head_dim))


@pytest.fixture(scope="module")
def tiny_groups():
    import torch

    from kudacuda_b200.decode_engine import StaticDecodePlan, random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    cfg = tiny_config(layers=2, vocab=4096)
    bridge = KudaCudaBridge(device_id=0)
    weights = random_weights(bridge, cfg, seed=11, device="cuda:0")
    plan = StaticDecodePlan(bridge, weights, kv_bucket=64, max_tokens=64, device="cuda:0", persistent=True,
                            persistent_layout="groups")
    stream = torch.cuda.Stream()
    plan.capture(stream)
    yield cfg, bridge, weights, plan, stream
    bridge.reset_graph()
    bridge.shutdown()


@pytest.mark.parametrize("which", ["qkv", "o", "gate_up", "down"])
def test_device_retile_matches_oracle(tiny_groups, which):
    """The K-split group layout (kudacuda_sm100_decode_layers_persistent)."""

    cfg, bridge, w, plan, stream = tiny_groups
    L = w.layers[1]
    idx = {"qkv": 0, "o": 1, "gate_up": 2, "down": 3}[which]
    codes, absm = plan.persistent.tiles[4 + idx]  # layer 1
    np_mats = {
        "qkv": (O.RETILE_QKV_ROPE, [L.q, L.k, L.v]),
        "o": (O.RETILE_PLAIN, [L.o]),
        "gate_up": (O.RETILE_SWIGLU, [L.gate, L.up]),
        "down": (O.RETILE_PLAIN, [L.down]),
    }[which]
    mode, lins = np_mats
    mats = [(lin.packed.reshape(-1).cpu().numpy(), lin.absmax.cpu().numpy(), lin.rows) for lin in lins]
    ref_codes, ref_abs = O.retile_nf4(mode, mats, lins[0].k, cfg.head_dim)
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)
    np.testing.assert_array_equal(absm.cpu().numpy().view(np.uint32), ref_abs.view(np.uint32))


@pytest.fixture(scope="module")
def one_layer_persistent():
    import torch

    from kudacuda_b200.decode_engine import StaticDecodePlan, random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    cfg = tiny_config(layers=1, vocab=4096)
    bridge = KudaCudaBridge(device_id=0)
    weights = random_weights(bridge, cfg, seed=29, device="cuda:0")
    plan = StaticDecodePlan(bridge, weights, kv_bucket=128, max_tokens=128, device="cuda:0", persistent=True)
    stream = torch.cuda.Stream()
    plan.capture(stream)
    yield cfg, bridge, weights, plan, stream
    bridge.reset_graph()
    bridge.shutdown()


@pytest.mark.parametrize("pos", [0, 9, 100])
def test_persistent_layer_against_oracle(one_layer_persistent, pos):
    """One layer in a persistent launch against the oracle's layer, with random
    earlier cache rows at positions < pos (one layer: a two-layer random-init
    chain amplifies bf16 rounding differences past the element bound for the
    per-op path as much as for this one)."""

    import torch

    cfg, bridge, w, plan, stream = one_layer_persistent
    plan.reset_cache()
    rng = np.random.default_rng(pos + 3)
    kc0 = O.bf16_bits(rng.normal(0, 1, tuple(plan.buffers.kcache.shape)).astype(np.float32))
    vc0 = O.bf16_bits(rng.normal(0, 1, tuple(plan.buffers.vcache.shape)).astype(np.float32))
    plan.buffers.kcache.copy_(torch.from_numpy(kc0.view(np.int16)).view(torch.bfloat16).to(plan.device))
    plan.buffers.vcache.copy_(torch.from_numpy(vc0.view(np.int16)).view(torch.bfloat16).to(plan.device))
    plan.set_state(321, pos, stream)
    plan.replay(stream)
    stream.synchronize()
    assert bridge.error_word(clear=True) == 0
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    x = emb[321].copy()
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    kcs = [kc0[i].copy() for i in range(cfg.layers)]
    vcs = [vc0[i].copy() for i in range(cfg.layers)]
    for li, L in enumerate(w.layers):
        O.layer_step_hf(_layer_np(L), ocfg, x, kcs[li], vcs[li], plan.kv_bucket, pos, cos[pos], sin[pos])
    norm_close(O.bf16_to_f32(_b16(plan.buffers.x)), O.bf16_to_f32(x))
    # the appended rows (RoPE'd k, v) match the oracle's append to within a bf16 ulp
    kc_gpu, vc_gpu = _b16(plan.buffers.kcache), _b16(plan.buffers.vcache)
    for li in range(cfg.layers):
        for got, ref in ((kc_gpu[li][:, pos], kcs[li][:, pos]), (vc_gpu[li][:, pos], vcs[li][:, pos])):
            norm_close(O.bf16_to_f32(got), O.bf16_to_f32(ref))
        # rows before pos are untouched
        np.testing.assert_array_equal(kc_gpu[li][:, :pos], kc0[li][:, :pos])
    _, logits_ref = O.lm_head_argmax(x, _b16(w.final_norm), emb, cfg.eps, want_logits=True)
    norm_close(O.bf16_to_f32(_b16(plan.buffers.logits)), O.bf16_to_f32(logits_ref))


def test_persistent_graph_and_repeats_bit_identical(tiny_persistent):
    import torch

    cfg, bridge, w, plan, stream = tiny_persistent
    outs = []
    for mode in ("eager", "graph", "graph"):
        plan.reset_cache()
        plan.set_state(77, 3, stream)
        if mode == "eager":
            with torch.cuda.stream(stream):
                plan.record(int(stream.cuda_stream))
        else:
            plan.replay(stream)
        stream.synchronize()
        outs.append((_b16(plan.buffers.x).copy(), _b16(plan.buffers.logits).copy(),
                     _b16(plan.buffers.kcache).copy(), plan.buffers.state.cpu().numpy().copy()))
    for other in outs[1:]:
        for a, b in zip(outs[0], other):
            np.testing.assert_array_equal(a, b)
    assert bridge.error_word(clear=True) == 0


def test_persistent_greedy_teacher_forced_top1(tiny_persistent):
    from kudacuda_b200.decode_engine import greedy_generate

    cfg, bridge, w, plan, stream = tiny_persistent
    prompt = [5, 17, 300, 4000]
    n_new = 8
    toks = greedy_generate(plan, prompt, n_new, stream)
    assert bridge.error_word(clear=True) == 0
    seq = prompt + toks
    layers = [_layer_np(L) for L in w.layers]
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    fn = _b16(w.final_norm)
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    kcs = [np.zeros((cfg.kv_heads, plan.kv_bucket, cfg.head_dim), dtype=np.uint16) for _ in layers]
    vcs = [np.zeros_like(kcs[0]) for _ in layers]
    agree = 0
    for pos in range(len(seq) - 1):
        x = emb[seq[pos]].copy()
        for li, layer in enumerate(layers):
            O.layer_step_hf(layer, ocfg, x, kcs[li], vcs[li], plan.kv_bucket, pos, cos[pos], sin[pos])
        tok, _ = O.lm_head_argmax(x, fn, emb, cfg.eps)
        if pos >= len(prompt) - 1:
            agree += int(tok == seq[pos + 1])
    rate = agree / n_new
    assert rate >= 0.75, f"teacher-forced top-1 agreement {rate:.2f}"


def test_release_source_weights_keeps_the_step(tiny_persistent):
    """After the bitsandbytes copies are freed the persistent step (which
    streams its own re-tiled copy) gives the same tokens, and the memory
    comes back."""

    import torch

    from kudacuda_b200.decode_engine import StaticDecodePlan, random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge, NativeCudaError

    cfg, bridge0, w0, plan0, stream0 = tiny_persistent
    bridge = KudaCudaBridge(device_id=0)
    w = random_weights(bridge, tiny_config(layers=2, vocab=4096), seed=12, device="cuda:0")
    with pytest.raises(NativeCudaError):  # a per-op plan streams the source weights themselves
        StaticDecodePlan(bridge, w, kv_bucket=64, max_tokens=64, device="cuda:0").release_source_weights()
    plan = StaticDecodePlan(bridge, w, kv_bucket=64, max_tokens=64, device="cuda:0", persistent=True)
    stream = torch.cuda.Stream()
    plan.capture(stream)

    def tokens():
        out = []
        plan.reset_cache()
        tok = 42
        for pos in range(6):
            tok = plan.step_host(tok, pos, stream)
            out.append(tok)
        return out

    before = tokens()
    torch.cuda.synchronize()
    m0 = torch.cuda.memory_allocated()
    freed = plan.release_source_weights()
    torch.cuda.synchronize()
    assert freed > 0 and torch.cuda.memory_allocated() <= m0 - freed // 2
    assert tokens() == before
    assert bridge.error_word(clear=True) == 0
    bridge.reset_graph()
    bridge.shutdown()


def test_persistent_rejects_unsupported_shapes(tiny_persistent):
    from kudacuda_b200.kudacuda_sidecar import NativeCudaError

    cfg, bridge, w, plan, stream = tiny_persistent
    with pytest.raises(NativeCudaError):
        bridge.persistent_scratch_bytes(layers=2, hidden=2048, q_heads=16, kv_heads=2, head_dim=64,
                                        intermediate=11008, kv_capacity=64)
    assert bridge.retile_groups(O.RETILE_PLAIN, (100, 0, 0)) == -1
    assert bridge.retile_groups(O.RETILE_SWIGLU, (64, 96, 0)) == -1


def test_groups_layout_layer_against_oracle(tiny_groups):
    """The K-split persistent kernel (layout "groups") still computes a layer
    within the composed-output bound."""

    cfg, bridge, w, plan, stream = tiny_groups
    plan.reset_cache()
    plan.set_state(321, 0, stream)
    plan.replay(stream)
    stream.synchronize()
    assert bridge.error_word(clear=True) == 0
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    x = emb[321].copy()
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    for L in w.layers:
        kc = np.zeros((cfg.kv_heads, plan.kv_bucket, cfg.head_dim), dtype=np.uint16)
        vc = np.zeros_like(kc)
        O.layer_step_hf(_layer_np(L), ocfg, x, kc, vc, plan.kv_bucket, 0, cos[0], sin[0])
    norm_close(O.bf16_to_f32(_b16(plan.buffers.x)), O.bf16_to_f32(x))


@pytest.mark.gpu
def test_bound_host_step_matches_graph_step_host(tiny_persistent):
    """The pre-bound host step (buffers and stream resolved once, the form a
    decode loop uses) calls the same C entry as graph_step_host: the same
    tokens from the same start, also through the plan's step_host."""

    import torch

    cfg, bridge, w, plan, stream = tiny_persistent
    sp = int(stream.cuda_stream)

    def run(bound):
        plan.reset_cache()
        hi = torch.zeros(4, dtype=torch.int32).pin_memory()
        ho = torch.zeros(1, dtype=torch.int32).pin_memory()
        step = bridge.bind_graph_step_host(hi, plan.buffers.state, ho, plan.buffers.next_token, stream_ptr=sp)
        tok, out = 7, []
        for pos in range(5):
            hi[0], hi[1], hi[2] = tok, pos, pos + 1
            if bound:
                step()
            else:
                bridge.graph_step_host(hi, plan.buffers.state, ho, plan.buffers.next_token, stream_ptr=sp)
            tok = int(ho[0])
            out.append(tok)
        return out

    ref = run(False)
    assert run(True) == ref
    plan.reset_cache()
    got, tok = [], 7
    for pos in range(5):
        tok = plan.step_host(tok, pos, stream)
        got.append(tok)
    assert got == ref
    assert bridge.error_word(clear=True) == 0
