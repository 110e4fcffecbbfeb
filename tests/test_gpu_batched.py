"""GPU parity of the batched decode path (B independent sequences per step),
through the C ABI via the bridge.

* the device re-tile (kudacuda_sm100_batch_retile) against the oracle's numpy
  restatement, bit-exact;
* the tcgen05 GEMM (kudacuda_sm100_batch_gemm) against the oracle's batched
  projection (bf16-dequantised NF4 times bf16 activations, exact in float64):
  every element within 1e-4 of the sum of |w * x| (fp32 accumulation over up
  to 11008 terms), padded batch columns exactly zero, rows of the shared
  partials buffer outside the matrix untouched;
* one whole batched step against the oracle's per-sequence layer, with every
  sequence at its own position over its own random cache (norm-wise 1e-2);
* graph replay against eager execution: bit-identical (fixed split order);
* ragged-prompt greedy decode: teacher-forced top-1 agreement.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests.test_gpu_decode import _b16, _layer_np, norm_close

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bridge():
    import torch

    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    torch.cuda.set_device(0)
    br = KudaCudaBridge(device_id=0)
    yield br
    br.shutdown()


@pytest.mark.parametrize(
    "rows,k,batch,n_pad,ksplit,weight_type",
    [
        (128, 64, 16, 16, 1, 0),      # one tile, one K block
        (300, 256, 5, 16, 1, 0),      # ragged M tile, one split
        (300, 2048, 20, 32, 3, 0),    # uneven split of 32 K blocks
        (2560, 2048, 64, 64, 0, 0),   # q|k|v rows, full batch, suggested split
        (2048, 11008, 33, 64, 0, 0),  # down_proj shape
        (1000, 512, 3, 16, 2, 1),     # bf16 weights (lm_head form)
        (300, 256, 5, 16, 1, 2),      # re-tiled NF4, ragged last tile
        (2560, 2048, 64, 64, 0, 2),   # re-tiled q|k|v
        (2048, 11008, 40, 64, 0, 2),  # re-tiled down_proj
        (4352, 2048, 30, 32, 3, 2),   # re-tiled, n_pad 32, uneven split
    ],
)
def test_batch_gemm_against_oracle(bridge, rows, k, batch, n_pad, ksplit, weight_type):
    import torch

    dev = "cuda:0"
    g = torch.Generator(device="cpu").manual_seed(rows * 7 + k + batch)
    w = (torch.randn((rows, k), generator=g) * 0.02).to(torch.bfloat16)
    x = torch.zeros((n_pad, k), dtype=torch.bfloat16)
    x[:batch] = torch.randn((batch, k), generator=g).to(torch.bfloat16)
    if weight_type in (0, 2):
        packed, absmax = O.nf4_quantize(O.bf16_to_f32(w.view(torch.int16).numpy().view(np.uint16)).reshape(-1))
        wd = torch.from_numpy(np.ascontiguousarray(packed)).to(dev)
        ad = torch.from_numpy(np.ascontiguousarray(absmax)).to(dev)
        if weight_type == 2:
            rt = torch.empty(bridge.batch_retile_bytes(rows, k), dtype=torch.uint8, device=dev)
            bridge.dispatch_batch_retile(wd, ad, rt, rows=rows, k=k, stream_ptr=0)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(rt.cpu().numpy(), O.batch_retile(packed, absmax, rows, k))
            wd, ad = rt, None
    else:
        packed, absmax = w.view(torch.int16).numpy().view(np.uint16), None
        wd, ad = w.to(dev), None
    if ksplit == 0:
        ksplit = bridge.batch_gemm_ksplit(rows, k)
    assert 1 <= ksplit <= k // 64
    total = rows + 40  # the matrix sits at row_offset 17 inside a larger partials buffer
    sentinel = 12345.0
    part = torch.full((ksplit * total * n_pad,), sentinel, dtype=torch.float32, device=dev)
    xd = x.to(dev)
    s = torch.cuda.Stream()
    bridge.dispatch_batch_gemm(wd, ad, xd, part, weight_type=weight_type, rows=rows, k=k, n_pad=n_pad, ksplit=ksplit,
                               row_offset=17, total_rows=total, stream_ptr=int(s.cuda_stream))
    s.synchronize()
    assert bridge.error_word(clear=True) == 0
    p = part.view(ksplit, total, n_pad).cpu().numpy().astype(np.float64)
    assert np.all(p[:, :17] == sentinel) and np.all(p[:, 17 + rows:] == sentinel)
    got = p[:, 17:17 + rows].sum(axis=0)
    ref, mag = O.batch_gemm_ref(packed, absmax, rows, k, x.view(torch.int16).numpy().view(np.uint16),
                                weight_type=min(weight_type, 1) if weight_type != 2 else 0)
    assert np.all(got[:, batch:] == 0.0)
    err = np.abs(got - ref)
    bound = 1e-4 * mag + 1e-6
    worst = np.unravel_index(np.argmax(err / bound), err.shape)
    assert np.all(err <= bound), f"row {worst[0]} seq {worst[1]}: {got[worst]} vs {ref[worst]}"


@pytest.fixture(scope="module")
def batched_one_layer(bridge):
    import torch

    from kudacuda_b200.decode_engine import BatchedDecodePlan, random_weights, tiny_config

    cfg = tiny_config(layers=1, vocab=4096)
    weights = random_weights(bridge, cfg, seed=31, device="cuda:0")
    plan = BatchedDecodePlan(bridge, weights, batch=5, kv_bucket=128, max_tokens=128, device="cuda:0")
    stream = torch.cuda.Stream()
    plan.capture(stream)
    yield cfg, weights, plan, stream
    bridge.reset_graph()


def test_batched_step_against_oracle_per_sequence(bridge, batched_one_layer):
    """Five sequences at positions 0, 9, 100, 37, 126 over their own random caches."""

    import torch

    cfg, w, plan, stream = batched_one_layer
    positions = [0, 9, 100, 37, 126]
    tokens = [321, 5, 4095, 77, 1000]
    plan.reset_cache()
    rng = np.random.default_rng(41)
    shape = tuple(plan.buffers.kcache.shape)
    kc0 = O.bf16_bits(rng.normal(0, 1, shape).astype(np.float32))
    vc0 = O.bf16_bits(rng.normal(0, 1, shape).astype(np.float32))
    plan.buffers.kcache.copy_(torch.from_numpy(kc0.view(np.int16)).view(torch.bfloat16).to(plan.device))
    plan.buffers.vcache.copy_(torch.from_numpy(vc0.view(np.int16)).view(torch.bfloat16).to(plan.device))
    plan.set_state(tokens, positions, stream)
    plan.replay(stream)
    stream.synchronize()
    assert bridge.error_word(clear=True) == 0
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    layer = _layer_np(w.layers[0])
    xs = _b16(plan.buffers.x)
    kc_gpu, vc_gpu = _b16(plan.buffers.kcache), _b16(plan.buffers.vcache)
    state = plan.buffers.state.cpu().numpy()
    fn = _b16(w.final_norm)
    for b, (tok, pos) in enumerate(zip(tokens, positions)):
        x = emb[tok].copy()
        kc, vc = kc0[0, b].copy(), vc0[0, b].copy()
        O.layer_step_hf(layer, ocfg, x, kc, vc, plan.kv_bucket, pos, cos[pos], sin[pos])
        # the batched path rounds every dequantised weight to bf16 (the
        # Transformers + bitsandbytes arithmetic) where the oracle's layer keeps
        # them fp32 (the reference kernels'): a few elements of the composed
        # layer output differ by ~3 bf16 ulps, so the element bound is 2e-2
        # of the largest value; the norm-wise bound stays 1e-2
        norm_close(O.bf16_to_f32(xs[b]), O.bf16_to_f32(x), elem_rel=2e-2)
        norm_close(O.bf16_to_f32(kc_gpu[0, b][:, pos]), O.bf16_to_f32(kc[:, pos]))
        norm_close(O.bf16_to_f32(vc_gpu[0, b][:, pos]), O.bf16_to_f32(vc[:, pos]))
        np.testing.assert_array_equal(kc_gpu[0, b][:, :pos], kc0[0, b][:, :pos])
        np.testing.assert_array_equal(kc_gpu[0, b][:, pos + 1:], kc0[0, b][:, pos + 1:])
        assert list(state[b][1:3]) == [pos + 1, pos + 2]
        ref_tok, logits = O.lm_head_argmax(x, fn, emb, cfg.eps, want_logits=True)
        if ref_tok != state[b][0]:  # a near-tie may flip by a rounding step
            lf = O.bf16_to_f32(logits)
            assert lf[state[b][0]] >= lf[ref_tok] - 2e-2 * abs(lf[ref_tok]) - 2e-3


def test_batched_graph_matches_eager_bit_identical(bridge, batched_one_layer):
    import torch

    cfg, w, plan, stream = batched_one_layer
    outs = []
    for mode in ("eager", "graph", "graph"):
        plan.reset_cache()
        plan.set_state([1, 2, 3, 4, 5], [3, 0, 7, 1, 2], stream)
        if mode == "eager":
            with torch.cuda.stream(stream):
                plan.record(int(stream.cuda_stream))
        else:
            plan.replay(stream)
        stream.synchronize()
        outs.append((_b16(plan.buffers.x).copy(), _b16(plan.buffers.kcache).copy(),
                     plan.buffers.state.cpu().numpy().copy()))
    for other in outs[1:]:
        for a, b in zip(outs[0], other):
            np.testing.assert_array_equal(a, b)
    assert bridge.error_word(clear=True) == 0


def test_batched_greedy_ragged_prompts_teacher_forced(bridge):
    import torch

    from kudacuda_b200.decode_engine import BatchedDecodePlan, batched_greedy_generate, random_weights, tiny_config

    cfg = tiny_config(layers=2, vocab=4096)
    w = random_weights(bridge, cfg, seed=13, device="cuda:0")
    plan = BatchedDecodePlan(bridge, w, batch=3, kv_bucket=64, max_tokens=64, device="cuda:0")
    stream = torch.cuda.Stream()
    plan.capture(stream)
    prompts = [[5, 17, 300, 4000], [9], [1, 2, 3, 4, 5, 6]]
    n_new = 6
    outs = batched_greedy_generate(plan, prompts, n_new, stream)
    assert bridge.error_word(clear=True) == 0
    layers = [_layer_np(L) for L in w.layers]
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    fn = _b16(w.final_norm)
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    agree, total = 0, 0
    for prompt, gen in zip(prompts, outs):
        assert len(gen) == n_new
        seq = prompt + gen
        kcs = [np.zeros((cfg.kv_heads, plan.kv_bucket, cfg.head_dim), dtype=np.uint16) for _ in layers]
        vcs = [np.zeros_like(kcs[0]) for _ in layers]
        for pos in range(len(seq) - 1):
            x = emb[seq[pos]].copy()
            for li, layer in enumerate(layers):
                O.layer_step_hf(layer, ocfg, x, kcs[li], vcs[li], plan.kv_bucket, pos, cos[pos], sin[pos])
            tok, _ = O.lm_head_argmax(x, fn, emb, cfg.eps)
            if pos >= len(prompt) - 1:
                agree += int(tok == seq[pos + 1])
                total += 1
    rate = agree / total
    assert rate >= 0.75, f"teacher-forced top-1 agreement {rate:.2f}"
    bridge.reset_graph()


def test_batched_rejects_bad_arguments(bridge):
    import torch

    from kudacuda_b200.kudacuda_sidecar import NativeCudaError

    x = torch.zeros((16, 128), dtype=torch.bfloat16, device="cuda:0")
    w = torch.zeros((128, 128), dtype=torch.bfloat16, device="cuda:0")
    part = torch.zeros(16 * 128 * 4, dtype=torch.float32, device="cuda:0")
    with pytest.raises(NativeCudaError):  # n_pad 8 is not a supported N here
        bridge.dispatch_batch_gemm(w, None, x[:8], part, weight_type=1, rows=128, k=128, n_pad=8, ksplit=1,
                                   stream_ptr=0)
    with pytest.raises(NativeCudaError):  # ksplit above K/64
        bridge.dispatch_batch_gemm(w, None, x, part, weight_type=1, rows=128, k=128, n_pad=16, ksplit=3,
                                   stream_ptr=0)
    with pytest.raises(ValueError):
        bridge.batch_argmax_workspace_bytes(65)


def test_batch_tp_pieces_exact(bridge):
    """The tensor-parallel pieces: split sums in split order, per-sequence
    argmax pairs with a rank's index base, and the select over ranks (lowest
    index on ties) with the state advance."""

    import torch

    dev = "cuda:0"
    rng = np.random.default_rng(3)
    ks, rows, npad, batch, vocab, world = 3, 300, 32, 20, 1000, 3
    part = torch.from_numpy(rng.normal(0, 1, (ks, rows, npad)).astype(np.float32)).to(dev)
    out = torch.zeros(rows * npad, dtype=torch.float32, device=dev)
    bridge.dispatch_batch_split_sum(part, out, ksplit=ks, rows=rows, n_pad=npad, stream_ptr=0)
    p = part.cpu().numpy()
    ref = (p[0] + p[1]) + p[2]
    np.testing.assert_array_equal(out.view(rows, npad).cpu().numpy(), ref)
    # argmax pairs over a vocabulary slice with planted ties
    logits = rng.normal(0, 1, (1, vocab, npad)).astype(np.float32)
    logits[0, 700, :batch] = 9.0
    logits[0, 200, 3] = 9.0  # tie for sequence 3: the lower index wins
    lt = torch.from_numpy(logits).to(dev)
    ws = torch.zeros(bridge.batch_argmax_workspace_bytes(batch) // 4, dtype=torch.float32, device=dev)
    pairs = torch.zeros((batch, 2), dtype=torch.int32, device=dev)
    bridge.dispatch_batch_argmax_pairs(lt, ws, pairs, ksplit=1, vocab=vocab, n_pad=npad, batch=batch,
                                       index_base=5000, stream_ptr=0)
    pr = pairs.cpu().numpy()
    assert pr[3, 1] == 5200 and all(pr[b, 1] == 5700 for b in range(batch) if b != 3)
    assert np.all(pr[:, 0].view(np.float32) == 9.0)
    # select over three ranks' pairs, then the state advance
    g = np.zeros((world, batch, 2), dtype=np.int32)
    vals = rng.normal(0, 1, (world, batch)).astype(np.float32)
    vals[2, 4] = vals[0, 4] = 50.0  # tie across ranks: rank 0's (lower) index wins
    g[:, :, 0] = vals.view(np.int32)
    g[:, :, 1] = np.arange(world)[:, None] * 1000 + np.arange(batch)[None, :]
    gathered = torch.from_numpy(g).to(dev)
    state = torch.tensor([[1, 10 + b, 11 + b, 0] for b in range(batch)], dtype=torch.int32, device=dev)
    hist = torch.zeros((batch, 64), dtype=torch.int32, device=dev)
    bridge.dispatch_batch_select_advance(gathered, state, hist, world=world, batch=batch, stream_ptr=0)
    st = state.cpu().numpy()
    best = np.argmax(vals, axis=0)
    for b in range(batch):
        assert st[b, 0] == g[best[b], b, 1] and st[b, 1] == 11 + b and st[b, 2] == 12 + b
        assert hist[b, 11 + b].item() == st[b, 0]
    assert st[4, 0] == 4  # rank 0's index on the tie
    assert bridge.error_word(clear=True) == 0


def _split_sum_np(p):
    s = np.zeros(p.shape[1:], dtype=np.float32)
    for k in range(p.shape[0]):  # split order, from +0, in fp32
        s = s + p[k]
    return s


@pytest.mark.parametrize(
    "n_pad,batch,ksplit,rows",
    [
        (16, 5, 1, 300),     # ragged last tile, one split
        (32, 20, 3, 300),
        (64, 64, 17, 2048),  # more splits than one round of loads
        (64, 33, 2, 200),
    ],
)
def test_batch_epilogues_against_numpy(bridge, n_pad, batch, ksplit, rows):
    """The residual and SwiGLU epilogues against a numpy restatement: split
    sums in split order, bf16 rounding points as Transformers; the residual is
    bit-exact, SwiGLU within one bf16 step (CUDA expf vs numpy exp) on at most
    0.1% of elements; sequences from `batch` up are not written.  The batched
    RMSNorm (a tree sum of squares) against the same arithmetic with an exact
    sum of squares: the fp32 scale may differ in its last bits and, through the
    two bf16 roundings (x * scale, then * weight), an element by up to two bf16
    steps on at most 1% of elements.  Against the oracle, whose sequential fp32
    sum over 2,048 squares is itself off by ~1e-5 relative (26 flips in a row
    against the exact sum on these inputs), at most 3%."""

    import torch

    from kudacuda_b200.kudacuda_sidecar import NativeCudaError

    dev = "cuda:0"
    rng = np.random.default_rng(11 + n_pad + ksplit)
    part_np = rng.normal(0, 1, (ksplit, rows, n_pad)).astype(np.float32)
    part = torch.from_numpy(part_np).to(dev)
    s = _split_sum_np(part_np)  # [rows][n_pad]
    # residual
    x0 = O.bf16_bits(rng.normal(0, 1, (n_pad, rows)).astype(np.float32))
    x = torch.from_numpy(x0.view(np.int16)).to(dev)
    bridge.dispatch_batch_residual(part, x, ksplit=ksplit, rows=rows, n_pad=n_pad, batch=batch, stream_ptr=0)
    ref = x0.copy()
    ref[:batch] = O.bf16_bits(O.bf16_to_f32(x0[:batch]) + O.bf16_to_f32(O.bf16_bits(s.T[:batch].copy())))
    np.testing.assert_array_equal(x.cpu().numpy().view(np.uint16), ref)
    # SwiGLU over gate | up halves
    inter = rows // 2
    h = torch.zeros((n_pad, inter), dtype=torch.int16, device=dev)
    bridge.dispatch_batch_swiglu(part, h, ksplit=ksplit, intermediate=inter, n_pad=n_pad, batch=batch, stream_ptr=0)
    g = O.bf16_to_f32(O.bf16_bits(s[:inter].T[:batch].copy()))
    u = O.bf16_to_f32(O.bf16_bits(s[inter:2 * inter].T[:batch].copy()))
    act = O.bf16_to_f32(O.bf16_bits((g / (np.float32(1) + np.exp(-g))).astype(np.float32)))
    href = O.bf16_bits((act * u).astype(np.float32))
    got = h.cpu().numpy().view(np.uint16)
    diff = np.abs(got[:batch].astype(np.int32) - href.astype(np.int32))
    assert diff.max() <= 1 and np.count_nonzero(diff) <= max(1, diff.size // 1000)
    assert not got[batch:].any()
    # RMSNorm, one CTA per sequence
    hidden = 2048 if rows >= 2048 else 256
    xr = O.bf16_bits(rng.normal(0, 1, (batch, hidden)).astype(np.float32))
    wr = O.bf16_bits(rng.normal(1, 0.1, hidden).astype(np.float32))
    out = torch.zeros((batch, hidden), dtype=torch.int16, device=dev)
    bridge.dispatch_batch_rmsnorm(torch.from_numpy(xr.view(np.int16)).to(dev), torch.from_numpy(wr.view(np.int16)).to(dev),
                                  out, batch=batch, hidden=hidden, epsilon=1e-6, stream_ptr=0)
    got = out.cpu().numpy().view(np.uint16)
    for b in range(batch):
        xf = O.bf16_to_f32(xr[b])
        ss = np.float32((xf.astype(np.float64) ** 2).sum())
        inv = np.float32(1) / np.sqrt(ss / np.float32(hidden) + np.float32(1e-6))
        hn = O.bf16_to_f32(O.bf16_bits((xf * inv).astype(np.float32)))
        exact = O.bf16_bits((O.bf16_to_f32(wr) * hn).astype(np.float32))
        d = np.abs(got[b].astype(np.int32) - exact.astype(np.int32))
        assert d.max() <= 2 and np.count_nonzero(d) <= hidden // 100
        d = np.abs(got[b].astype(np.int32) - O.rmsnorm_hf_bf16(xr[b].copy(), wr, 1e-6).astype(np.int32))
        assert d.max() <= 2 and np.count_nonzero(d) <= 3 * hidden // 100
    # partials off a 16-byte boundary are refused, not read
    with pytest.raises(NativeCudaError):
        bridge.dispatch_batch_residual(part.view(-1)[1:], x, ksplit=1, rows=rows, n_pad=n_pad, batch=batch,
                                       stream_ptr=0)
    assert bridge.error_word(clear=True) == 0


def test_batched_untied_nf4_lm_head_against_oracle(bridge):
    """An untied NF4 lm_head (the Llama form) goes through the vocabulary-
    parallel pieces (argmax pairs + select) even on one rank; each sequence's
    token must be the oracle's argmax or within a rounding step of it."""

    import dataclasses

    import torch

    from kudacuda_b200.decode_engine import BatchedDecodePlan, random_weights, tiny_config

    cfg = dataclasses.replace(tiny_config(layers=1, vocab=4096), tie_embeddings=False, name="tiny-untied")
    w = random_weights(bridge, cfg, seed=17, device="cuda:0")
    assert w.lm_head is not None
    plan = BatchedDecodePlan(bridge, w, batch=4, kv_bucket=64, max_tokens=64, device="cuda:0")
    stream = torch.cuda.Stream()
    plan.capture(stream)
    tokens, positions = [7, 100, 2000, 4000], [0, 5, 17, 63]
    plan.reset_cache()
    plan.set_state(tokens, positions, stream)
    plan.replay(stream)
    stream.synchronize()
    assert bridge.error_word(clear=True) == 0
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    layer = _layer_np(w.layers[0])
    lm = O.bf16_to_f32(O.bf16_bits(O.nf4_dequant(w.lm_head.packed.reshape(-1).cpu().numpy(),
                                                 w.lm_head.absmax.cpu().numpy(), cfg.vocab * cfg.hidden)))
    lm = lm.reshape(cfg.vocab, cfg.hidden).astype(np.float64)
    st = plan.buffers.state.cpu().numpy()
    for b, (tok, pos) in enumerate(zip(tokens, positions)):
        x = emb[tok].copy()
        kc = np.zeros((cfg.kv_heads, plan.kv_bucket, cfg.head_dim), dtype=np.uint16)
        vc = np.zeros_like(kc)
        O.layer_step_hf(layer, ocfg, x, kc, vc, plan.kv_bucket, pos, cos[pos], sin[pos])
        xn = O.bf16_to_f32(O.rmsnorm_hf_bf16(x, _b16(w.final_norm), cfg.eps)).astype(np.float64)
        logits = O.bf16_to_f32(O.bf16_bits((lm @ xn).astype(np.float32)))
        ref = int(np.argmax(logits))
        got = int(st[b, 0])
        assert got == ref or logits[got] >= logits[ref] - 2e-2 * abs(logits[ref]) - 2e-3
        assert st[b, 1] == pos + 1
    plan.release()


def test_batched_prefill_then_persistent_decode_teacher_forced():
    """A 70-token prompt through the batched path (two chunks, the second
    padded) into a persistent decode plan's cache, then greedy decode on the
    device: teacher-forced top-1 agreement with the oracle over the generated
    tokens, and the prompt's cache rows close to the oracle's."""

    import torch

    from kudacuda_b200.decode_engine import BatchedPrefill, StaticDecodePlan, random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    cfg = tiny_config(layers=2, vocab=4096)
    br = KudaCudaBridge(device_id=0)
    w = random_weights(br, cfg, seed=23, device="cuda:0")
    plan = StaticDecodePlan(br, w, kv_bucket=256, max_tokens=256, device="cuda:0", persistent=True)
    stream = torch.cuda.Stream()
    plan.reset_cache()
    pre = BatchedPrefill(plan, chunk=64)
    plan.capture(stream)
    rng = np.random.default_rng(8)
    prompt = [int(t) for t in rng.integers(0, cfg.vocab, 70)]
    plan.reset_cache()
    plan.buffers.history.zero_()
    first = pre.prefill(prompt, stream)
    n_new = 8
    plan.buffers.history[len(prompt)] = first
    plan.generate_device(n_new - 1, stream)
    stream.synchronize()
    assert br.error_word(clear=True) == 0
    gen = [int(t) for t in plan.buffers.history[len(prompt):len(prompt) + n_new].cpu().tolist()]
    seq = prompt + gen
    layers = [_layer_np(L) for L in w.layers]
    emb = _b16(w.embedding).reshape(cfg.vocab, cfg.hidden)
    fn = _b16(w.final_norm)
    cos, sin = _b16(plan.buffers.rope_cos), _b16(plan.buffers.rope_sin)
    ocfg = dict(hidden=cfg.hidden, q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                inter=cfg.intermediate, eps=cfg.eps)
    kcs = [np.zeros((cfg.kv_heads, plan.kv_bucket, cfg.head_dim), dtype=np.uint16) for _ in layers]
    vcs = [np.zeros_like(kcs[0]) for _ in layers]
    agree = 0
    kc_gpu = _b16(plan.buffers.kcache)
    for pos in range(len(seq) - 1):
        x = emb[seq[pos]].copy()
        for li, layer in enumerate(layers):
            O.layer_step_hf(layer, ocfg, x, kcs[li], vcs[li], plan.kv_bucket, pos, cos[pos], sin[pos])
        tok, _ = O.lm_head_argmax(x, fn, emb, cfg.eps)
        if pos >= len(prompt) - 1:
            agree += int(tok == seq[pos + 1])
    # the prompt's key rows (positions 0..69): layer 0's come straight from the
    # embeddings (the 1e-2 bar); layer 1's are composed through a random-init
    # layer, whose rounding differences grow to ~1e-2 on their own (2e-2 bar)
    norm_close(O.bf16_to_f32(kc_gpu[0][:, :len(prompt)]), O.bf16_to_f32(kcs[0][:, :len(prompt)]))
    norm_close(O.bf16_to_f32(kc_gpu[1][:, :len(prompt)]), O.bf16_to_f32(kcs[1][:, :len(prompt)]), rel=2e-2)
    rate = agree / n_new
    assert rate >= 0.75, f"teacher-forced top-1 agreement {rate:.2f}"
    pre.plan.release()
    pre.bridge.shutdown()
    br.reset_graph()
    br.shutdown()


@pytest.mark.parametrize("batch", [5, 40])
def test_fused_epilogues_bit_identical_to_separate(bridge, batch):
    """The GEMMs with fused epilogues (last split CTA of each tile finishes the
    op) against the GEMMs + separate epilogue kernels: the same split order,
    so every output bit is the same -- residual stream, caches, next tokens."""

    import torch

    from kudacuda_b200.decode_engine import BatchedDecodePlan, random_weights, tiny_config

    cfg = tiny_config(layers=2, vocab=4096)
    w = random_weights(bridge, cfg, seed=5, device="cuda:0")
    plans = [BatchedDecodePlan(bridge, w, batch=batch, kv_bucket=128, max_tokens=128, device="cuda:0", fused=f)
             for f in (True, False)]
    plans[0].FUSE_MAX_SPLITS = 64  # every projection through its fused epilogue
    rng = np.random.default_rng(batch)
    shape = tuple(plans[0].buffers.kcache.shape)
    kc0 = torch.from_numpy(O.bf16_bits(rng.normal(0, 1, shape).astype(np.float32)).view(np.int16))
    vc0 = torch.from_numpy(O.bf16_bits(rng.normal(0, 1, shape).astype(np.float32)).view(np.int16))
    tokens = [int(t) for t in rng.integers(0, cfg.vocab, batch)]
    positions = [int(p) for p in rng.integers(0, 120, batch)]
    stream = torch.cuda.Stream()
    outs = []
    for plan in plans:
        plan.buffers.kcache.copy_(kc0.view(torch.bfloat16).to("cuda:0"))
        plan.buffers.vcache.copy_(vc0.view(torch.bfloat16).to("cuda:0"))
        for step in range(2):  # two steps: the tickets reset themselves between launches
            plan.set_state(tokens, [p + step for p in positions], stream)
            with torch.cuda.stream(stream):
                plan.record(int(stream.cuda_stream))
            stream.synchronize()
        outs.append((_b16(plan.buffers.x).copy(), _b16(plan.buffers.kcache).copy(), _b16(plan.buffers.vcache).copy(),
                     plan.buffers.state.cpu().numpy().copy()))
    assert bridge.error_word(clear=True) == 0
    for a, b in zip(*outs):
        np.testing.assert_array_equal(a, b)
    assert int(plans[0].tickets.abs().sum().item()) == 0
    assert plans[0].launches_per_step < plans[1].launches_per_step
