"""CPU test of the tensor-parallel decode maths with two gloo ranks.

Each rank takes its slices of the dense weights with the product's own
sharding (decode_engine.tp_shard / shard_rows / shard_cols -- what
random_weights(shard=(rank, world)) uses before quantising on the device):
column-parallel q/k/v (by heads) and gate/up (by rows), row-parallel o_proj
and down (by K, on 64-element block boundaries), then NF4-quantises each shard
(the oracle's quantiser, bit-exact with the device one).  Each rank runs its
half of the layer, an fp32 allreduce of the row-parallel partials and the
single-GPU residual roundings x = bf16(x + bf16(sum)).  Both ranks must
reproduce the oracle's unsharded layer step (oracle.layer_step_hf) on the
full matrices quantised whole -- so a slice off a 64-element block, or a
wrong head range, fails -- the only difference being the fp32 summation
order of the two K halves.  A vocab-parallel lm_head argmax (local argmax
over bf16-rounded logits, allgather of pairs, lowest index on ties) must pick
the unsharded argmax.
"""

import os
import socket

import numpy as np
import pytest

H, QH, KVH, D, INTER, CAP, POS, EPS, WORLD = 1024, 8, 2, 128, 2048, 64, 9, 1e-6, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config():
    from kudacuda_b200.decode_engine import QWEN25_3B

    from dataclasses import replace

    return replace(QWEN25_3B, name="tp-test", hidden=H, layers=1, q_heads=QH, kv_heads=KVH, head_dim=D,
                   intermediate=INTER, vocab=512)


def _model():
    """Dense bf16-valued weights (float32 arrays) of one layer + inputs."""

    from oracle import oracle as O

    rng = np.random.default_rng(20260824)

    def bf16(a):
        return O.bf16_bits(np.asarray(a, dtype=np.float32))

    def dense(rows, k):
        return O.bf16_to_f32(bf16(rng.normal(0, 0.02, size=(rows, k))))

    layer = {
        "in_norm": bf16(1 + rng.normal(0, 0.02, H)), "post_norm": bf16(1 + rng.normal(0, 0.02, H)),
        "q": dense(QH * D, H), "k": dense(KVH * D, H), "v": dense(KVH * D, H), "o": dense(H, QH * D),
        "gate": dense(INTER, H), "up": dense(INTER, H), "down": dense(H, INTER),
        "q_b": bf16(rng.normal(0, 0.02, QH * D)), "k_b": bf16(rng.normal(0, 0.02, KVH * D)),
        "v_b": bf16(rng.normal(0, 0.02, KVH * D)),
    }
    x = bf16(rng.normal(0, 1, H))
    kc = bf16(rng.normal(0, 1, (KVH, CAP, D)))
    vc = bf16(rng.normal(0, 1, (KVH, CAP, D)))
    inv = 1.0 / (1e6 ** (np.arange(0, D, 2) / D))
    cos = bf16(np.cos(POS * inv))
    sin = bf16(np.sin(POS * inv))
    lm = bf16(rng.normal(0, 0.02, (512, H)))  # a small vocab-parallel lm_head (bf16 rows)
    return layer, x, kc, vc, cos, sin, lm


def _nf4(w):
    from oracle import oracle as O

    packed, absmax = O.nf4_quantize(np.ascontiguousarray(w, dtype=np.float32))
    return packed.reshape(w.shape[0], w.shape[1] // 2), absmax.reshape(w.shape[0], w.shape[1] // 64)


def _flat(w):
    return np.ascontiguousarray(w[0]).reshape(-1), np.ascontiguousarray(w[1]).reshape(-1)


def _rank(rank: int, port: int, out: dict) -> None:
    import torch
    import torch.distributed as dist

    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from kudacuda_b200.decode_engine import shard_cols, shard_rows, tp_shard

        layer, x, kc, vc, cos, sin, lm = _model()
        sh = tp_shard(_config(), rank, WORLD)
        qh, kvh, il = sh.q[1] // D, sh.kv[1] // D, sh.inter[1]
        f32 = O.bf16_to_f32

        def linear(xin, w, rows_, k, bias=None):  # Transformers' bf16 linear on the oracle's fp32 dot
            y = O.bf16_bits(O.nf4_gemv(f32(xin), *_flat(w), rows_, k))
            if bias is not None:
                y = O.bf16_bits(f32(y) + f32(bias))
            return y

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        # ---- attention block, this rank's heads (the product's slices, then NF4)
        xn = O.rmsnorm_hf_bf16(x, layer["in_norm"], EPS)
        q = linear(xn, _nf4(shard_rows(layer["q"], sh.q)), qh * D, H, shard_rows(layer["q_b"], sh.q))
        k = linear(xn, _nf4(shard_rows(layer["k"], sh.kv)), kvh * D, H, shard_rows(layer["k_b"], sh.kv))
        v = linear(xn, _nf4(shard_rows(layer["v"], sh.kv)), kvh * D, H, shard_rows(layer["v_b"], sh.kv))
        q = O.rope_hf_bf16(q, qh, D, cos, sin)
        k = O.rope_hf_bf16(k, kvh, D, cos, sin)
        kc_l = kc[rank * kvh:(rank + 1) * kvh].copy()
        vc_l = vc[rank * kvh:(rank + 1) * kvh].copy()
        kc_l[:, POS] = k.reshape(kvh, D)
        vc_l[:, POS] = v.reshape(kvh, D)
        attn = O.gqa_decode(q, kc_l.reshape(-1), vc_l.reshape(-1), O.BF16, qh, kvh, D, POS + 1, CAP, 1 / np.sqrt(D))
        part = O.nf4_gemv(f32(attn), *_flat(_nf4(shard_cols(layer["o"], sh.q))), H, qh * D)
        xr = O.bf16_bits(f32(x) + f32(O.bf16_bits(allreduce(part))))
        # ---- MLP block, this rank's intermediate rows
        xn = O.rmsnorm_hf_bf16(xr, layer["post_norm"], EPS)
        g = f32(linear(xn, _nf4(shard_rows(layer["gate"], sh.inter)), il, H))
        u = f32(linear(xn, _nf4(shard_rows(layer["up"], sh.inter)), il, H))
        act = f32(O.bf16_bits(g / (1 + np.exp(-g))))
        hmid = O.bf16_bits(act * u)
        part = O.nf4_gemv(f32(hmid), *_flat(_nf4(shard_cols(layer["down"], sh.inter))), H, il)
        xr = O.bf16_bits(f32(xr) + f32(O.bf16_bits(allreduce(part))))
        out["x"] = xr
        # ---- vocab-parallel argmax over bf16-rounded logits
        lg = f32(O.bf16_bits(f32(shard_rows(lm, sh.vocab)) @ f32(xr)))
        loc = int(np.argmax(lg))  # numpy keeps the first (lowest) index on ties
        pair = torch.tensor([float(lg[loc]), float(sh.vocab[0] + loc)], dtype=torch.float64)
        gathered = [torch.zeros(2, dtype=torch.float64) for _ in range(WORLD)]
        dist.all_gather(gathered, pair)
        best = min(gathered, key=lambda p: (-p[0].item(), p[1].item()))
        out["token"] = int(best[1].item())
    finally:
        dist.destroy_process_group()


def _worker(rank, port, q):
    out = {}
    _rank(rank, port, out)
    q.put((rank, out))


def test_two_rank_layer_matches_unsharded_oracle():
    import torch.multiprocessing as mp

    from oracle import oracle as O

    O.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0

    layer, x, kc, vc, cos, sin, lm = _model()
    for name in ("q", "k", "v", "o", "gate", "up", "down"):  # the unsharded model: each matrix quantised whole
        layer[name] = _nf4(layer[name])
    ref = x.copy()
    O.layer_step_hf(layer, dict(hidden=H, q_heads=QH, kv_heads=KVH, head_dim=D, inter=INTER, eps=EPS), ref,
                    kc.copy(), vc.copy(), CAP, POS, cos, sin)
    r = O.bf16_to_f32(ref)
    for rank in range(WORLD):
        got = O.bf16_to_f32(results[rank]["x"])
        rel = np.linalg.norm(got - r) / np.linalg.norm(r)
        assert rel <= 1e-3, f"rank {rank}: relative difference {rel:.2e}"
        # the bf16 values differ only where the two fp32 summation orders round differently
        assert np.mean(results[rank]["x"] == ref) >= 0.98
    assert results[0]["x"].tobytes() == results[1]["x"].tobytes()  # ranks agree exactly
    lg = O.bf16_to_f32(O.bf16_bits(O.bf16_to_f32(lm) @ O.bf16_to_f32(results[0]["x"])))
    assert results[0]["token"] == results[1]["token"] == int(np.argmax(lg))


def test_tp_shard_plan_rejects_uneven_or_unaligned_splits():
    from dataclasses import replace

    from kudacuda_b200.decode_engine import LLAMA3_8B, tp_shard

    sh = tp_shard(LLAMA3_8B, 3, 8)
    assert sh.q == (3 * 512, 512) and sh.kv == (3 * 128, 128) and sh.inter == (3 * 1792, 1792)
    assert sh.vocab == (3 * 16032, 16032)
    with pytest.raises(ValueError):
        tp_shard(LLAMA3_8B, 0, 3)  # 32 heads over 3 ranks
    with pytest.raises(ValueError):
        tp_shard(replace(LLAMA3_8B, intermediate=14336 + 8 * 32), 0, 8)  # K slice off a 64-block
