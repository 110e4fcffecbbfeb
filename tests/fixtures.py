"""Deterministic inputs shared by the CPU and GPU tests.

Two families:
  * the reference smoke-test patterns, restated from the reference's own
    native tests (cited per function);
  * seeded synthetic model data of the BASELINE shapes: weights N(0, 0.02)
    quantised to NF4 (blocksize 64), activations / KV N(0, 1), biases
    N(0, 0.02), norm weights 1 + N(0, 0.02); seed 20260824 (the reference's
    tools/correctness/run_qwen2_gqa_check.py:41).
"""

from __future__ import annotations

import numpy as np

from oracle import oracle as O

SEED = 20260824


# ------------------------------------------------------------------ smoke patterns
def smoke_pack(logical_count: int, salt: int, mult: int = 5) -> np.ndarray:
    """tests/nf4_tiled_gemv_smoke.cu:28-35 (mult 5) and tests/nf4_fused_qkv_smoke.cu:41-47 (mult 7)."""

    idx = np.arange(0, logical_count, 2, dtype=np.int64)
    even = (idx * mult + salt) & 0x0F
    odd = ((idx + 1) * mult + salt) & 0x0F
    return ((even << 4) | odd).astype(np.uint8)


def smoke_scales(count: int, base: float, mod: int, step: float) -> np.ndarray:
    """tests/nf4_tiled_gemv_smoke.cu:68-70: base + (i % mod) * step, fp32."""

    i = np.arange(count, dtype=np.int64)
    return (np.float32(base) + (i % mod).astype(np.float32) * np.float32(step)).astype(np.float32)


def smoke_qkv_case(dtype: int = O.F16):
    """tests/nf4_tiled_gemv_smoke.cu:46-75 -- hidden 2048, q_out 2048, kv_out 256."""

    hidden, q_out, kv_out = 2048, 2048, 256
    i = np.arange(hidden, dtype=np.float32)
    conv = O.f16_bits if dtype == O.F16 else O.bf16_bits
    x = conv(np.sin(i * np.float32(0.013)).astype(np.float32))
    nw = conv((np.float32(0.75) + (np.arange(hidden) % 23).astype(np.float32) * np.float32(0.004)).astype(np.float32))
    qw = smoke_pack(q_out * hidden, 1)
    kw = smoke_pack(kv_out * hidden, 3)
    vw = smoke_pack(kv_out * hidden, 7)
    qa = smoke_scales(q_out * hidden // 64, 0.2, 19, 0.009)
    ka = smoke_scales(kv_out * hidden // 64, 0.25, 17, 0.011)
    va = smoke_scales(kv_out * hidden // 64, 0.18, 13, 0.013)
    qb = conv(((np.arange(q_out) % 11) - 5).astype(np.float32) * np.float32(0.002))
    kb = conv(((np.arange(kv_out) % 7) - 3).astype(np.float32) * np.float32(0.003))
    vb = conv(((np.arange(kv_out) % 5) - 2).astype(np.float32) * np.float32(0.004))
    return dict(x=x, nw=nw, q=(qw, qa, qb, q_out), k=(kw, ka, kb, kv_out), v=(vw, va, vb, kv_out), eps=1e-5)


def smoke_swiglu_case(dtype: int = O.BF16):
    """tests/nf4_swiglu_bf16_smoke.cu:50-60 (bf16) / tests/nf4_swiglu_smoke.cu (f16)."""

    hidden, inter = 2048, 11008
    i = np.arange(hidden, dtype=np.float32)
    conv = O.f16_bits if dtype == O.F16 else O.bf16_bits
    x = conv(np.sin(i * np.float32(0.013)).astype(np.float32))
    nw = conv((np.float32(0.75) + (np.arange(hidden) % 23).astype(np.float32) * np.float32(0.004)).astype(np.float32))
    gw = smoke_pack(inter * hidden, 1)
    uw = smoke_pack(inter * hidden, 7)
    ga = smoke_scales(inter * hidden // 64, 0.12, 19, 0.003)
    ua = smoke_scales(inter * hidden // 64, 0.15, 17, 0.004)
    return dict(x=x, nw=nw, gate=(gw, ga), up=(uw, ua), inter=inter, eps=1e-5)


def smoke_gqa_case(kv_len: int = 37, dtype: int = O.F16):
    """tests/qwen2_gqa_smoke.cu:31-63 -- q/k/v sin/cos ramps, 16/2/128 heads."""

    qh, kvh, d = 16, 2, 128
    conv = O.f16_bits if dtype == O.F16 else O.bf16_bits
    qi = np.arange(qh * d, dtype=np.float32)
    ci = np.arange(kvh * kv_len * d, dtype=np.float32)
    q = conv((np.sin(qi * np.float32(0.017)) * np.float32(0.75)).astype(np.float32))
    k = conv((np.cos(ci * np.float32(0.011)) * np.float32(0.55)).astype(np.float32))
    v = conv((np.sin(ci * np.float32(0.023)) * np.float32(0.65)).astype(np.float32))
    return dict(q=q, k=k, v=v, kv_len=kv_len, scale=np.float32(1.0 / 11.313708498984761))


# ------------------------------------------------------------------ seeded model data
def rng(seed: int = SEED) -> np.random.Generator:
    return np.random.default_rng(seed)


def nf4_weight(g: np.random.Generator, rows: int, k: int, std: float = 0.02):
    """N(0, std) weights, rounded to bf16 (the model dtype) then NF4-quantised."""

    w = O.bf16_to_f32(O.bf16_bits(g.standard_normal((rows, k), dtype=np.float32) * np.float32(std)))
    packed, absmax = O.nf4_quantize(w.reshape(-1))
    return packed, absmax


def bf16_normal(g: np.random.Generator, n: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    return O.bf16_bits((g.standard_normal(n, dtype=np.float32) * np.float32(std) + np.float32(mean)).astype(np.float32))


def rope_tables(max_pos: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """Qwen2RotaryEmbedding default rope (Transformers): inv_freq = 1 / theta^(2i/d)
    in fp32, freqs = pos * inv_freq in fp32, cos/sin in fp32 rounded to bf16.
    Only the first head_dim/2 columns are kept (emb = cat(freqs, freqs))."""

    import torch

    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq.float())
    cos = freqs.cos().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    sin = freqs.sin().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return np.ascontiguousarray(cos), np.ascontiguousarray(sin)


def qwen_layer(g: np.random.Generator, hidden=2048, q_heads=16, kv_heads=2, head_dim=128, inter=11008, bias=True):
    qo, kvo = q_heads * head_dim, kv_heads * head_dim
    layer = {
        "in_norm": bf16_normal(g, hidden, 0.02, 1.0),
        "post_norm": bf16_normal(g, hidden, 0.02, 1.0),
        "q": nf4_weight(g, qo, hidden),
        "k": nf4_weight(g, kvo, hidden),
        "v": nf4_weight(g, kvo, hidden),
        "o": nf4_weight(g, hidden, qo),
        "gate": nf4_weight(g, inter, hidden),
        "up": nf4_weight(g, inter, hidden),
        "down": nf4_weight(g, hidden, inter),
    }
    if bias:
        layer["q_b"] = bf16_normal(g, qo, 0.02)
        layer["k_b"] = bf16_normal(g, kvo, 0.02)
        layer["v_b"] = bf16_normal(g, kvo, 0.02)
    return layer
