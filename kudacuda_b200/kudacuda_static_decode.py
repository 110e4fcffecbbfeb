"""Fixed-shape decode for a Transformers Qwen2/Llama model, B200 edition.

Mirrors the reference's static-decode interface
(python/kudacuda_static_decode.py:80-447: ``GraphStaticCache``,
``StaticDecodeContract``, ``StaticDecodeGraphRunner`` with ``capture`` /
``replay`` / ``invalidate`` / ``captured`` / ``model_fingerprint``), but the
captured graph is not a Transformers forward with patched attention: the
runner converts the model's linears to NF4 (blocksize 64, fp32 absmax, on the
device with the library's quantiser, or takes bitsandbytes-packed tensors as
they are), and captures this library's whole decode step -- embedding, 36
fused layer blocks, lm_head + argmax, state advance -- as one CUDA graph
guarded by a ``DecodeGraphKey``.  Replay writes {token, position} on the
device through the C ABI; nothing is recomputed on the host.

``GraphStaticCache`` exposes the fixed-capacity KV buffers of a plan with the
cache methods Transformers code calls (``update``, ``get_seq_length``,
``get_max_length``, ``get_max_cache_shape``, ``len``).
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from typing import Any, Optional

from .decode_engine import (
    DecoderConfig,
    LayerWeights,
    ModelWeights,
    NF4Linear,
    StaticDecodePlan,
    quantize_nf4,
)
from .kudacuda_graph_plan import GraphContractError
from .kudacuda_sidecar import KudaCudaBridge, NativeCudaError


# ------------------------------------------------------------------ Transformers model -> NF4 decode weights
def _cfg_get(cfg: Any, *names: str, default: Any = None) -> Any:
    for n in names:
        v = getattr(cfg, n, None)
        if v is not None:
            return v
    return default


def decoder_config_from_transformers(model: Any) -> DecoderConfig:
    """DecoderConfig of a Qwen2ForCausalLM / LlamaForCausalLM (or their base model)."""

    cfg = model.config
    hidden = int(cfg.hidden_size)
    heads = int(cfg.num_attention_heads)
    head_dim = int(_cfg_get(cfg, "head_dim", default=hidden // heads) or hidden // heads)
    rope = _cfg_get(cfg, "rope_theta")
    if rope is None:
        params = _cfg_get(cfg, "rope_parameters", "rope_scaling", default={}) or {}
        rope = params.get("rope_theta", 10000.0) if isinstance(params, dict) else 10000.0
    layers = _decoder_layers(model)
    attn = layers[0].self_attn
    qkv_bias = getattr(attn.q_proj, "bias", None) is not None
    return DecoderConfig(
        name=str(_cfg_get(cfg, "model_type", default="decoder")),
        hidden=hidden,
        layers=int(cfg.num_hidden_layers),
        q_heads=heads,
        kv_heads=int(_cfg_get(cfg, "num_key_value_heads", default=heads)),
        head_dim=head_dim,
        intermediate=int(cfg.intermediate_size),
        vocab=int(cfg.vocab_size),
        rope_theta=float(rope),
        eps=float(_cfg_get(cfg, "rms_norm_eps", default=1e-6)),
        qkv_bias=qkv_bias,
        tie_embeddings=bool(_cfg_get(cfg, "tie_word_embeddings", default=False)),
    )


def _base(model: Any) -> Any:
    return getattr(model, "model", model)


def _decoder_layers(model: Any) -> list:
    return list(_base(model).layers)


def _linear_nf4(bridge: KudaCudaBridge, torch: Any, linear: Any, device: Any, stream_ptr: int) -> NF4Linear:
    """A bitsandbytes Linear4bit keeps its packed storage (validated like the
    reference's ``_validate_nf4_weight``); a dense linear is quantised on the
    device."""

    w = linear.weight
    state = getattr(w, "quant_state", None)
    if state is not None:
        rows, k = (int(v) for v in state.shape)
        KudaCudaBridge._validate_nf4_weight(w, state.absmax, expected_shape=(rows, k), label="linear weight")
        return NF4Linear(w, state.absmax, rows, k)
    dense = w.detach().to(device=device, dtype=torch.bfloat16).contiguous()
    return quantize_nf4(bridge, torch, dense, stream_ptr)


def weights_from_transformers(bridge: KudaCudaBridge, model: Any, *, device: Any = "cuda:0",
                              torch_module: Any = None) -> ModelWeights:
    if torch_module is None:
        import torch as torch_module
    torch = torch_module
    cfg = decoder_config_from_transformers(model)
    sp = int(torch.cuda.current_stream(device).cuda_stream)

    def bf16(t: Any) -> Any:
        return t.detach().to(device=device, dtype=torch.bfloat16).contiguous()

    layers = []
    for layer in _decoder_layers(model):
        a, m = layer.self_attn, layer.mlp
        layers.append(
            LayerWeights(
                in_norm=bf16(layer.input_layernorm.weight),
                post_norm=bf16(layer.post_attention_layernorm.weight),
                q=_linear_nf4(bridge, torch, a.q_proj, device, sp),
                k=_linear_nf4(bridge, torch, a.k_proj, device, sp),
                v=_linear_nf4(bridge, torch, a.v_proj, device, sp),
                o=_linear_nf4(bridge, torch, a.o_proj, device, sp),
                gate=_linear_nf4(bridge, torch, m.gate_proj, device, sp),
                up=_linear_nf4(bridge, torch, m.up_proj, device, sp),
                down=_linear_nf4(bridge, torch, m.down_proj, device, sp),
                q_bias=None if a.q_proj.bias is None else bf16(a.q_proj.bias),
                k_bias=None if a.k_proj.bias is None else bf16(a.k_proj.bias),
                v_bias=None if a.v_proj.bias is None else bf16(a.v_proj.bias),
            )
        )
    base = _base(model)
    embedding = bf16(base.embed_tokens.weight)
    lm_head = None
    if not cfg.tie_embeddings:
        lm_head = _linear_nf4(bridge, torch, model.lm_head, device, sp)
    torch.cuda.synchronize(device)
    return ModelWeights(cfg, layers, embedding, bf16(base.norm.weight), lm_head)


# ------------------------------------------------------------------ static cache view
class GraphStaticCache:
    """Fixed-capacity KV view of a plan's caches ([layers][kv_heads][cap][d])."""

    def __init__(self, key_cache: Any, value_cache: Any, *, seq_length: int = 0) -> None:
        self.key_cache = key_cache
        self.value_cache = value_cache
        self.max_cache_len = int(key_cache.shape[2])
        self._seq = int(seq_length)

    @classmethod
    def from_plan(cls, plan: StaticDecodePlan, *, seq_length: int = 0) -> "GraphStaticCache":
        return cls(plan.buffers.kcache, plan.buffers.vcache, seq_length=seq_length)

    def update(self, key_states: Any, value_states: Any, layer_idx: int, cache_kwargs: Optional[dict] = None,
               *args: Any, **kwargs: Any) -> tuple[Any, Any]:
        """Write [1, kv_heads, n, d] rows at ``cache_position`` (index_copy on
        the token axis) and return the layer's full fixed-size K/V."""

        kwargs = dict(cache_kwargs or {}, **kwargs)
        pos = kwargs.get("cache_position")
        k_layer, v_layer = self.key_cache[layer_idx], self.value_cache[layer_idx]
        if pos is None:
            raise GraphContractError("GraphStaticCache.update needs cache_position")
        if int(pos.max()) >= self.max_cache_len:
            raise GraphContractError("cache_position exceeds the static KV capacity")
        k_layer.index_copy_(1, pos, key_states[0].to(k_layer.dtype))
        v_layer.index_copy_(1, pos, value_states[0].to(v_layer.dtype))
        if layer_idx == 0:
            self._seq = max(self._seq, int(pos.max()) + 1)
        return k_layer.unsqueeze(0), v_layer.unsqueeze(0)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._seq

    def get_max_length(self, layer_idx: int = 0) -> int:
        return self.max_cache_len

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.max_cache_len

    def __len__(self) -> int:
        return int(self.key_cache.shape[0])


# ------------------------------------------------------------------ runner
@dataclass(frozen=True)
class StaticDecodeContract:
    tactic_name: str = "decode_step_sm100_v1"
    kv_bucket: int = 512
    batch_size: int = 1
    query_len: int = 1


class StaticDecodeGraphRunner:
    """Capture one decode step of a Transformers decoder as this library's
    CUDA graph; replay it per token."""

    def __init__(self, bridge: KudaCudaBridge, model: Any, torch_module: Any = None, *,
                 device: Any = "cuda:0") -> None:
        if torch_module is None:
            import torch as torch_module
        self.bridge = bridge
        self.model = model
        self.torch = torch_module
        self.device = device
        self.plan: Optional[StaticDecodePlan] = None
        self.cache: Optional[GraphStaticCache] = None
        self.contract: Optional[StaticDecodeContract] = None
        self.stream: Any = None
        self.fallback_reason: Optional[str] = None
        self._weights: Optional[ModelWeights] = None
        self._host_in = None
        self._host_out = None

    @property
    def captured(self) -> bool:
        return self.plan is not None and self.plan.captured

    @staticmethod
    def model_fingerprint(model: Any) -> str:
        """Architecture identity of the model (config fields that shape the graph)."""

        cfg = decoder_config_from_transformers(model)
        return hashlib.sha256(repr(cfg).encode()).hexdigest()[:16]

    def capture(self, *, kv_bucket: int = 512, stream: Any = None,
                tactic_name: str = "decode_step_sm100_v1") -> None:
        torch = self.torch
        if self.captured:
            raise GraphContractError("runner already holds a captured graph; invalidate it first")
        try:
            if self._weights is None:
                self._weights = weights_from_transformers(self.bridge, self.model, device=self.device,
                                                          torch_module=torch)
            self.stream = stream or torch.cuda.Stream(device=self.device)
            self.plan = StaticDecodePlan(self.bridge, self._weights, kv_bucket=kv_bucket, device=self.device,
                                         torch_module=torch)
            self.plan.capture(self.stream)
        except Exception as exc:
            self.invalidate(f"capture failed: {exc}")
            raise
        self.cache = GraphStaticCache.from_plan(self.plan)
        self.contract = StaticDecodeContract(tactic_name=tactic_name, kv_bucket=int(kv_bucket))
        self._host_in = torch.zeros(4, dtype=torch.int32).pin_memory()
        self._host_out = torch.zeros(1, dtype=torch.int32).pin_memory()

    def replay(self, token_id: int, position: int, *, stream: Any = None) -> int:
        """One decode step for ``token_id`` at ``position``; returns the greedy
        next token (host-synchronous, through kudacuda_sm100_graph_step_host)."""

        if not self.captured or self.plan is None:
            raise GraphContractError("runner has no captured graph")
        if stream is not None and stream is not self.stream:
            raise GraphContractError("replay stream differs from the capture stream")
        if not 0 <= int(position) < self.plan.kv_bucket:
            raise GraphContractError(f"position {position} outside the KV bucket {self.plan.kv_bucket}")
        b = self.plan.buffers
        self._host_in[0], self._host_in[1], self._host_in[2] = int(token_id), int(position), int(position) + 1
        self.bridge.graph_step_host(self._host_in, b.state, self._host_out, b.next_token,
                                    stream_ptr=int(self.stream.cuda_stream))
        if self.cache is not None:
            self.cache._seq = max(self.cache._seq, int(position) + 1)
        return int(self._host_out[0])

    def generate(self, prompt: list[int], new_tokens: int) -> list[int]:
        """Greedy continuation of ``prompt`` (prompt tokens through decode steps)."""

        if self.plan is None:
            raise GraphContractError("runner has no captured graph")
        self.plan.reset_cache()
        if self.cache is not None:
            self.cache._seq = 0
        nxt = 0
        for i, tok in enumerate(prompt):
            nxt = self.replay(tok, i)
        out = [nxt]
        for j in range(1, int(new_tokens)):
            out.append(self.replay(out[-1], len(prompt) + j - 1))
        return out

    def invalidate(self, reason: str) -> None:
        self.fallback_reason = str(reason)
        if self.plan is not None:
            self.plan.graph_plan.invalidate()
        try:
            self.bridge.reset_graph()
        except NativeCudaError:
            pass
        self.plan = None
        self.cache = None
