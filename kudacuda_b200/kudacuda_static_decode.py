"""Fixed-shape decode for a Transformers Qwen2/Llama model, B200 edition.

A drop-in for the reference's static-decode module
(python/kudacuda_static_decode.py:80-447): ``GraphStaticCache`` (with
``from_dynamic_cache``), ``StaticDecodeContract`` and
``StaticDecodeGraphRunner`` take the same calls -- ``capture(*, input_ids,
position_ids, attention_mask, cache_position, past_key_values,
logical_kv_len, kv_bucket, tactic_name, stream_ptr, stream, device_id,
model_kwargs, workspace)`` and ``replay(*, next_token, position_ids,
cache_position, logical_kv_len, stream_ptr)``, both returning the logits
[1, 1, vocab] of the step -- so tools/benchmark/benchmark_gemma.py:292-350
drives it unchanged.

What is captured differs: not a Transformers forward with patched attention
but this library's whole decode step (embedding, every decoder layer in one
persistent launch, final RMSNorm + tied lm_head, state advance), over NF4
weights converted once from the model (bitsandbytes-packed tensors are taken
as they are; dense linears are quantised on the device) and over the
caller's GraphStaticCache tensors, which the step reads and appends to in
place.  Replay writes the token (a device copy), position and KV length, then
replays the graph; nothing of the model runs on the host.
"""

from __future__ import annotations

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
from .kudacuda_graph_plan import DecodeGraphKey, GraphContractError
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


# ------------------------------------------------------------------ static cache
def _cache_layers(cache: Any) -> list:
    """Per-layer entries of a Transformers cache: ``cache.layers`` (objects
    with keys/values) or parallel key_cache / value_cache lists."""

    layers = getattr(cache, "layers", None)
    if layers is not None:
        return list(layers)
    keys, values = getattr(cache, "key_cache", None), getattr(cache, "value_cache", None)
    if keys is not None and values is not None:
        return list(zip(keys, values))
    return []


def _layer_kv(entry: Any, index: int) -> tuple[Any, Any]:
    if isinstance(entry, tuple) and len(entry) == 2:
        return entry
    for kname, vname in (("keys", "values"), ("key_cache", "value_cache")):
        k, v = getattr(entry, kname, None), getattr(entry, vname, None)
        if k is not None and v is not None:
            return k, v
    raise GraphContractError(f"cache layer {index} has no key/value tensors")


def _shape(value: Any) -> tuple[int, ...]:
    return tuple(int(v) for v in getattr(value, "shape", ()))


class GraphStaticCache:
    """Fixed-capacity KV cache for graph replay: per-layer K and V tensors
    [batch, kv_heads, max_cache_len, head_dim] and a device-resident
    ``cache_position`` (the reference's GraphStaticCache,
    python/kudacuda_static_decode.py:80-172)."""

    def __init__(self, *, key_cache: list, value_cache: list, cache_position: Any, sequence_length: int,
                 max_cache_len: int) -> None:
        self.key_cache = list(key_cache)
        self.value_cache = list(value_cache)
        self.cache_position = cache_position
        self._sequence_length = int(sequence_length)
        self.max_cache_len = int(max_cache_len)
        self.layers = list(zip(self.key_cache, self.value_cache))

    @classmethod
    def from_dynamic_cache(cls, torch_module: Any, dynamic_cache: Any, *, max_cache_len: int) -> "GraphStaticCache":
        """Copy a prefilled Transformers cache into fixed-capacity tensors
        (rows past the prefix are zero)."""

        torch = torch_module
        entries = _cache_layers(dynamic_cache)
        if not entries:
            raise GraphContractError("dynamic cache does not expose cache layers")
        cap = int(max_cache_len)
        keys, values = [], []
        for i, entry in enumerate(entries):
            k, v = _layer_kv(entry, i)
            if k.dim() != 4 or _shape(v) != _shape(k):
                raise GraphContractError(f"cache layer {i} is not a rank-4 KV pair")
            n = int(k.shape[-2])
            if n > cap:
                raise GraphContractError("max_cache_len is smaller than the prefetched cache")
            shape = (int(k.shape[0]), int(k.shape[1]), cap, int(k.shape[3]))
            kt = torch.zeros(shape, dtype=k.dtype, device=k.device)
            vt = torch.zeros(shape, dtype=v.dtype, device=v.device)
            kt[..., :n, :].copy_(k)
            vt[..., :n, :].copy_(v)
            keys.append(kt)
            values.append(vt)
        seq = int(dynamic_cache.get_seq_length())
        pos = torch.tensor([seq], dtype=torch.long, device=keys[0].device)
        return cls(key_cache=keys, value_cache=values, cache_position=pos, sequence_length=seq, max_cache_len=cap)

    def update(self, key_states: Any, value_states: Any, layer_idx: int, *args: Any, **kwargs: Any) -> tuple[Any, Any]:
        """Write the step's rows at ``cache_position`` (token axis) and return
        the layer's full fixed-size K/V (what Transformers attention reads)."""

        if int(key_states.shape[-2]) != int(self.cache_position.numel()):
            raise GraphContractError("graph cache position count does not match key update length")
        self.key_cache[layer_idx].index_copy_(2, self.cache_position, key_states)
        self.value_cache[layer_idx].index_copy_(2, self.cache_position, value_states)
        return self.key_cache[layer_idx], self.value_cache[layer_idx]

    def get_seq_length(self, layer_idx: int = 0) -> int:
        return self._sequence_length

    def get_max_length(self, layer_idx: int = 0) -> int:
        return self.max_cache_len

    def get_max_cache_shape(self, layer_idx: int = 0) -> int:
        return self.max_cache_len

    def __len__(self) -> int:
        return len(self.key_cache)


# ------------------------------------------------------------------ runner
@dataclass(frozen=True)
class StaticDecodeContract:
    key: DecodeGraphKey
    stream_ptr: int
    logical_kv_len: int


class StaticDecodeGraphRunner:
    """Capture one complete decode step and replay it by pointer identity
    (the reference's StaticDecodeGraphRunner, with its capture / replay /
    invalidate signatures and status fields)."""

    def __init__(self, bridge: KudaCudaBridge, model: Any, torch_module: Any = None) -> None:
        if torch_module is None:
            import torch as torch_module
        self.bridge = bridge
        self.model = model
        self.torch = torch_module
        self.contract: Optional[StaticDecodeContract] = None
        self.static_inputs: dict[str, Any] = {}
        self.cache: Any = None
        self.kv_len_device: Any = None
        self.logits: Any = None
        self.status = "not-requested"
        self.reason: Optional[str] = None
        self.capture_ms: Optional[float] = None
        self.replay_count = 0
        self.backend = "native"
        self.cuda_graph: Any = None
        self.workspace: Any = None
        self.plan: Optional[StaticDecodePlan] = None
        self._weights: Optional[ModelWeights] = None
        self._stream: Any = None
        self._host: Any = None
        self._host_next = 0

    @property
    def captured(self) -> bool:
        return self.contract is not None and self.status == "captured"

    @staticmethod
    def model_fingerprint(model: Any) -> str:
        """Identity of the model the graph was built for: class, model type,
        layer count, hidden size, vocabulary and dtype."""

        config = getattr(model, "config", None)
        fields = (type(model).__name__, getattr(config, "model_type", ""), getattr(config, "num_hidden_layers", ""),
                  getattr(config, "hidden_size", ""), getattr(config, "vocab_size", ""),
                  str(getattr(config, "torch_dtype", "")))
        return "|".join(str(f) for f in fields)

    def prepare_weights(self, device: Any = None) -> ModelWeights:
        """The model's decode weights (NF4), converted once and reused by every
        capture; callable before capture (e.g. to build an eager model on the
        same NF4 values)."""

        if device is None:
            device = next(self.model.parameters()).device
        if self._weights is None:
            self._weights = weights_from_transformers(self.bridge, self.model, device=device, torch_module=self.torch)
        return self._weights

    def capture(self, *, input_ids: Any, position_ids: Any, attention_mask: Any, cache_position: Any,
                past_key_values: GraphStaticCache, logical_kv_len: int, kv_bucket: int, tactic_name: str,
                stream_ptr: int, stream: Any = None, device_id: int = 0, model_kwargs: Any = None,
                workspace: Any = None) -> Any:
        """Build the plan over ``past_key_values``' tensors, capture one step,
        replay it once for ``input_ids`` at position ``logical_kv_len`` and
        return its logits [1, 1, vocab].  ``attention_mask`` and
        ``model_kwargs`` are accepted for signature parity and not read: the
        step attends over exactly ``logical_kv_len + 1`` cached rows."""

        import time

        torch = self.torch
        if self.captured:
            raise GraphContractError("graph runner already has a captured forward")
        if _shape(input_ids) != (1, 1):
            raise GraphContractError("static decode captures batch 1, query length 1")
        cache = past_key_values
        if int(kv_bucket) != int(cache.max_cache_len):
            raise GraphContractError("kv_bucket differs from the graph cache's max_cache_len")
        if not 0 <= int(logical_kv_len) < int(kv_bucket):
            raise GraphContractError("logical_kv_len + 1 exceeds the KV bucket")
        t0 = time.perf_counter()
        device = input_ids.device
        try:
            weights = self.prepare_weights(device)
            kv = (cache.key_cache, cache.value_cache)
            try:
                plan = StaticDecodePlan(self.bridge, weights, kv_bucket=int(kv_bucket), device=device,
                                        torch_module=torch, persistent=True, kv_cache=kv)
            except NativeCudaError:  # shapes outside the persistent kernel: the per-op step
                plan = StaticDecodePlan(self.bridge, weights, kv_bucket=int(kv_bucket), device=device,
                                        torch_module=torch, kv_cache=kv)
            self.plan = plan
            self._stream = stream if stream is not None else torch.cuda.ExternalStream(int(stream_ptr))
            if int(self._stream.cuda_stream) != int(stream_ptr):
                raise GraphContractError("stream and stream_ptr name different streams")
            self.bridge.reset_graph()
            plan.capture(self._stream, warm_position=int(logical_kv_len))
        except Exception as error:
            self.plan = None
            try:
                self.bridge.reset_graph()
            except NativeCudaError:
                pass
            self.status = "fallback"
            self.reason = f"capture_failed:{type(error).__name__}:{error}"
            raise GraphContractError(self.reason) from error
        self.static_inputs = {"input_ids": input_ids.clone(), "position_ids": position_ids.clone(),
                              "attention_mask": attention_mask, "cache_position": cache_position}
        self.cache = cache
        self.workspace = workspace
        self.kv_len_device = plan.buffers.state[2:3]
        self.logits = plan.buffers.logits.view(1, 1, -1)
        # pinned host slots for the per-step state copies; a slot is reused
        # only after the copies that read it have run (its event)
        self._host = [(torch.zeros(4, dtype=torch.int32).pin_memory(), torch.zeros(1, dtype=torch.long).pin_memory(),
                       torch.cuda.Event()) for _ in range(4)]
        self._host_next = 0
        self.contract = StaticDecodeContract(key=plan.graph_key, stream_ptr=int(stream_ptr),
                                             logical_kv_len=int(logical_kv_len) + 1)
        self.status = "captured"
        self.reason = None
        self._step(input_ids, int(logical_kv_len))
        self.replay_count = 1
        self.capture_ms = (time.perf_counter() - t0) * 1e3
        return self.logits

    def _step(self, token: Any, logical_kv_len: int) -> None:
        """state <- {token (device copy), position, kv_len}; cache_position <-
        position; replay -- all ordered on the capture stream."""

        torch = self.torch
        b = self.plan.buffers
        pos = int(logical_kv_len)
        state_h, pos_h, done = self._host[self._host_next]
        self._host_next = (self._host_next + 1) % len(self._host)
        done.synchronize()  # the copies that last read this slot have run
        state_h[0], state_h[1], state_h[2], state_h[3] = 0, pos, pos + 1, 0
        pos_h[0] = pos
        with torch.cuda.stream(self._stream):
            b.state.copy_(state_h, non_blocking=True)
            b.state[0:1].copy_(token.reshape(-1)[:1], non_blocking=True)
            self.cache.cache_position.copy_(pos_h, non_blocking=True)
            done.record(self._stream)
        self.plan.replay(self._stream)

    def replay(self, *, next_token: Any, position_ids: Any, cache_position: int, logical_kv_len: int,
               stream_ptr: int) -> Any:
        """One decode step for ``next_token`` with ``logical_kv_len`` rows
        already cached; returns the logits [1, 1, vocab] (device buffer,
        overwritten by the next replay).  The step's RoPE position and cache
        row are ``cache_position`` (equal to ``position_ids`` in every caller
        of the reference)."""

        if not self.captured or self.contract is None or self.plan is None:
            raise GraphContractError("graph runner has no captured forward")
        if int(stream_ptr) != self.contract.stream_ptr:
            raise GraphContractError("graph replay stream changed")
        if int(logical_kv_len) + 1 > self.contract.key.kv_bucket:
            raise GraphContractError("graph replay KV length exceeds the captured bucket")
        if _shape(next_token) != _shape(self.static_inputs["input_ids"]):
            raise GraphContractError("graph replay token shape changed")
        if _shape(position_ids) != _shape(self.static_inputs["position_ids"]):
            raise GraphContractError("graph replay position shape changed")
        if int(cache_position) != int(logical_kv_len):
            raise GraphContractError("cache_position must equal logical_kv_len (one new row per step)")
        self.plan.verify_key()
        self._step(next_token, int(logical_kv_len))
        self.replay_count += 1
        return self.logits

    def generate(self, prompt: list[int], new_tokens: int, *, kv_bucket: int = 512) -> list[int]:
        """Greedy continuation of ``prompt`` with the prompt fed through decode
        steps (no Transformers prefill); captures on first use."""

        torch = self.torch
        device = next(self.model.parameters()).device
        first = torch.tensor([[int(prompt[0])]], dtype=torch.long, device=device)
        if not self.captured:
            cfg = decoder_config_from_transformers(self.model)
            shape = (1, cfg.kv_heads, int(kv_bucket), cfg.head_dim)
            keys = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.layers)]
            values = [torch.zeros(shape, dtype=torch.bfloat16, device=device) for _ in range(cfg.layers)]
            cache = GraphStaticCache(key_cache=keys, value_cache=values,
                                     cache_position=torch.zeros(1, dtype=torch.long, device=device),
                                     sequence_length=0, max_cache_len=int(kv_bucket))
            stream = torch.cuda.Stream(device=device)
            logits = self.capture(input_ids=first, position_ids=first * 0, attention_mask=None,
                                  cache_position=cache.cache_position, past_key_values=cache, logical_kv_len=0,
                                  kv_bucket=int(kv_bucket), tactic_name="decode_step_sm100_persistent_v1",
                                  stream_ptr=int(stream.cuda_stream), stream=stream)
        else:
            self.plan.reset_cache()
            logits = self.replay(next_token=first, position_ids=first * 0, cache_position=0, logical_kv_len=0,
                                 stream_ptr=self.contract.stream_ptr)
        sp = self.contract.stream_ptr
        out: list[int] = []
        i = 1
        while len(out) < int(new_tokens):
            if i < len(prompt):
                tok = torch.tensor([[int(prompt[i])]], dtype=torch.long, device=device)
            else:
                tok = torch.argmax(logits[:, -1, :], dim=-1, keepdim=True)
                out.append(int(tok.item()))
                if len(out) == int(new_tokens):
                    break
            pos = torch.tensor([[i]], dtype=torch.long, device=device)
            logits = self.replay(next_token=tok, position_ids=pos, cache_position=i, logical_kv_len=i, stream_ptr=sp)
            i += 1
        return out

    def invalidate(self, reason: str) -> None:
        try:
            self.bridge.reset_graph()
        except NativeCudaError:
            pass
        if self.plan is not None:
            self.plan.graph_plan.invalidate()
        self.plan = None
        self.contract = None
        self.status = "fallback"
        self.reason = str(reason)
