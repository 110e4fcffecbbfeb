"""NF4 batch-1 decode engine for Qwen2/Llama-architecture models on sm_100a.

One decode step (one token) is the op sequence below, every op a C-ABI call
into the sm_100a library:

    embedding[token]                          -> x (bf16 residual stream)
    per layer:
      RMSNorm + NF4 q/k/v (+bias) + RoPE + KV append at pos   (1 kernel)
      split-KV GQA over kv_len = pos + 1, last CTA combines    (1 kernel)
      NF4 o_proj + residual add                               (1 kernel)
      RMSNorm + NF4 gate/up + SwiGLU                          (1 kernel)
      NF4 down_proj + residual add                            (1 kernel)
    final RMSNorm + tied bf16 lm_head + argmax                (1 kernel)
    advance: token <- argmax, pos += 1                        (1 kernel)

The whole step is captured once into a CUDA graph through the reference's
graph ABI (kudacuda_begin_capture / end_capture / replay_graph) and replayed
per token; every kernel is launched with programmatic dependent launch so its
weight streaming starts while the previous kernel finishes.  All buffers are
allocated before capture and never move, so the graph key (pointer identity,
python/kudacuda_graph_plan.py:14-28 of the reference) stays valid.

The per-token state lives on the device as int32 {token, position, kv_len}.
The host either leaves the loop on the device (replay N times, read the token
history once) or drives it step by step through
kudacuda_sm100_graph_step_host (host token in, host token out), which is the
reference benchmark's per-token loop (tools/benchmark/benchmark_gemma.py:328-352).

Tensor parallelism (Megatron-style: column-parallel q/k/v/gate/up, row-parallel
o/down, sum-allreduce of the partial residual update) is provided by
kudacuda_b200.tensor_parallel on top of the same plan.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field, replace
from typing import Any, Optional

from .kudacuda_graph_plan import DecodeGraphKey, KudaCudaGraphPlan
from .kudacuda_sidecar import KudaCudaBridge, NativeCudaError


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    hidden: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    eps: float
    qkv_bias: bool
    tie_embeddings: bool

    @property
    def q_out(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def kv_out(self) -> int:
        return self.kv_heads * self.head_dim

    def nf4_layer_params(self) -> int:
        h, i = self.hidden, self.intermediate
        return h * self.q_out + 2 * h * self.kv_out + self.q_out * h + 2 * h * i + i * h

    def weight_bytes_per_token(self) -> dict[str, int]:
        """Algorithmic bytes read per decode token (weights; KV separate)."""

        p = self.nf4_layer_params() * self.layers
        nf4 = p // 2 + p // 16  # packed nibbles + fp32 absmax per 64
        lm = self.vocab * self.hidden * 2 if self.tie_embeddings else (self.vocab * self.hidden * 9) // 16
        norms = self.layers * 2 * self.hidden * 2 + self.hidden * 2
        bias = self.layers * (self.q_out + 2 * self.kv_out) * 2 if self.qkv_bias else 0
        return {"nf4_absmax": nf4, "lm_head": lm, "norms_bias": norms + bias}

    def kv_bytes_per_token(self, kv_len: int) -> int:
        # K and V rows of every layer up to kv_len, plus the appended row
        return self.layers * 2 * self.kv_heads * self.head_dim * 2 * (kv_len + 1)


QWEN25_3B = DecoderConfig("qwen2.5-3b", 2048, 36, 16, 2, 128, 11008, 151936, 1.0e6, 1.0e-6, True, True)
LLAMA3_8B = DecoderConfig("llama-3-8b", 4096, 32, 32, 8, 128, 14336, 128256, 5.0e5, 1.0e-5, False, False)


def tiny_config(layers: int = 2, vocab: int = 4096) -> DecoderConfig:
    """Config-1/2 layer shapes with few layers and a small vocabulary (tests)."""

    return replace(QWEN25_3B, name=f"qwen2.5-3b-{layers}l", layers=layers, vocab=vocab)


@dataclass
class NF4Linear:
    packed: Any  # uint8 [rows * k / 2, 1] (bitsandbytes Params4bit storage)
    absmax: Any  # float32 [rows * k / 64]
    rows: int
    k: int

    def as_tuple(self, bias: Any = None) -> tuple:
        return (self.packed, self.absmax, bias)


@dataclass
class LayerWeights:
    in_norm: Any
    post_norm: Any
    q: NF4Linear
    k: NF4Linear
    v: NF4Linear
    o: NF4Linear
    gate: NF4Linear
    up: NF4Linear
    down: NF4Linear
    q_bias: Any = None
    k_bias: Any = None
    v_bias: Any = None


@dataclass
class ModelWeights:
    config: DecoderConfig
    layers: list[LayerWeights]
    embedding: Any  # bf16 [vocab, hidden]
    final_norm: Any  # bf16 [hidden]
    lm_head: Optional[NF4Linear] = None  # untied NF4 lm_head (Llama)


def _randn_bf16(torch: Any, shape: tuple, std: float, gen: Any, device: Any, mean: float = 0.0) -> Any:
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    return (t * std + mean).to(torch.bfloat16)


def quantize_nf4(bridge: KudaCudaBridge, torch: Any, w_bf16: Any, stream_ptr: int) -> NF4Linear:
    rows, k = int(w_bf16.shape[0]), int(w_bf16.shape[1])
    n = rows * k
    packed = torch.empty((n // 2, 1), dtype=torch.uint8, device=w_bf16.device)
    absmax = torch.empty((n // 64,), dtype=torch.float32, device=w_bf16.device)
    bridge.dispatch_nf4_quantize(w_bf16.contiguous(), packed, absmax, stream_ptr=stream_ptr)
    return NF4Linear(packed, absmax, rows, k)


@dataclass(frozen=True)
class TPShard:
    """This rank's (start, count) along each tensor-parallel dimension
    (Megatron-style): ``q`` -- q_proj rows and o_proj K (heads x head_dim);
    ``kv`` -- k/v rows; ``inter`` -- gate/up rows and down K; ``vocab`` --
    lm_head rows (vocab-parallel)."""

    q: tuple[int, int]
    kv: tuple[int, int]
    inter: tuple[int, int]
    vocab: tuple[int, int]


def tp_shard(config: DecoderConfig, rank: int, world: int) -> TPShard:
    """The slices rank ``rank`` of ``world`` holds.  Row-parallel K slices
    (o_proj, down) fall on 64-element NF4 block boundaries, so a shard's codes
    and absmax are exactly the full matrix's."""

    c = config
    if not 0 <= rank < world or c.q_heads % world or c.kv_heads % world or c.intermediate % world or c.vocab % world:
        raise ValueError(f"tensor parallelism over {world} ranks needs q_heads, kv_heads, intermediate and vocab "
                         f"divisible by {world}")
    qn, kvn, il, vl = (c.q_heads // world) * c.head_dim, (c.kv_heads // world) * c.head_dim, c.intermediate // world, \
        c.vocab // world
    if qn % 64 or il % 64:
        raise ValueError("row-parallel K slices must be multiples of the NF4 block (64)")
    return TPShard(q=(rank * qn, qn), kv=(rank * kvn, kvn), inter=(rank * il, il), vocab=(rank * vl, vl))


def shard_rows(w: Any, sl: tuple[int, int]) -> Any:
    """Column-parallel slice: rows [start, start + count) (torch or numpy)."""

    return w[sl[0]:sl[0] + sl[1]]


def shard_cols(w: Any, sl: tuple[int, int]) -> Any:
    """Row-parallel slice: K columns [start, start + count) (torch or numpy)."""

    return w[:, sl[0]:sl[0] + sl[1]]


def random_weights(bridge: KudaCudaBridge, config: DecoderConfig, *, seed: int = 20260824, device: Any = "cuda:0",
                   torch_module: Any = None, shard: tuple[int, int] = (0, 1)) -> ModelWeights:
    """Synthetic weights of the BASELINE distribution: linears N(0, 0.02) in
    bf16, NF4-quantised (blocksize 64) on the device by the library's own
    quantiser; norms 1 + N(0, 0.02); q/k/v biases N(0, 0.02); embedding
    N(0, 0.02).  ``shard=(rank, world)`` keeps only this rank's tensor-parallel
    slices (column-parallel q/k/v/gate/up, row-parallel o/down), generated
    from the full matrices so every world size sees the same model."""

    if torch_module is None:
        import torch as torch_module
    torch = torch_module
    rank, world = shard
    gen = torch.Generator(device=device)
    gen.manual_seed(int(seed))
    stream_ptr = int(torch.cuda.current_stream(device).cuda_stream)
    c = config
    sh = tp_shard(c, rank, world)

    def cols(w: Any, sl: tuple[int, int]) -> Any:
        return shard_cols(w, sl).contiguous()

    def rows(w: Any, sl: tuple[int, int]) -> Any:
        return shard_rows(w, sl).contiguous()

    layers = []
    for _ in range(c.layers):
        in_norm = _randn_bf16(torch, (c.hidden,), 0.02, gen, device, 1.0)
        post_norm = _randn_bf16(torch, (c.hidden,), 0.02, gen, device, 1.0)
        wq = _randn_bf16(torch, (c.q_out, c.hidden), 0.02, gen, device)
        wk = _randn_bf16(torch, (c.kv_out, c.hidden), 0.02, gen, device)
        wv = _randn_bf16(torch, (c.kv_out, c.hidden), 0.02, gen, device)
        wo = _randn_bf16(torch, (c.hidden, c.q_out), 0.02, gen, device)
        wg = _randn_bf16(torch, (c.intermediate, c.hidden), 0.02, gen, device)
        wu = _randn_bf16(torch, (c.intermediate, c.hidden), 0.02, gen, device)
        wd = _randn_bf16(torch, (c.hidden, c.intermediate), 0.02, gen, device)
        biases = [None, None, None]
        if c.qkv_bias:
            biases = [_randn_bf16(torch, (n,), 0.02, gen, device) for n in (c.q_out, c.kv_out, c.kv_out)]
        layers.append(
            LayerWeights(
                in_norm=in_norm,
                post_norm=post_norm,
                q=quantize_nf4(bridge, torch, rows(wq, sh.q), stream_ptr),
                k=quantize_nf4(bridge, torch, rows(wk, sh.kv), stream_ptr),
                v=quantize_nf4(bridge, torch, rows(wv, sh.kv), stream_ptr),
                o=quantize_nf4(bridge, torch, cols(wo, sh.q), stream_ptr),
                gate=quantize_nf4(bridge, torch, rows(wg, sh.inter), stream_ptr),
                up=quantize_nf4(bridge, torch, rows(wu, sh.inter), stream_ptr),
                down=quantize_nf4(bridge, torch, cols(wd, sh.inter), stream_ptr),
                q_bias=None if biases[0] is None else rows(biases[0], sh.q),
                k_bias=None if biases[1] is None else rows(biases[1], sh.kv),
                v_bias=None if biases[2] is None else rows(biases[2], sh.kv),
            )
        )
        del wq, wk, wv, wo, wg, wu, wd
    embedding = _randn_bf16(torch, (c.vocab, c.hidden), 0.02, gen, device)
    final_norm = _randn_bf16(torch, (c.hidden,), 0.02, gen, device, 1.0)
    lm_head = None
    if not c.tie_embeddings:  # vocab-parallel: this rank's rows of the NF4 lm_head
        w_lm = _randn_bf16(torch, (c.vocab, c.hidden), 0.02, gen, device)
        lm_head = quantize_nf4(bridge, torch, rows(w_lm, sh.vocab), stream_ptr)
        del w_lm
    torch.cuda.synchronize(device)
    return ModelWeights(c, layers, embedding, final_norm, lm_head)


def rope_tables(torch: Any, max_pos: int, head_dim: int, theta: float, device: Any) -> tuple[Any, Any]:
    """Transformers' default RoPE tables (Qwen2RotaryEmbedding / LlamaRotaryEmbedding):
    inv_freq = 1 / theta^(2i/d) in fp32, freqs = pos * inv_freq, cos/sin rounded to
    bf16; the first d/2 columns (emb = cat(freqs, freqs))."""

    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = torch.outer(torch.arange(max_pos, dtype=torch.float32), inv_freq.float())
    return (freqs.cos().to(torch.bfloat16).contiguous().to(device), freqs.sin().to(torch.bfloat16).contiguous().to(device))


class TensorParallel:
    """Row-parallel reductions and the vocab-parallel NF4 lm_head of a
    tensor-parallel decode step (Megatron-style sharding: column-parallel
    q/k/v and gate/up, row-parallel o_proj and down).

    * ``residual_linear``: the row-parallel GEMV writes this rank's fp32
      partial, an allreduce(sum) adds the ranks' partials, and the residual
      add applies the single-GPU epilogue's roundings:
      ``x = bf16(x + bf16(sum))``.
    * ``lm_head``: RMSNorm + NF4 GEMV over this rank's vocabulary rows (fp32
      logits), local argmax on bf16-rounded logits, allgather of the
      (value, index) pairs, lowest-index maximum -> next token.

    ``group`` is a torch.distributed process group (NCCL for GPUs) or None
    for one rank; collectives run on the decode stream so they are captured
    in the step's CUDA graph.
    """

    def __init__(self, plan: "StaticDecodePlan", *, rank: int = 0, world: int = 1, group: Any = None) -> None:
        torch = plan.torch
        self.rank, self.world, self.group = int(rank), int(world), group
        c, dev = plan.config, plan.device
        self.partial = torch.zeros(c.hidden, dtype=torch.float32, device=dev)
        lm = plan.weights.lm_head
        self.v_loc = lm.rows if lm is not None else 0
        self.logits = torch.zeros(max(self.v_loc, 1), dtype=torch.float32, device=dev)
        br = plan.bridge
        self.arg_ws = torch.zeros(br.argmax_workspace_bytes() // 4, dtype=torch.float32, device=dev)
        self.arg_ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pair = torch.zeros(2, dtype=torch.int32, device=dev)  # {float value bits, int32 index}
        self.gathered = torch.zeros(2 * self.world, dtype=torch.int32, device=dev)

    def _allreduce(self, t: Any) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, group=self.group)

    def residual_linear(self, plan: "StaticDecodePlan", x: Any, lin: "NF4Linear", stream_ptr: int) -> int:
        br = plan.bridge
        if self.world == 1:
            br.dispatch_nf4_linear_residual(x, lin.packed, lin.absmax, plan.buffers.x, rows=lin.rows, k=lin.k,
                                            stream_ptr=stream_ptr)
            return 1
        br.dispatch_nf4_gemv(x, lin.packed, lin.absmax, self.partial, rows=lin.rows, k=lin.k, stream_ptr=stream_ptr)
        self._allreduce(self.partial)
        br.dispatch_residual_add_f32(self.partial, plan.buffers.x, stream_ptr=stream_ptr)
        return 2

    def lm_head(self, plan: "StaticDecodePlan", stream_ptr: int) -> int:
        b, w, c, br = plan.buffers, plan.weights, plan.config, plan.bridge
        br.dispatch_rmsnorm_nf4_gemv(b.x, w.final_norm, (w.lm_head.packed, w.lm_head.absmax), self.logits,
                                     epsilon=c.eps, stream_ptr=stream_ptr)
        br.dispatch_argmax_shard(self.logits, self.arg_ws, self.arg_ticket, self.pair,
                                 index_base=self.rank * self.v_loc, stream_ptr=stream_ptr)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.gathered, self.pair, group=self.group)
            br.dispatch_select_token(self.gathered, b.next_token, count=self.world, stream_ptr=stream_ptr)
        else:
            br.dispatch_select_token(self.pair, b.next_token, count=1, stream_ptr=stream_ptr)
        return 3


class _TorchGraphBridge:
    """begin/end/replay on a torch.cuda.CUDAGraph (thread-local capture), for
    steps that contain NCCL collectives issued through torch.distributed."""

    def __init__(self, torch_module: Any) -> None:
        self.torch = torch_module
        self.graph = None
        self._ctx = None

    def begin_capture(self, *, stream_ptr: int) -> None:
        torch = self.torch
        self.graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.ExternalStream(int(stream_ptr))
        self._ctx = torch.cuda.stream(stream)
        self._ctx.__enter__()
        self.graph.capture_begin(capture_error_mode="thread_local")

    def end_capture(self, *, stream_ptr: int) -> None:
        try:
            self.graph.capture_end()
        finally:
            self._ctx.__exit__(None, None, None)
            self._ctx = None

    def replay_graph(self, *, stream_ptr: int) -> None:
        torch = self.torch
        with torch.cuda.stream(torch.cuda.ExternalStream(int(stream_ptr))):
            self.graph.replay()

    def reset(self) -> None:
        self.graph = None


@dataclass
class DecodeBuffers:
    state: Any  # int32 [4]: token, position, kv_len, (pad)
    x: Any  # bf16 [hidden]
    q: Any  # bf16 [q_heads * d]
    attn: Any  # bf16 [q_heads * d]
    h: Any  # bf16 [intermediate]
    kcache: Any  # bf16 [layers, kv_heads, cap, d]
    vcache: Any
    gqa_ws: Any
    gqa_tickets: Any
    gqa_ws_bytes: int
    lm_ws: Any
    lm_ticket: Any
    logits: Any  # bf16 [vocab]
    next_token: Any  # int32 [1]
    history: Any  # int32 [max_tokens]
    rope_cos: Any
    rope_sin: Any
    lm_scratch: Any = None  # f32 logits for an NF4 lm_head


class LayerCaches:
    """Caller-owned per-layer K (or V) caches as one indexable object: item
    ``li`` is layer li's [kv_heads, cap, head_dim] bf16 view (the tensors may
    be [1, kv_heads, cap, head_dim], as Transformers' caches are);
    ``zero_()`` clears every layer."""

    def __init__(self, tensors: list) -> None:
        self.layers = [t.view(t.shape[-3], t.shape[-2], t.shape[-1]) for t in tensors]

    def __getitem__(self, i: int) -> Any:
        return self.layers[i]

    def __len__(self) -> int:
        return len(self.layers)

    @property
    def shape(self) -> tuple:
        return (len(self.layers), *tuple(self.layers[0].shape))

    def zero_(self) -> "LayerCaches":
        for t in self.layers:
            t.zero_()
        return self

    def data_ptrs(self) -> list[int]:
        return [int(t.data_ptr()) for t in self.layers]


def _buffer_ptrs(t: Any) -> list[int]:
    return t.data_ptrs() if isinstance(t, LayerCaches) else [int(t.data_ptr())]


class TPExchange:
    """The exchange buffers of the tensor-parallel row-split kernel: every rank
    allocates one (kudacuda_sm100_tp_exchange_bytes: o_proj then down partials,
    [world][hidden] tagged words each, zeroed once), exports a CUDA IPC
    handle, gathers the others' handles over the process group and maps them;
    ``peers`` is the device table of the world buffer addresses as this
    process sees them (plain peer memory over NVLink, no multicast object).
    ``close`` is collective: every rank unmaps the peers' buffers, then frees
    its own."""

    def __init__(self, bridge: KudaCudaBridge, torch: Any, *, rank: int, world: int, group: Any, hidden: int,
                 device: Any) -> None:
        import torch.distributed as dist

        self.bridge, self.rank, self.world, self.group = bridge, int(rank), int(world), group
        nbytes = bridge.tp_exchange_bytes(world, hidden)
        self.own, handle = bridge.ipc_alloc(nbytes)
        handles: list[Any] = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        addrs = []
        self.opened: list[int] = []
        for p_, h in enumerate(handles):
            if p_ == self.rank:
                addrs.append(self.own)
            else:
                ptr = bridge.ipc_open(h)
                self.opened.append(ptr)
                addrs.append(ptr)
        self.peers = torch.tensor(addrs, dtype=torch.int64, device=device)
        self.closed = False

    def close(self) -> None:
        if self.closed:
            return
        import torch.distributed as dist

        dist.barrier(group=self.group)
        for ptr in self.opened:
            self.bridge.ipc_close(ptr, owned=False)
        dist.barrier(group=self.group)
        self.bridge.ipc_close(self.own, owned=True)
        self.closed = True


class PersistentLayers:
    """Device data of the persistent decode path for one plan: every layer's
    q/k/v, o, gate/up and down weights copied once into the stream layout of
    the persistent kernel (the bitsandbytes tensors stay as they are for the
    per-op ABI), the device layer table and the kernel's self-resetting
    scratch.

    ``layout="rows"`` (default): kudacuda_sm100_decode_layers_rows -- 16-row
    tiles, each owned by one CTA that finishes its rows (576-byte units from
    kudacuda_sm100_nf4_retile16).  ``layout="groups"``:
    kudacuda_sm100_decode_layers_persistent -- 64-row groups split over CTAs
    along K, partial sums summed by the consumers."""

    SLOTS = 16

    def __init__(self, plan: "StaticDecodePlan", layout: str = "rows", exchange: Optional[TPExchange] = None) -> None:
        if layout not in ("rows", "groups"):
            raise ValueError(f"unknown persistent layout {layout!r}")
        if exchange is not None and layout != "rows":
            raise NativeCudaError("tensor parallelism runs on the row-split persistent kernel only")
        self.exchange = exchange
        torch = plan.torch
        br, c, w, b = plan.bridge, plan.config, plan.weights, plan.buffers
        dev = plan.device
        self.plan = plan
        self.layout = layout
        sp = int(torch.cuda.current_stream(dev).cuda_stream)
        d = c.head_dim
        self.tiles: list[tuple[Any, ...]] = []
        table = torch.zeros((c.layers, self.SLOTS), dtype=torch.int64)
        for li, L in enumerate(w.layers):
            ops = (
                (br.RETILE_QKV_ROPE, [(L.q.packed, L.q.absmax, L.q.rows), (L.k.packed, L.k.absmax, L.k.rows),
                                      (L.v.packed, L.v.absmax, L.v.rows)], L.q.k),
                (br.RETILE_PLAIN, [(L.o.packed, L.o.absmax, L.o.rows)], L.o.k),
                (br.RETILE_SWIGLU, [(L.gate.packed, L.gate.absmax, L.gate.rows),
                                    (L.up.packed, L.up.absmax, L.up.rows)], L.gate.k),
                (br.RETILE_PLAIN, [(L.down.packed, L.down.absmax, L.down.rows)], L.down.k),
            )
            row: list[int] = []
            for mode, mats, k in ops:
                rows = tuple(m[2] for m in mats) + (0,) * (3 - len(mats))
                if layout == "rows":
                    tiles = br.retile16_tiles(mode, rows, d)
                    if tiles < 1:
                        raise NativeCudaError(f"persistent decode cannot re-tile layer {li} (mode {mode}, rows {rows})")
                    units = torch.empty(tiles * (k // 64) * 576, dtype=torch.uint8, device=dev)
                    br.dispatch_nf4_retile16(mode, mats, units, k=k, head_dim=d, stream_ptr=sp)
                    self.tiles.append((units,))
                    row.append(units.data_ptr())
                else:
                    groups = br.retile_groups(mode, rows, d)
                    if groups < 1:
                        raise NativeCudaError(f"persistent decode cannot re-tile layer {li} (mode {mode}, rows {rows})")
                    codes = torch.empty(groups * 64 * k // 2, dtype=torch.uint8, device=dev)
                    absm = torch.empty(groups * 64 * k // 64, dtype=torch.float32, device=dev)
                    br.dispatch_nf4_retile(mode, mats, codes, absm, k=k, head_dim=d, stream_ptr=sp)
                    self.tiles.append((codes, absm))
                    row += [codes.data_ptr(), absm.data_ptr()]
            ptr = lambda t: 0 if t is None else int(t.data_ptr())  # noqa: E731
            row += [ptr(L.in_norm), ptr(L.post_norm), ptr(L.q_bias), ptr(L.k_bias), ptr(L.v_bias),
                    int(b.kcache[li].data_ptr()), int(b.vcache[li].data_ptr())]
            row += [0] * (self.SLOTS - len(row))
            table[li] = torch.tensor(row, dtype=torch.int64)
        self.table = table.to(dev)
        dims = dict(layers=c.layers, hidden=c.hidden, q_heads=plan.q_heads, kv_heads=plan.kv_heads, head_dim=d,
                    intermediate=plan.inter, kv_capacity=plan.kv_bucket)
        nbytes = br.rows_scratch_bytes(**dims) if layout == "rows" else br.persistent_scratch_bytes(**dims)
        self.scratch = torch.zeros((nbytes + 3) // 4, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)

    # the row-split kernel's launch counter (the tags' epoch): int32 word 2 of its scratch
    _EPOCH_WORD = 2

    def epoch(self) -> int:
        if self.layout != "rows":
            raise NativeCudaError("only the row-split kernel keeps a launch epoch")
        return int(self.scratch[self._EPOCH_WORD].item())

    def set_epoch(self, value: int) -> None:
        """Recovery after a step that did not run on every rank (tensor
        parallelism): the ranks agree on one epoch above every rank's own --
        for example the max over ranks plus one -- so that no word written
        before the failure carries a tag a later step expects."""

        if self.layout != "rows":
            raise NativeCudaError("only the row-split kernel keeps a launch epoch")
        self.plan.torch.cuda.synchronize(self.plan.device)
        self.scratch[self._EPOCH_WORD] = int(value)
        self.plan.torch.cuda.synchronize(self.plan.device)

    def pointers(self) -> list[int]:
        out = [int(self.table.data_ptr()), int(self.scratch.data_ptr())]
        if self.exchange is not None:
            out.append(int(self.exchange.peers.data_ptr()))
        for tensors in self.tiles:
            out += [int(t.data_ptr()) for t in tensors]
        return out

    def record(self, stream_ptr: int, *, taps: Any = None, spin_limit: int = 0, stall_counter: int = -1) -> int:
        """Launch the kernel (one launch).  ``taps``/``spin_limit``/``stall_counter``
        are the kernel's test hooks."""

        p, b, c = self.plan, self.plan.buffers, self.plan.config
        kw = dict(layers=c.layers, max_pos=int(b.rope_cos.shape[0]), hidden=c.hidden, q_heads=p.q_heads,
                  kv_heads=p.kv_heads, head_dim=c.head_dim, intermediate=p.inter, kv_capacity=p.kv_bucket,
                  epsilon=c.eps, scale=1.0 / math.sqrt(c.head_dim), stream_ptr=stream_ptr, taps=taps,
                  spin_limit=spin_limit, stall_counter=stall_counter)
        if self.exchange is not None:
            if taps is not None or spin_limit or stall_counter != -1:
                raise NativeCudaError("the tensor-parallel persistent launch has no test hooks")
            for k in ("taps", "spin_limit", "stall_counter"):
                kw.pop(k)
            ex = self.exchange
            p.bridge.dispatch_decode_layers_rows_tp(self.table, b.x, b.state, b.rope_cos, b.rope_sin, self.scratch,
                                                    world=ex.world, rank=ex.rank, peers=ex.peers, **kw)
        elif self.layout == "rows":
            p.bridge.dispatch_decode_layers_rows(self.table, b.x, b.state, b.rope_cos, b.rope_sin, self.scratch, **kw)
        else:
            p.bridge.dispatch_decode_layers_persistent(self.table, b.x, b.state, b.rope_cos, b.rope_sin, self.scratch,
                                                       **kw)
        return 1

    def tap_layout(self) -> dict[str, tuple[int, int]]:
        """(offset, length) of each intermediate in one layer's tap record."""

        p, c = self.plan, self.plan.config
        names = (("xn", c.hidden), ("q", p.q_heads * c.head_dim), ("k", p.kv_heads * c.head_dim),
                 ("v", p.kv_heads * c.head_dim), ("att", p.q_heads * c.head_dim), ("x1", c.hidden),
                 ("xn2", c.hidden), ("h", p.inter), ("x2", c.hidden))
        out, off = {}, 0
        for n, ln in names:
            out[n] = (off, ln)
            off += ln
        out["stride"] = (off, 0)
        return out

    def new_taps(self) -> Any:
        p, c = self.plan, self.plan.config
        n = p.bridge.persistent_tap_elements(layers=c.layers, hidden=c.hidden, q_heads=p.q_heads,
                                             kv_heads=p.kv_heads, head_dim=c.head_dim, intermediate=p.inter)
        assert n == c.layers * self.tap_layout()["stride"][0]
        return p.torch.zeros(n, dtype=p.torch.bfloat16, device=p.device)



class StaticDecodePlan:
    """Fixed-shape decode step for one model on one device: buffers, the op
    sequence, and its CUDA graph.  ``kv_bucket`` is the cache capacity (the
    reference's graph KV bucket, python/kudacuda_static_decode.py:100-145)."""

    def __init__(self, bridge: KudaCudaBridge, weights: ModelWeights, *, kv_bucket: int = 512,
                 max_tokens: Optional[int] = None, device: Any = "cuda:0", torch_module: Any = None,
                 allreduce: Any = None, keep_logits: bool = True, persistent: bool = False,
                 kv_cache: Optional[tuple[list, list]] = None, persistent_layout: str = "rows") -> None:
        """``kv_cache=(keys, values)``: caller-owned per-layer caches (bf16,
        contiguous, [1 or absent, kv_heads, kv_bucket, head_dim]) used in
        place of the plan's own -- e.g. a Transformers prefill cache."""
        if torch_module is None:
            import torch as torch_module
        self.torch = torch_module
        self.bridge = bridge
        self.weights = weights
        self.config = weights.config
        self.device = device
        self.kv_bucket = int(kv_bucket)
        self.allreduce = allreduce  # (rank, world, process group) for tensor parallelism, or None
        self.keep_logits = keep_logits
        torch = self.torch
        c = self.config
        L0 = weights.layers[0]
        self.q_heads = L0.q.rows // c.head_dim
        self.kv_heads = L0.k.rows // c.head_dim
        self.inter = L0.gate.rows
        max_tokens = int(max_tokens or self.kv_bucket)
        bf16 = torch.bfloat16
        cap = self.kv_bucket
        ws, tickets, nbytes = bridge.gqa_workspace(batch=1, query_heads=self.q_heads, kv_heads=self.kv_heads,
                                                   kv_extent=cap, device=device, torch_module=torch)
        lm_bytes = bridge.lm_head_workspace_bytes()
        cos, sin = rope_tables(torch, max(cap, max_tokens) + 1, c.head_dim, c.rope_theta, device)
        if kv_cache is None:
            kcache = torch.zeros((c.layers, self.kv_heads, cap, c.head_dim), dtype=bf16, device=device)
            vcache = torch.zeros((c.layers, self.kv_heads, cap, c.head_dim), dtype=bf16, device=device)
        else:
            keys, values = (list(t) for t in kv_cache)
            want = (self.kv_heads, cap, c.head_dim)
            if len(keys) != c.layers or len(values) != c.layers:
                raise NativeCudaError(f"kv_cache needs {c.layers} key and value tensors")
            for t in keys + values:
                if (t.dtype != bf16 or not t.is_contiguous() or tuple(t.shape[-3:]) != want or
                        (t.dim() == 4 and int(t.shape[0]) != 1) or t.dim() not in (3, 4) or
                        t.device != torch.device(device)):
                    raise NativeCudaError(f"kv_cache tensors must be contiguous bf16 [1, {want[0]}, {want[1]}, "
                                          f"{want[2]}] on {device}; got {tuple(t.shape)} {t.dtype} {t.device}")
            kcache, vcache = LayerCaches(keys), LayerCaches(values)
        self.buffers = DecodeBuffers(
            state=torch.zeros(4, dtype=torch.int32, device=device),
            x=torch.zeros(c.hidden, dtype=bf16, device=device),
            q=torch.zeros(self.q_heads * c.head_dim, dtype=bf16, device=device),
            attn=torch.zeros(self.q_heads * c.head_dim, dtype=bf16, device=device),
            h=torch.zeros(self.inter, dtype=bf16, device=device),
            kcache=kcache,
            vcache=vcache,
            gqa_ws=ws,
            gqa_tickets=tickets,
            gqa_ws_bytes=nbytes,
            lm_ws=torch.zeros(lm_bytes // 4, dtype=torch.float32, device=device),
            lm_ticket=torch.zeros(1, dtype=torch.int32, device=device),
            logits=torch.zeros(c.vocab, dtype=bf16, device=device),
            next_token=torch.zeros(1, dtype=torch.int32, device=device),
            history=torch.zeros(max_tokens, dtype=torch.int32, device=device),
            rope_cos=cos,
            rope_sin=sin,
        )
        self.graph_plan = KudaCudaGraphPlan(bridge)
        self.graph_key: Optional[DecodeGraphKey] = None
        self.launches_per_step = 0
        # tensor parallelism / untied NF4 lm_head: ``allreduce`` may be a
        # (rank, world, group) tuple; steps with collectives are captured as a
        # torch CUDA graph (thread-local capture) instead of the handle's graph
        self.tp: Optional[TensorParallel] = None
        if allreduce is not None or weights.lm_head is not None:
            rank, world, group = allreduce if isinstance(allreduce, tuple) else (0, 1, None)
            self.tp = TensorParallel(self, rank=rank, world=world, group=group)
        self._torch_graph = _TorchGraphBridge(torch_module) if self.tp is not None and self.tp.world > 1 else None
        if self._torch_graph is not None:
            self.graph_plan = KudaCudaGraphPlan(self._torch_graph)
        # persistent path: all layers of a step in one cooperative launch over
        # weights re-tiled once into the kernel's stream layout
        self.persistent: Optional[PersistentLayers] = None
        self.tp_exchange: Optional[TPExchange] = None
        if persistent:
            if self.tp is not None and self.tp.world > 1:
                # o_proj / down partials are exchanged inside the kernel (peer memory)
                self.tp_exchange = TPExchange(bridge, torch, rank=self.tp.rank, world=self.tp.world,
                                              group=self.tp.group, hidden=c.hidden, device=device)
            self.persistent = PersistentLayers(self, layout=persistent_layout, exchange=self.tp_exchange)

    @property
    def captured(self) -> bool:
        return self.graph_plan.captured

    def release_source_weights(self) -> int:
        """Free the bitsandbytes copies of the decoder layers' NF4 tensors of a
        persistent plan, whose step streams only its own re-tiled copy; until
        then the plan holds the layer weights twice.  Build every other
        consumer of the source weights first (a BatchedPrefill re-tiles its own
        copy at construction): afterwards the tensors are empty and any later
        use of them (the per-op path, a new prefill) fails the NF4 shape
        checks.  Returns the bytes released."""

        if self.persistent is None:
            raise NativeCudaError("release_source_weights: only a persistent plan streams its own weight copy")
        freed = 0
        for L in self.weights.layers:
            for name in ("q", "k", "v", "o", "gate", "up", "down"):
                lin = getattr(L, name)
                freed += lin.packed.numel() * lin.packed.element_size() + lin.absmax.numel() * lin.absmax.element_size()
                lin.packed = lin.packed.new_empty((0,))
                lin.absmax = lin.absmax.new_empty((0,))
        return int(freed)

    def make_graph_key(self) -> DecodeGraphKey:
        """The static contract of the captured step: shapes, bucket and every
        device pointer the graph bakes in (buffers, caches, weights)."""

        b, w, c = self.buffers, self.weights, self.config
        ptrs = [p for t in (b.state, b.x, b.q, b.attn, b.h, b.kcache, b.vcache, b.gqa_ws, b.gqa_tickets,
                            b.lm_ws, b.lm_ticket, b.logits, b.next_token, b.history, b.rope_cos, b.rope_sin,
                            w.embedding, w.final_norm) for p in _buffer_ptrs(t)]
        if self.persistent is not None:
            ptrs += self.persistent.pointers()
        for L in w.layers:
            ptrs += [L.in_norm.data_ptr(), L.post_norm.data_ptr()]
            if self.persistent is None:  # the persistent step reads only its re-tiled copy
                for lin in (L.q, L.k, L.v, L.o, L.gate, L.up, L.down):
                    ptrs += [lin.packed.data_ptr(), lin.absmax.data_ptr()]
            ptrs += [0 if t is None else t.data_ptr() for t in (L.q_bias, L.k_bias, L.v_bias)]
        d = c.head_dim
        return DecodeGraphKey(
            device_id=int(self.torch.device(self.device).index or 0),
            tactic_name=("decode_step_sm100_v1" if self.persistent is None else
                         f"decode_step_sm100_persistent_{self.persistent.layout}_v1"),
            layer_count=c.layers,
            query_shape=(1, self.q_heads, 1, d),
            key_shape=(1, self.kv_heads, self.kv_bucket, d),
            value_shape=(1, self.kv_heads, self.kv_bucket, d),
            output_shape=(1, self.q_heads, 1, d),
            kv_bucket=self.kv_bucket,
            pointers=tuple(int(p) for p in ptrs),
            model_fingerprint=c.name,
            dtype="bfloat16",
            quantization="nf4-blocksize64-fp32absmax",
        )

    # ------------------------------------------------------------------ one step
    def record(self, stream_ptr: int) -> int:
        """Enqueue one decode step on the stream; returns the number of kernels."""

        b, c, w, br = self.buffers, self.config, self.weights, self.bridge
        pos_dev = b.state[1:2]
        kvlen_dev = b.state[2:3]
        n = 0
        br.dispatch_embedding(w.embedding, b.state[0:1], b.x, stream_ptr=stream_ptr)
        n += 1
        scale = 1.0 / math.sqrt(c.head_dim)
        if self.persistent is not None:
            n += self.persistent.record(stream_ptr)
            n += self._lm_head(stream_ptr)
            br.dispatch_decode_advance(b.state, b.next_token, history=b.history, stream_ptr=stream_ptr)
            n += 1
            self.launches_per_step = n
            return n
        for li, L in enumerate(w.layers):
            kc, vc = b.kcache[li], b.vcache[li]
            br.dispatch_attention_input(b.x, L.in_norm, L.q.as_tuple(L.q_bias), L.k.as_tuple(L.k_bias),
                                        L.v.as_tuple(L.v_bias), b.rope_cos, b.rope_sin, pos_dev, b.q, kc, vc,
                                        q_heads=self.q_heads, kv_heads=self.kv_heads, head_dim=c.head_dim,
                                        kv_capacity=self.kv_bucket, epsilon=c.eps, stream_ptr=stream_ptr)
            br.dispatch_gqa_decode_splitkv(b.q, kc, vc, b.attn, b.gqa_ws, b.gqa_tickets, kv_len_device=kvlen_dev,
                                           batch=1, kv_len=self.kv_bucket, kv_stride=self.kv_bucket,
                                           query_heads=self.q_heads, kv_heads=self.kv_heads, scale=scale,
                                           stream_ptr=stream_ptr, workspace_bytes=b.gqa_ws_bytes)
            n += 2
            n += self._residual_linear(b.attn, L.o, stream_ptr)
            br.dispatch_swiglu_bf16(b.x, L.post_norm, (L.gate.packed, L.gate.absmax), (L.up.packed, L.up.absmax), b.h,
                                    epsilon=c.eps, stream_ptr=stream_ptr)
            n += 1
            n += self._residual_linear(b.h, L.down, stream_ptr)
        n += self._lm_head(stream_ptr)
        br.dispatch_decode_advance(b.state, b.next_token, history=b.history, stream_ptr=stream_ptr)
        n += 1
        self.launches_per_step = n
        return n

    def _residual_linear(self, x: Any, lin: NF4Linear, stream_ptr: int) -> int:
        if self.tp is None:
            self.bridge.dispatch_nf4_linear_residual(x, lin.packed, lin.absmax, self.buffers.x, rows=lin.rows, k=lin.k,
                                                     stream_ptr=stream_ptr)
            return 1
        return self.tp.residual_linear(self, x, lin, stream_ptr)

    def _lm_head(self, stream_ptr: int) -> int:
        b, w, c = self.buffers, self.weights, self.config
        if w.lm_head is None:
            self.bridge.dispatch_lm_head_argmax(b.x, w.final_norm, w.embedding, b.next_token, b.lm_ws, b.lm_ticket,
                                                logits=b.logits if self.keep_logits else None, epsilon=c.eps,
                                                stream_ptr=stream_ptr)
            return 1
        if self.tp is None:
            raise NativeCudaError("an untied NF4 lm_head needs the tensor-parallel hook")
        return self.tp.lm_head(self, stream_ptr)

    # ------------------------------------------------------------------ state
    def set_state(self, token: int, position: int, stream: Any = None) -> None:
        """Write {token, position, kv_len} to the device state, ordered after
        all work already queued on ``stream`` (and the current stream)."""

        torch = self.torch
        if stream is not None:
            stream.synchronize()
        torch.cuda.synchronize(self.device)
        self.buffers.state.copy_(torch.tensor([token, position, position + 1, 0], dtype=torch.int32),
                                 non_blocking=False)

    def reset_cache(self) -> None:
        self.torch.cuda.synchronize(self.device)
        self.buffers.kcache.zero_()
        self.buffers.vcache.zero_()
        self.torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ graph
    def capture(self, stream: Any, *, warm_position: int = 0) -> None:
        """Warm every kernel once eagerly (lazy attribute set-up), restore the
        state, then capture one step into the handle's graph.  The warm-up
        step runs token 0 at ``warm_position`` and writes that cache row, so
        a caller whose cache already holds rows passes the first row it will
        decode (the first replay rewrites it)."""

        torch = self.torch
        sp = int(stream.cuda_stream)
        saved_state = self.buffers.state.clone()
        saved_hist = self.buffers.history.clone()
        wp = int(warm_position)
        if not 0 <= wp < self.kv_bucket:
            raise NativeCudaError(f"warm_position {wp} outside the KV bucket {self.kv_bucket}")
        self.buffers.state.copy_(torch.tensor([0, wp, wp + 1, 0], dtype=torch.int32))
        torch.cuda.synchronize(self.device)
        with torch.cuda.stream(stream):
            self.record(sp)
        stream.synchronize()
        word = self.bridge.error_word(clear=True)
        if word:
            raise NativeCudaError(f"decode step raised device error word {word:#x}")
        self.buffers.state.copy_(saved_state)
        self.buffers.history.copy_(saved_hist)
        torch.cuda.synchronize(self.device)
        if self._torch_graph is None:
            self.bridge.reset_graph()
        else:
            self._torch_graph.reset()
        self.graph_plan.invalidate()
        key = self.make_graph_key()
        self.graph_plan.begin_capture(key, stream_ptr=sp)
        try:
            self.record(sp)
        except Exception:
            try:
                self.graph_plan.end_capture(key, stream_ptr=sp)
            finally:
                self.graph_plan.invalidate()
                if self._torch_graph is None:
                    self.bridge.reset_graph()
            raise
        self.graph_plan.end_capture(key, stream_ptr=sp)
        self.graph_key = key

    def replay(self, stream: Any) -> None:
        """Replay the captured step under its key (a different stream is a
        GraphContractError); ``verify_key()`` re-derives the key when the
        caller may have swapped tensors."""

        if self.graph_key is None:
            raise NativeCudaError("no captured decode graph")
        self.graph_plan.replay(self.graph_key, stream_ptr=int(stream.cuda_stream))

    def verify_key(self) -> None:
        from .kudacuda_graph_plan import GraphContractError

        if self.graph_key is None or self.make_graph_key() != self.graph_key:
            raise GraphContractError("decode graph key changed since capture (tensors were replaced)")

    # ------------------------------------------------------------------ generation
    def prefill(self, prompt: list[int], stream: Any) -> int:
        """Feed the prompt through decode steps (positions 0..n-1); returns the
        first generated token.  Requires a captured graph."""

        if not self.captured:
            raise NativeCudaError("capture the decode graph before prefill")
        if len(prompt) + 1 > self.kv_bucket:
            raise ValueError("prompt does not fit the KV bucket")
        torch = self.torch
        torch.cuda.synchronize(self.device)
        nxt = 0
        for i, tok in enumerate(prompt):
            nxt = self.step_host(int(tok), i, stream)
        return nxt

    def step_host(self, token: int, position: int, stream: Any) -> int:
        """One decode step driven from the host: state in, replay, next token
        out, all on the replay stream (so a state write never lands while the
        previous step still runs); host-synchronous.  Uses the library's
        one-call kudacuda_sm100_graph_step_host for the handle's graph."""

        torch = self.torch
        if getattr(self, "_host_in", None) is None:
            self._host_in = torch.zeros(4, dtype=torch.int32).pin_memory()
            self._host_out = torch.zeros(1, dtype=torch.int32).pin_memory()
            self._host_in_np, self._host_out_np = self._host_in.numpy(), self._host_out.numpy()
            self._bound_step, self._bound_stream = None, None
        hi, ho = self._host_in, self._host_out
        hin = self._host_in_np  # a view of the pinned buffer: no tensor indexing per step
        hin[0], hin[1], hin[2] = int(token), int(position), int(position) + 1
        sp = int(stream.cuda_stream)
        if self._torch_graph is None:
            if self._bound_stream != sp:
                self._bound_step = self.bridge.bind_graph_step_host(hi, self.buffers.state, ho, self.buffers.next_token,
                                                                    stream_ptr=sp)
                self._bound_stream = sp
            self._bound_step()
            return int(self._host_out_np[0])
        else:
            with torch.cuda.stream(stream):
                self.buffers.state.copy_(hi, non_blocking=True)
            self.replay(stream)
            with torch.cuda.stream(stream):
                ho.copy_(self.buffers.next_token, non_blocking=True)
            stream.synchronize()
        return int(ho[0])

    def generate_device(self, steps: int, stream: Any) -> None:
        """Replay the graph ``steps`` times with no host interaction; the
        generated tokens accumulate in buffers.history."""

        for _ in range(int(steps)):
            self.replay(stream)


def greedy_generate(plan: StaticDecodePlan, prompt: list[int], new_tokens: int, stream: Any) -> list[int]:
    """Prompt via decode steps, then ``new_tokens`` greedy tokens on the device."""

    stream.synchronize()
    plan.reset_cache()
    plan.buffers.history.zero_()
    first = plan.prefill(prompt, stream)
    n = len(prompt)
    if n + new_tokens > plan.buffers.history.numel() or n + new_tokens > plan.kv_bucket:
        raise ValueError("generation exceeds the KV bucket / history")
    plan.buffers.history[n] = first
    # state after prefill: token = first, position = n
    plan.generate_device(new_tokens - 1, stream)
    stream.synchronize()
    return [int(t) for t in plan.buffers.history[n:n + new_tokens].cpu().tolist()]


# ---------------------------------------------------------------------- batched decode
@dataclass
class RetiledNF4:
    data: Any  # uint8: one 4,608-byte record per 128-row tile and 64-element K block
    rows: int
    k: int


def retile_nf4(bridge: KudaCudaBridge, torch: Any, lins: list[NF4Linear], stream_ptr: int,
               interleave64: bool = False) -> RetiledNF4:
    """Row-concatenate NF4 matrices (same K) and copy them into the batched
    GEMM's streaming form (kudacuda_sm100_batch_retile).  ``interleave64``
    (two matrices of equal rows, a multiple of 64): rows 64t..64t+63 of the
    first, then the same rows of the second, tile after tile -- the order
    the fused SwiGLU GEMM wants."""

    rows = sum(l.rows for l in lins)
    k = lins[0].k
    if interleave64:
        a, b = lins
        if a.rows != b.rows or a.rows % 64:
            raise ValueError("interleaving needs two matrices of equal rows, a multiple of 64")
        g = a.rows // 64
        packed = torch.stack([a.packed.reshape(g, 64, k // 2), b.packed.reshape(g, 64, k // 2)], dim=1).reshape(-1)
        absmax = torch.stack([a.absmax.reshape(g, 64, k // 64), b.absmax.reshape(g, 64, k // 64)], dim=1).reshape(-1)
    elif len(lins) == 1:
        packed, absmax = lins[0].packed, lins[0].absmax
    else:
        packed = torch.cat([l.packed.reshape(-1) for l in lins])
        absmax = torch.cat([l.absmax.reshape(-1) for l in lins])
    out = torch.empty(bridge.batch_retile_bytes(rows, k), dtype=torch.uint8, device=packed.device)
    bridge.dispatch_batch_retile(packed, absmax, out, rows=rows, k=k, stream_ptr=stream_ptr)
    return RetiledNF4(out, rows, k)


@dataclass
class BatchedBuffers:
    state: Any  # int32 [B, 4]: token, position, kv_len, (pad) per sequence
    pos: Any  # int32 [B] (the positions, for the RoPE epilogue)
    kv_len: Any  # int32 [B] (the lengths, for attention)
    x: Any  # bf16 [B, hidden] residual stream
    xn: Any  # bf16 [n_pad, hidden] normalised activations (rows >= B stay zero)
    q: Any  # bf16 [B, q_heads * d]
    attn: Any  # bf16 [n_pad, q_heads * d]
    h: Any  # bf16 [n_pad, intermediate]
    partials: Any  # f32 split-K partial sums, shared by every GEMM of the step
    kcache: Any  # bf16 [layers, B, kv_heads, cap, d]
    vcache: Any
    gqa_ws: Any
    gqa_tickets: Any
    arg_ws: Any
    history: Any  # int32 [B, max_tokens]
    rope_cos: Any
    rope_sin: Any
    red: Any = None  # f32 [hidden, n_pad]: a row-parallel partial, allreduced (tensor parallelism)
    pairs: Any = None  # int32 [B, 2]: this rank's (value bits, index) per sequence (vocab-parallel lm_head)
    gathered: Any = None  # int32 [world, B, 2]


class BatchedDecodePlan:
    """Fixed-shape decode step for B independent sequences (each with its own
    position and KV length) on one device.  Every projection is one tensor-core
    GEMM over the padded batch (``kudacuda_sm100_batch_gemm``: NF4 dequantised
    to bf16 in shared memory, tcgen05 MMA, fp32 accumulator in TMEM) followed
    by a small epilogue; every NF4 matrix is re-tiled once at plan build into
    the GEMM's streaming form, q|k|v and gate|up concatenated so each is one
    GEMM.  The lm_head is the same GEMM over the bf16 tied
    embedding (or the NF4 lm_head), then a per-sequence argmax that advances
    each sequence's state.  The step is captured into the handle's CUDA graph.

    Arithmetic per sequence is the Transformers + bitsandbytes batched forward
    (weights dequantised to bf16, bf16 matmul with fp32 accumulation); the
    reference's sidecar admits batch 1 only (python/kudacuda_sidecar.py:145-153)."""

    TACTIC = "decode_step_sm100_batched_tcgen05_v1"
    # a fused epilogue is reduced by one CTA per tile, so only ops with few splits fuse
    FUSE_MAX_SPLITS = 2

    def __init__(self, bridge: KudaCudaBridge, weights: ModelWeights, *, batch: int, kv_bucket: int = 2048,
                 max_tokens: Optional[int] = None, device: Any = "cuda:0", torch_module: Any = None,
                 allreduce: Any = None, shared_cache: Optional[tuple] = None, fused: bool = False) -> None:
        """``shared_cache=(kcache, vcache)``, bf16 [layers, kv_heads, cap, d]:
        the batch is the tokens of ONE sequence's prompt (positions and causal
        lengths per entry), appending to and attending over that one cache --
        e.g. a StaticDecodePlan's (prefill through the batched path)."""
        if torch_module is None:
            import torch as torch_module
        self.torch = torch = torch_module
        self.bridge = bridge
        self.weights = weights
        self.config = c = weights.config
        self.device = device
        self.batch = B = int(batch)
        if not 1 <= B <= 64:
            raise ValueError("batched decode supports 1..64 sequences")
        self.n_pad = 16 if B <= 16 else (32 if B <= 32 else 64)
        self.shared = shared_cache is not None
        if self.shared:
            kv_bucket = int(shared_cache[0].shape[2])
        self.kv_bucket = cap = int(kv_bucket)
        L0 = weights.layers[0]
        self.q_heads = L0.q.rows // c.head_dim
        self.kv_heads = L0.k.rows // c.head_dim
        self.inter = L0.gate.rows
        d = c.head_dim
        max_tokens = int(max_tokens or cap)
        bf16 = torch.bfloat16
        # every projection re-tiled once into the GEMM's streaming form (one
        # contiguous record per 128-row tile and K block); q|k|v and gate|up
        # are concatenated by rows first (NF4 rows and their absmax concatenate)
        # With ``fused`` the epilogues of projections with at most
        # FUSE_MAX_SPLITS splits run inside their GEMM (the last CTA of each
        # tile's splits finishes the op), and gate|up are interleaved in 64-row
        # tiles (gate rows 64t.. then the same up rows) so one tile holds both
        # halves of its SwiGLU outputs.  Off by default: the separate epilogue
        # kernels overlap the next launch (programmatic dependent launch) and
        # measured faster (batch 64: 5.54 ms per step, 5.98 with gate|up
        # fused, 8.30 with every projection fused).
        sp0 = int(torch.cuda.current_stream(device).cuda_stream)
        self.fused = bool(fused)
        self.qkv: list[RetiledNF4] = []
        self.gu: list[RetiledNF4] = []
        self.o: list[RetiledNF4] = []
        self.down: list[RetiledNF4] = []
        for L in weights.layers:
            self.qkv.append(retile_nf4(bridge, torch, [L.q, L.k, L.v], sp0))
            self.gu.append(retile_nf4(bridge, torch, [L.gate, L.up], sp0, interleave64=self.fused))
            self.o.append(retile_nf4(bridge, torch, [L.o], sp0))
            self.down.append(retile_nf4(bridge, torch, [L.down], sp0))
        self.lm_nf4 = retile_nf4(bridge, torch, [weights.lm_head], sp0) if weights.lm_head is not None else None
        torch.cuda.synchronize(device)
        self.qkv_rows = self.qkv[0].rows
        ks = bridge.batch_gemm_ksplit
        self.ks_qkv = ks(self.qkv_rows, c.hidden)
        self.ks_o = ks(c.hidden, L0.o.k)
        self.ks_gu = ks(2 * self.inter, c.hidden)
        self.ks_dn = ks(c.hidden, self.inter)
        lm_rows = weights.lm_head.rows if weights.lm_head is not None else c.vocab
        self.ks_lm = ks(lm_rows, c.hidden)
        part = max(self.ks_qkv * self.qkv_rows, self.ks_o * c.hidden, self.ks_gu * 2 * self.inter,
                   self.ks_dn * c.hidden, self.ks_lm * lm_rows) * self.n_pad
        ws, tickets = bridge.gqa_batch_workspace(batch=B, query_heads=self.q_heads, kv_heads=self.kv_heads,
                                                 kv_stride=cap, device=device, torch_module=torch)
        cos, sin = rope_tables(torch, max(cap, max_tokens) + 1, d, c.rope_theta, device)
        ntiles = max((self.qkv_rows + 127) // 128, (c.hidden + 127) // 128, (2 * self.inter + 127) // 128)
        self.tickets = torch.zeros(ntiles, dtype=torch.int32, device=device)  # fused epilogues (self-resetting)
        self.buffers = BatchedBuffers(
            state=torch.zeros((B, 4), dtype=torch.int32, device=device),
            pos=torch.zeros(B, dtype=torch.int32, device=device),
            kv_len=torch.zeros(B, dtype=torch.int32, device=device),
            x=torch.zeros((B, c.hidden), dtype=bf16, device=device),
            xn=torch.zeros((self.n_pad, c.hidden), dtype=bf16, device=device),
            q=torch.zeros((B, self.q_heads * d), dtype=bf16, device=device),
            attn=torch.zeros((self.n_pad, self.q_heads * d), dtype=bf16, device=device),
            h=torch.zeros((self.n_pad, self.inter), dtype=bf16, device=device),
            partials=torch.zeros(part, dtype=torch.float32, device=device),
            kcache=(shared_cache[0] if self.shared else
                    torch.zeros((c.layers, B, self.kv_heads, cap, d), dtype=bf16, device=device)),
            vcache=(shared_cache[1] if self.shared else
                    torch.zeros((c.layers, B, self.kv_heads, cap, d), dtype=bf16, device=device)),
            gqa_ws=ws,
            gqa_tickets=tickets,
            arg_ws=torch.zeros(bridge.batch_argmax_workspace_bytes(B) // 4, dtype=torch.float32, device=device),
            history=torch.zeros((B, max_tokens), dtype=torch.int32, device=device),
            rope_cos=cos,
            rope_sin=sin,
        )
        # tensor parallelism (Megatron sharding as in TensorParallel): the
        # row-parallel o_proj/down partials are summed over splits, allreduced
        # and added; the NF4 lm_head is vocabulary-parallel (per-sequence
        # argmax pairs, allgather, select)
        rank, world, group = allreduce if isinstance(allreduce, tuple) else (0, 1, None)
        self.tp_rank, self.tp_world, self.tp_group = int(rank), int(world), group
        if self.tp_world > 1 or weights.lm_head is not None:
            self.buffers.red = torch.zeros(c.hidden * self.n_pad, dtype=torch.float32, device=device)
            self.buffers.pairs = torch.zeros((B, 2), dtype=torch.int32, device=device)
            self.buffers.gathered = torch.zeros((self.tp_world, B, 2), dtype=torch.int32, device=device)
        self._torch_graph = _TorchGraphBridge(torch) if self.tp_world > 1 else None
        self.graph_plan = KudaCudaGraphPlan(self._torch_graph if self._torch_graph is not None else bridge)
        self.graph_key: Optional[DecodeGraphKey] = None
        self.launches_per_step = 0

    @property
    def captured(self) -> bool:
        return self.graph_plan.captured

    def _projection_residual(self, lin: "RetiledNF4", x: Any, ksplit: int, sp: int) -> int:
        """x += lin . x_in: one fused launch on one rank; otherwise the GEMM, then
        the (row-parallel) residual.  Returns the launches."""

        b = self.buffers
        if self.fused and self.tp_world == 1 and ksplit <= self.FUSE_MAX_SPLITS:
            self.bridge.dispatch_batch_gemm_residual(lin.data, None, x, b.partials, self.tickets, b.x, weight_type=2,
                                                     rows=lin.rows, k=lin.k, n_pad=self.n_pad, ksplit=ksplit,
                                                     batch=self.batch, stream_ptr=sp)
            return 1
        self._gemm(lin, x, ksplit, sp)
        return 1 + self._row_parallel_residual(ksplit, sp)

    def _row_parallel_residual(self, ksplit: int, sp: int) -> int:
        """x += this layer's row-parallel output: the split sum of every rank, allreduced."""

        b, c, br = self.buffers, self.config, self.bridge
        if self.tp_world == 1:
            br.dispatch_batch_residual(b.partials, b.x, ksplit=ksplit, rows=c.hidden, n_pad=self.n_pad,
                                       batch=self.batch, stream_ptr=sp)
            return 1
        import torch.distributed as dist

        br.dispatch_batch_split_sum(b.partials, b.red, ksplit=ksplit, rows=c.hidden, n_pad=self.n_pad, stream_ptr=sp)
        dist.all_reduce(b.red, group=self.tp_group)
        br.dispatch_batch_residual(b.red, b.x, ksplit=1, rows=c.hidden, n_pad=self.n_pad, batch=self.batch,
                                   stream_ptr=sp)
        return 2

    def release(self) -> None:
        """Drop the captured graph (before destroying a process group whose
        collectives it holds)."""

        self.graph_plan.invalidate()
        if self._torch_graph is not None:
            self._torch_graph.reset()

    def make_graph_key(self) -> DecodeGraphKey:
        b, w, c = self.buffers, self.weights, self.config
        ptrs = [t.data_ptr() for t in (b.state, b.pos, b.kv_len, b.x, b.xn, b.q, b.attn, b.h, b.partials, b.kcache,
                                       b.vcache, b.gqa_ws, b.gqa_tickets, b.arg_ws, b.history, b.rope_cos, b.rope_sin,
                                       w.embedding, w.final_norm)]
        for li, L in enumerate(w.layers):
            ptrs += [L.in_norm.data_ptr(), L.post_norm.data_ptr()]
            ptrs += [t.data.data_ptr() for t in (self.qkv[li], self.o[li], self.gu[li], self.down[li])]
            ptrs.append(self.tickets.data_ptr())
            ptrs += [0 if t is None else t.data_ptr() for t in (L.q_bias, L.k_bias, L.v_bias)]
        if self.lm_nf4 is not None:
            ptrs.append(self.lm_nf4.data.data_ptr())
        d = c.head_dim
        return DecodeGraphKey(
            device_id=int(self.torch.device(self.device).index or 0),
            tactic_name=self.TACTIC,
            layer_count=c.layers,
            query_shape=(self.batch, self.q_heads, 1, d),
            key_shape=(self.batch, self.kv_heads, self.kv_bucket, d),
            value_shape=(self.batch, self.kv_heads, self.kv_bucket, d),
            output_shape=(self.batch, self.q_heads, 1, d),
            kv_bucket=self.kv_bucket,
            pointers=tuple(int(p) for p in ptrs),
            model_fingerprint=c.name,
            dtype="bfloat16",
            quantization="nf4-blocksize64-fp32absmax",
        )

    def _gemm(self, lin: "RetiledNF4", x: Any, ksplit: int, sp: int) -> None:
        self.bridge.dispatch_batch_gemm(lin.data, None, x, self.buffers.partials, weight_type=2, rows=lin.rows,
                                        k=lin.k, n_pad=self.n_pad, ksplit=ksplit, stream_ptr=sp)

    def record(self, stream_ptr: int) -> int:
        """Enqueue one batched decode step; returns the number of kernels."""

        b, c, w, br = self.buffers, self.config, self.weights, self.bridge
        sp, B, npad = stream_ptr, self.batch, self.n_pad
        d = c.head_dim
        scale = 1.0 / math.sqrt(d)
        br.dispatch_batch_embedding(w.embedding, b.state, b.x, batch=B, hidden=c.hidden, vocab=c.vocab, stream_ptr=sp)
        br.dispatch_batch_state_views(b.state, b.pos, b.kv_len, batch=B, stream_ptr=sp)
        n = 2
        for li, L in enumerate(w.layers):
            br.dispatch_batch_rmsnorm(b.x, L.in_norm, b.xn, batch=B, hidden=c.hidden, epsilon=c.eps, stream_ptr=sp)
            if self.fused and self.ks_qkv <= self.FUSE_MAX_SPLITS:
                qkv = self.qkv[li]
                br.dispatch_batch_gemm_qkv_rope(qkv.data, None, b.xn, b.partials, self.tickets, L.q_bias, L.k_bias,
                                                L.v_bias, b.rope_cos, b.rope_sin, b.pos, b.q, b.kcache[li],
                                                b.vcache[li], weight_type=2, k=qkv.k, n_pad=npad, ksplit=self.ks_qkv,
                                                batch=B, q_heads=self.q_heads, kv_heads=self.kv_heads, head_dim=d,
                                                max_pos=int(b.rope_cos.shape[0]), kv_capacity=self.kv_bucket,
                                                shared_cache=self.shared, stream_ptr=sp)
                n -= 1
            else:
                self._gemm(self.qkv[li], b.xn, self.ks_qkv, sp)
                br.dispatch_batch_qkv_rope(b.partials, L.q_bias, L.k_bias, L.v_bias, b.rope_cos, b.rope_sin, b.pos,
                                           b.q, b.kcache[li], b.vcache[li], ksplit=self.ks_qkv, n_pad=npad, batch=B,
                                           q_heads=self.q_heads, kv_heads=self.kv_heads, head_dim=d,
                                           max_pos=int(b.rope_cos.shape[0]), kv_capacity=self.kv_bucket,
                                           shared_cache=self.shared, stream_ptr=sp)
            br.dispatch_gqa_decode_batch(b.q, b.kcache[li], b.vcache[li], b.attn, b.gqa_ws, b.gqa_tickets, b.kv_len,
                                         batch=B, kv_stride=self.kv_bucket, query_heads=self.q_heads,
                                         kv_heads=self.kv_heads, head_dim=d, scale=scale, shared_cache=self.shared,
                                         stream_ptr=sp)
            n += self._projection_residual(self.o[li], b.attn, self.ks_o, sp) - 2
            br.dispatch_batch_rmsnorm(b.x, L.post_norm, b.xn, batch=B, hidden=c.hidden, epsilon=c.eps, stream_ptr=sp)
            if self.fused and self.ks_gu <= self.FUSE_MAX_SPLITS:
                gu = self.gu[li]
                br.dispatch_batch_gemm_swiglu(gu.data, None, b.xn, b.partials, self.tickets, b.h, weight_type=2,
                                              intermediate=self.inter, k=gu.k, n_pad=npad, ksplit=self.ks_gu,
                                              batch=B, stream_ptr=sp)
                n -= 1
            else:
                self._gemm(self.gu[li], b.xn, self.ks_gu, sp)
                br.dispatch_batch_swiglu(b.partials, b.h, ksplit=self.ks_gu, intermediate=self.inter, n_pad=npad,
                                         batch=B, stream_ptr=sp)
            n += self._projection_residual(self.down[li], b.h, self.ks_dn, sp) - 2
            n += 11
        br.dispatch_batch_rmsnorm(b.x, w.final_norm, b.xn, batch=B, hidden=c.hidden, epsilon=c.eps, stream_ptr=sp)
        if w.lm_head is None:
            br.dispatch_batch_gemm(w.embedding, None, b.xn, b.partials, weight_type=1, rows=c.vocab, k=c.hidden,
                                   n_pad=npad, ksplit=self.ks_lm, stream_ptr=sp)
            br.dispatch_batch_argmax_advance(b.partials, b.arg_ws, b.state, b.history, ksplit=self.ks_lm,
                                             vocab=c.vocab, n_pad=npad, batch=B, stream_ptr=sp)
            n += 4
        else:  # vocabulary-parallel NF4 lm_head: this rank's rows, argmax pairs, gather, select
            v_loc = self.lm_nf4.rows
            self._gemm(self.lm_nf4, b.xn, self.ks_lm, sp)
            br.dispatch_batch_argmax_pairs(b.partials, b.arg_ws, b.pairs, ksplit=self.ks_lm, vocab=v_loc, n_pad=npad,
                                           batch=B, index_base=self.tp_rank * v_loc, stream_ptr=sp)
            if self.tp_world > 1:
                import torch.distributed as dist

                dist.all_gather_into_tensor(b.gathered, b.pairs, group=self.tp_group)
                gathered = b.gathered
            else:
                gathered = b.pairs
            br.dispatch_batch_select_advance(gathered, b.state, b.history, world=self.tp_world, batch=B, stream_ptr=sp)
            n += 5
        self.launches_per_step = n
        return n

    # ------------------------------------------------------------------ state
    def set_state(self, tokens: Any, positions: Any, stream: Any = None) -> None:
        """Write per-sequence {token, position, kv_len = position + 1} after all queued work."""

        torch = self.torch
        if stream is not None:
            stream.synchronize()
        torch.cuda.synchronize(self.device)
        tok = torch.as_tensor(list(tokens), dtype=torch.int32)
        pos = torch.as_tensor(list(positions), dtype=torch.int32)
        if tok.numel() != self.batch or pos.numel() != self.batch:
            raise ValueError("one token and one position per sequence")
        self.buffers.state.copy_(torch.stack([tok, pos, pos + 1, torch.zeros_like(pos)], dim=1))
        torch.cuda.synchronize(self.device)

    def reset_cache(self) -> None:
        self.torch.cuda.synchronize(self.device)
        self.buffers.kcache.zero_()
        self.buffers.vcache.zero_()
        self.torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ graph
    def capture(self, stream: Any) -> None:
        """Warm every kernel once eagerly on a valid state (token 0 at position
        0 for every sequence), restore the state, capture one step."""

        torch = self.torch
        sp = int(stream.cuda_stream)
        saved_state = self.buffers.state.clone()
        saved_hist = self.buffers.history.clone()
        self.buffers.state.zero_()
        self.buffers.state[:, 2] = 1
        torch.cuda.synchronize(self.device)
        with torch.cuda.stream(stream):
            self.record(sp)
        stream.synchronize()
        word = self.bridge.error_word(clear=True)
        if word:
            raise NativeCudaError(f"batched decode step raised device error word {word:#x}")
        self.buffers.state.copy_(saved_state)
        self.buffers.history.copy_(saved_hist)
        torch.cuda.synchronize(self.device)
        if self._torch_graph is None:
            self.bridge.reset_graph()
        else:
            self._torch_graph.reset()
        self.graph_plan.invalidate()
        key = self.make_graph_key()
        self.graph_plan.begin_capture(key, stream_ptr=sp)
        try:
            self.record(sp)
        except Exception:
            try:
                self.graph_plan.end_capture(key, stream_ptr=sp)
            finally:
                self.graph_plan.invalidate()
                if self._torch_graph is None:
                    self.bridge.reset_graph()
            raise
        self.graph_plan.end_capture(key, stream_ptr=sp)
        self.graph_key = key

    def replay(self, stream: Any) -> None:
        if self.graph_key is None:
            raise NativeCudaError("no captured batched decode graph")
        self.graph_plan.replay(self.graph_key, stream_ptr=int(stream.cuda_stream))

    def step_tokens(self, tokens: Any, positions: Any, stream: Any) -> list[int]:
        """One step driven from the host (prompts, teacher forcing): per-sequence
        token and position in, every sequence's next token out."""

        self.set_state(tokens, positions, stream)
        self.replay(stream)
        stream.synchronize()
        return [int(t) for t in self.buffers.state[:, 0].cpu().tolist()]


class BatchedPrefill:
    """Prompt prefill through the batched tensor-core path into a
    StaticDecodePlan's KV cache (the reference prefills token by token through
    Transformers, and its static-cache guard rejects multi-token steps,
    python/kudacuda_sidecar.py:791-792): the prompt goes in chunks of ``chunk``
    tokens, each chunk one batched step whose entries are the chunk's tokens at
    positions 64c + i with causal lengths, all appending to and attending over
    the decode plan's one cache.  The last chunk is padded with copies of the
    last token at the positions after the prompt (their cache rows are
    overwritten by the decode steps before any step reads them).  Afterwards
    the decode plan's state holds the first generated token at position
    len(prompt), so decoding continues with replay / generate_device.

    Capturing the chunk step runs it once eagerly at position 0 of the cache,
    so build this before the cache holds anything that must be kept."""

    def __init__(self, decode_plan: "StaticDecodePlan", *, chunk: int = 64) -> None:
        torch = decode_plan.torch
        self.decode = decode_plan
        self.chunk = int(chunk)
        b = decode_plan.buffers
        if isinstance(b.kcache, LayerCaches):
            raise NativeCudaError("batched prefill needs the plan's own [layers, kv_heads, cap, d] caches")
        # a handle of its own: a handle holds one graph, the decode plan's
        br = decode_plan.bridge
        self.bridge = KudaCudaBridge(device_id=br.device_id, lib_path=br.library_path, native_lib=br.lib)
        self.plan = BatchedDecodePlan(self.bridge, decode_plan.weights, batch=self.chunk,
                                      max_tokens=decode_plan.kv_bucket, device=decode_plan.device, torch_module=torch,
                                      shared_cache=(b.kcache, b.vcache))
        self.stream = torch.cuda.Stream(device=decode_plan.device)
        self.plan.capture(self.stream)

    def prefill(self, prompt: list[int], stream: Any) -> int:
        """Run the prompt; returns the first generated token (also left in the
        decode plan's state at position len(prompt))."""

        T = len(prompt)
        C = self.chunk
        nchunks = (T + C - 1) // C
        if T < 1 or nchunks * C > self.decode.kv_bucket:
            raise ValueError("prompt (padded to whole chunks) must fit the KV bucket")
        stream.synchronize()
        nxt = 0
        for ci in range(nchunks):
            toks = list(prompt[ci * C:(ci + 1) * C])
            n = len(toks)
            toks += [toks[-1]] * (C - n)
            self.plan.set_state(toks, [ci * C + i for i in range(C)], self.stream)
            self.plan.replay(self.stream)
            if ci == nchunks - 1:
                self.stream.synchronize()
                nxt = int(self.plan.buffers.state[n - 1, 0].item())
        if self.bridge.error_word(clear=True):
            raise NativeCudaError("batched prefill raised the device error word")
        self.decode.set_state(nxt, T, stream)
        return nxt


def batched_greedy_generate(plan: BatchedDecodePlan, prompts: list[list[int]], new_tokens: int,
                            stream: Any) -> list[list[int]]:
    """Ragged prompts through batched steps: while a sequence is inside its
    prompt its next prompt token is forced, afterwards it continues from its
    own greedy token.  Returns ``new_tokens`` generated tokens per sequence."""

    if len(prompts) != plan.batch:
        raise ValueError("one prompt per sequence")
    plan.reset_cache()
    lens = [len(p) for p in prompts]
    total = max(lens) + new_tokens
    if total > plan.kv_bucket:
        raise ValueError("generation exceeds the KV bucket")
    seqs = [list(p) for p in prompts]
    cur = [p[0] for p in prompts]
    for t in range(total - 1):
        nxt = plan.step_tokens(cur, [t] * plan.batch, stream)
        for i in range(plan.batch):
            if t + 1 < lens[i]:
                cur[i] = prompts[i][t + 1]
            else:
                seqs[i].append(nxt[i])
                cur[i] = nxt[i]
    return [s[lens[i]:lens[i] + new_tokens] for i, s in enumerate(seqs)]
