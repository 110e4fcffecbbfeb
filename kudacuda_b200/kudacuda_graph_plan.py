"""Static-contract guard for captured decode graphs.

Mirrors the reference's graph-plan interface (python/kudacuda_graph_plan.py:
``GraphContractError``, ``DecodeGraphKey``, ``KudaCudaGraphPlan``): a graph is
replayed only with the exact static key (device, tactic, layer count, tensor
shapes, KV bucket, every device pointer baked into the graph, model
fingerprint, dtype, quantisation) and the exact stream it was captured on;
anything else is a ``GraphContractError`` before the native replay is
reached.  The bridge it wraps needs ``begin_capture``, ``end_capture`` and
``replay_graph`` keyword methods taking ``stream_ptr``.

For tensor-parallel plans the key also records the rank and world size, so a
graph captured for one shard is never replayed on another.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional


class GraphContractError(RuntimeError):
    """A capture or replay broke the graph's static contract."""


@dataclass(frozen=True)
class DecodeGraphKey:
    """Everything that must be identical between capture and replay."""

    device_id: int
    tactic_name: str
    layer_count: int
    query_shape: tuple[int, ...]
    key_shape: tuple[int, ...]
    value_shape: tuple[int, ...]
    output_shape: tuple[int, ...]
    kv_bucket: int
    pointers: tuple[int, ...]
    model_fingerprint: str = ""
    dtype: str = ""
    quantization: str = ""
    tp_rank: int = 0
    tp_world: int = 1
    extra: tuple[Any, ...] = field(default=())


class KudaCudaGraphPlan:
    """Capture once, then replay only under the captured key and stream."""

    def __init__(self, bridge: Any) -> None:
        self.bridge = bridge
        self._pending: Optional[tuple[DecodeGraphKey, int]] = None  # capture in progress
        self._ready: Optional[tuple[DecodeGraphKey, int]] = None  # captured graph

    @property
    def captured(self) -> bool:
        return self._ready is not None

    @property
    def capturing(self) -> bool:
        return self._pending is not None

    def begin_capture(self, key: DecodeGraphKey, *, stream_ptr: int) -> None:
        if self._pending is not None:
            raise GraphContractError("graph plan is already capturing")
        if self._ready is not None:
            raise GraphContractError("graph plan already holds a captured graph; invalidate it first")
        self.bridge.begin_capture(stream_ptr=int(stream_ptr))
        self._pending = (key, int(stream_ptr))

    def end_capture(self, key: DecodeGraphKey, *, stream_ptr: int) -> None:
        if self._pending is None:
            raise GraphContractError("graph plan is not capturing")
        if self._pending != (key, int(stream_ptr)):
            raise GraphContractError("graph capture key or stream changed during capture")
        pending, self._pending = self._pending, None
        self.bridge.end_capture(stream_ptr=int(stream_ptr))  # a failure leaves nothing captured
        self._ready = pending

    def can_replay(self, key: DecodeGraphKey, *, stream_ptr: int) -> bool:
        return self._ready is not None and self._ready == (key, int(stream_ptr))

    def replay(self, key: DecodeGraphKey, *, stream_ptr: int) -> None:
        if self._ready is None:
            raise GraphContractError("graph plan has no captured graph")
        if not self.can_replay(key, stream_ptr=stream_ptr):
            raise GraphContractError("graph replay key or stream differs from the captured one")
        self.bridge.replay_graph(stream_ptr=int(stream_ptr))

    def invalidate(self) -> None:
        self._pending = None
        self._ready = None
