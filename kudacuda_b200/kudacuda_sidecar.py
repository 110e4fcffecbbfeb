"""Python bridge to the B200 KudaCuda library: contracts, guarded dispatch and
Transformers hooks.

Interface-compatible with the reference's python/kudacuda_sidecar.py (same
class and function names, argument meaning, ctypes argument order, error
types and fallback reasons), so code written against the reference bridge --
including its contract tests -- drives the sm_100a kernels unchanged.  The
sm100 additions (bf16 attention input block, bf16 SwiGLU, residual GEMVs,
split-KV GQA, lm_head argmax, quantiser) are extra ``dispatch_*`` methods.

Like the reference, the module imports only the standard library at import
time; torch and transformers are imported lazily by the paths that need them.
There is no CPU fallback inside the bridge: a native failure raises
NativeCudaError, and only the Transformers hooks fall back -- to the
framework's own forward, exactly as the reference's hooks do.
"""

from __future__ import annotations

import ctypes
import json
import math
import sys
from dataclasses import dataclass
from functools import wraps
from pathlib import Path
from types import MethodType
from typing import Any, Callable, Mapping, Optional

from . import native as _native

DEFAULT_MANIFEST = Path(__file__).resolve().parent / "manifests" / "b200-sm100.json"


class NativeCudaError(RuntimeError):
    """The native library rejected a request or a launch failed."""


def _normalize_cuda_handle(value: int) -> int:
    """PyTorch reports stream handles as signed integers; the ABI wants uint64."""

    return int(value) & 0xFFFFFFFFFFFFFFFF


def select_library_name(platform_name: Optional[str] = None) -> str:
    name = platform_name or sys.platform
    if name.startswith("win"):
        return "kudacuda.dll"
    if name == "darwin":
        return "libkudacuda.dylib"
    return "libkudacuda.so"


def load_manifest(path: str | Path) -> dict[str, Any]:
    """Read a tactic manifest and check the keys every bridge relies on."""

    manifest_path = Path(path)
    data = json.loads(manifest_path.read_text(encoding="utf-8"))
    if not isinstance(data, dict):
        raise ValueError(f"Manifest must contain a JSON object: {manifest_path}")
    for key in ("target_arch", "implemented_tactics", "contracts"):
        if key not in data:
            raise ValueError(f"Manifest missing required key '{key}': {manifest_path}")
    if not isinstance(data["implemented_tactics"], list):
        raise ValueError("Manifest 'implemented_tactics' must be a list")
    if not isinstance(data["contracts"], dict):
        raise ValueError("Manifest 'contracts' must be an object")
    return data


def _dtype_name(dtype: Any) -> str:
    return str(dtype).rsplit(".", 1)[-1].lower()


def _shape(t: Any) -> tuple[int, ...]:
    return tuple(int(v) for v in getattr(t, "shape", ()))


def _is_cuda_contiguous(t: Any) -> bool:
    if not bool(getattr(t, "is_cuda", False)):
        return False
    contiguous = getattr(t, "is_contiguous", None)
    return callable(contiguous) and bool(contiguous())


def _opt_int(m: Mapping[str, Any], key: str) -> Optional[int]:
    return int(m[key]) if m.get(key) is not None else None


@dataclass(frozen=True)
class TensorContract:
    """Shape/layout/dtype contract of one tactic (manifest 'contracts' entry)."""

    dtype: Optional[str] = None
    layout: Optional[str] = None
    rank: Optional[int] = None
    batch_size: Optional[int] = None
    seq_len: Optional[int] = None
    count_min: Optional[int] = None

    @classmethod
    def from_mapping(cls, m: Mapping[str, Any]) -> "TensorContract":
        return cls(
            dtype=_dtype_name(m["dtype"]) if m.get("dtype") else None,
            layout=str(m["layout"]).lower() if m.get("layout") else None,
            rank=_opt_int(m, "rank"),
            batch_size=_opt_int(m, "batch_size"),
            seq_len=_opt_int(m, "seq_len"),
            count_min=_opt_int(m, "count_min"),
        )

    def matches_shape(self, batch_size: int, seq_len: int) -> bool:
        if batch_size <= 0 or seq_len <= 0:
            return False
        if self.batch_size is not None and batch_size != self.batch_size:
            return False
        return self.seq_len is None or seq_len == self.seq_len

    def matches_tensor(self, tensor: Any) -> bool:
        if tensor is None:
            return True
        if not bool(getattr(tensor, "is_cuda", False)):
            return False
        if self.layout == "contiguous" and not _is_cuda_contiguous(tensor):
            return False
        if self.dtype is not None and _dtype_name(getattr(tensor, "dtype", "")) != self.dtype:
            return False
        if self.rank is not None:
            dim = getattr(tensor, "dim", None)
            if not callable(dim) or int(dim()) != self.rank:
                return False
        if self.count_min is not None:
            numel = getattr(tensor, "numel", None)
            if not callable(numel) or int(numel()) < self.count_min:
                return False
        return True


@dataclass(frozen=True)
class Qwen2GqaContract:
    """Decode-only Qwen2 GQA contract.  The reference profile is fixed to
    16 query heads, 2 KV heads and head_dim 128 (python/kudacuda_sidecar.py:145-153);
    a contract whose manifest entry sets ``"any_heads": true`` (the sm100
    split-KV tactic) accepts any head counts the kernel supports."""

    dtype: str
    layout: str
    batch_size: int
    query_len: int
    kv_len_min: int
    kv_len_max: int
    query_heads: int
    kv_heads: int
    head_dim: int
    any_heads: bool = False

    @classmethod
    def from_mapping(cls, m: Mapping[str, Any]) -> "Qwen2GqaContract":
        return cls(
            dtype=_dtype_name(m["dtype"]),
            layout=str(m["layout"]).lower(),
            batch_size=int(m["batch_size"]),
            query_len=int(m["query_len"]),
            kv_len_min=int(m["kv_len_min"]),
            kv_len_max=int(m["kv_len_max"]),
            query_heads=int(m["query_heads"]),
            kv_heads=int(m["kv_heads"]),
            head_dim=int(m["head_dim"]),
            any_heads=bool(m.get("any_heads", False)),
        )

    def heads_supported(self) -> bool:
        if self.any_heads:
            group = self.query_heads // self.kv_heads if self.kv_heads > 0 else 0
            return self.head_dim == 128 and group in (1, 2, 4, 8) and self.query_heads % self.kv_heads == 0
        return (self.query_heads, self.kv_heads, self.head_dim) == (16, 2, 128)

    def matches(self, batch_size: int, query_len: int, kv_len: int) -> bool:
        return (
            int(batch_size) == self.batch_size
            and int(query_len) == self.query_len
            and self.kv_len_min <= int(kv_len) <= self.kv_len_max
            and self.heads_supported()
        )

    def matches_tensor(self, tensor: Any, expected_shape: tuple[int, ...]) -> bool:
        if not bool(getattr(tensor, "is_cuda", False)):
            return False
        if self.layout == "contiguous" and not _is_cuda_contiguous(tensor):
            return False
        if _dtype_name(getattr(tensor, "dtype", "")) != self.dtype:
            return False
        return _shape(tensor) == expected_shape


def _qwen2_attention_dimensions(module: Any) -> tuple[int, int, int]:
    """(query_heads, kv_heads, head_dim) across Transformers attention layouts."""

    config = getattr(module, "config", None)
    q_heads = getattr(module, "num_heads", None)
    if q_heads is None:
        q_heads = getattr(config, "num_attention_heads", 0)
    kv_heads = getattr(module, "num_key_value_heads", None)
    if kv_heads is None:
        kv_heads = getattr(config, "num_key_value_heads", 0)
    head_dim = getattr(module, "head_dim", None)
    if head_dim is None:
        hidden = int(getattr(config, "hidden_size", 0))
        head_dim = hidden // int(q_heads) if q_heads else 0
    return int(q_heads), int(kv_heads), int(head_dim)


# Which native symbol serves a GQA tactic name (the reference's _qwen_symbol
# routing by name fragment, python/kudacuda_sidecar.py:483-492).
_GQA_ROUTES = (
    ("graph_v1", "kudacuda_qwen2_gqa_decode_graph"),
    ("group_tiled_v2", "kudacuda_qwen2_gqa_decode_group_tiled"),
    ("vectorized_v2", "kudacuda_qwen2_gqa_decode_vectorized"),
    ("workspace_v3", "kudacuda_qwen2_gqa_decode_workspace_v3"),
    ("splitkv", "kudacuda_sm100_gqa_decode"),
)

_QKV_SYMBOLS = {
    "": "kudacuda_qwen2_fused_rmsnorm_qkv_nf4",
    "_v2": "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2",
    "_v3": "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3",
}

_DTYPE_CODE = {"float32": 0, "float16": 1, "bfloat16": 2}


class KudaCudaBridge:
    """Own one native handle; validate every call against its contract and
    launch on the caller's stream through the C ABI."""

    def __init__(
        self,
        *,
        manifest: Mapping[str, Any] | str | Path = DEFAULT_MANIFEST,
        lib_path: str | Path | None = None,
        device_id: int = 0,
        native_lib: Any = None,
    ) -> None:
        self.manifest = load_manifest(manifest) if isinstance(manifest, (str, Path)) else dict(manifest)
        self.implemented_tactics = frozenset(self.manifest.get("implemented_tactics", ()))
        self.experimental_tactics = frozenset(self.manifest.get("experimental_tactics", ()))
        self.planned_tactics = frozenset(self.manifest.get("planned_tactics", ()))
        contracts = self.manifest.get("contracts", {})
        self.contracts = {name: TensorContract.from_mapping(c) for name, c in contracts.items()}
        self.qwen_contracts = {
            name: Qwen2GqaContract.from_mapping(c) for name, c in contracts.items() if "query_heads" in c
        }
        self.library_path: Path | None = Path(lib_path) if lib_path else None
        self.lib = native_lib if native_lib is not None else self._load_library(lib_path)
        self._configure_abi()
        self.native_attention_dispatcher = any(
            self._symbol(s) is not None
            for s in (
                "kudacuda_qwen2_gqa_decode",
                "kudacuda_qwen2_gqa_decode_group_tiled",
                "kudacuda_qwen2_gqa_decode_vectorized",
                "kudacuda_qwen2_gqa_decode_graph",
            )
        )
        for counter in (
            "native_attention_dispatches",
            "native_fused_qkv_dispatches",
            "native_fused_qkv_v2_dispatches",
            "native_fused_qkv_v3_dispatches",
            "native_swiglu_dispatches",
            "native_swiglu_bf16_dispatches",
            "native_swiglu_hook_calls",
            "native_sm100_dispatches",
        ):
            setattr(self, counter, 0)
        self._graph_kv_len_device: Any = None
        self._graph_kv_capacity: int | None = None
        self._graph_workspace: Any = None
        self._gqa_scratch: dict[Any, tuple[Any, Any, int]] = {}
        self.engine_handle = self.lib.kudacuda_create(int(device_id))
        if not self.engine_handle:
            raise NativeCudaError("kudacuda_create returned a null handle")
        self.device_id = int(device_id)
        self._closed = False
        self.freeze()

    # ---------------------------------------------------------------- plumbing
    def _load_library(self, lib_path: str | Path | None) -> Any:
        if lib_path is None:
            path = _native.DEFAULT_LIBRARY
        else:
            path = Path(lib_path)
        if not path.exists():
            raise FileNotFoundError(f"KudaCuda native library not found: {path}")
        self.library_path = path
        return ctypes.CDLL(str(path))

    def _configure_abi(self) -> None:
        for name, (restype, argtypes) in _native.SIGNATURES.items():
            fn = getattr(self.lib, name, None)
            if fn is None:
                continue
            try:
                fn.restype = restype
                fn.argtypes = argtypes
            except (AttributeError, TypeError):
                pass

    def _symbol(self, name: str) -> Any:
        return getattr(self.lib, name, None)

    # reference attribute names for the optional symbols
    @property
    def _qwen2_gqa_decode(self) -> Any:
        return self._symbol("kudacuda_qwen2_gqa_decode")

    @property
    def _qwen2_gqa_decode_graph(self) -> Any:
        return self._symbol("kudacuda_qwen2_gqa_decode_graph")

    @property
    def _qwen2_gqa_decode_workspace(self) -> Any:
        return self._symbol("kudacuda_qwen2_gqa_decode_workspace_v3")

    def _native_error(self) -> str:
        raw = self.lib.kudacuda_last_error(self.engine_handle)
        if isinstance(raw, bytes):
            return raw.decode("utf-8", errors="replace")
        return "unknown native CUDA error" if raw is None else str(raw)

    def _raise_if_failed(self, status: int, operation: str) -> None:
        if int(status) != 0:
            raise NativeCudaError(f"{operation} failed: {self._native_error()}")

    def _check_open(self) -> None:
        if self._closed:
            raise NativeCudaError("KudaCuda bridge is closed")

    def freeze(self) -> None:
        self._raise_if_failed(self.lib.kudacuda_freeze(self.engine_handle), "kudacuda_freeze")

    @staticmethod
    def _tensor_pointer(tensor: Any, label: str) -> int:
        data_ptr = getattr(tensor, "data_ptr", None)
        if not callable(data_ptr):
            raise ValueError(f"{label} does not expose data_ptr()")
        value = int(data_ptr())
        if value <= 0:
            raise ValueError(f"{label} has an invalid device pointer")
        return value

    @staticmethod
    def _optional_pointer(tensor: Any, label: str) -> int:
        return 0 if tensor is None else KudaCudaBridge._tensor_pointer(tensor, label)

    @staticmethod
    def _tensor_contract_matches(tensor: Any, *, dtype: Optional[str], rank: int) -> bool:
        if not _is_cuda_contiguous(tensor):
            return False
        dim = getattr(tensor, "dim", None)
        if not callable(dim) or int(dim()) != rank:
            return False
        return dtype is None or _dtype_name(getattr(tensor, "dtype", "")) == dtype

    def _enabled(self, tactic_name: str) -> bool:
        return tactic_name in self.implemented_tactics or tactic_name in self.experimental_tactics

    # ---------------------------------------------------------------- tactic lookup
    def matches_contract(self, tactic_name: str, batch_size: int, seq_len: int, *, tensor: Any = None) -> bool:
        if self._closed or tactic_name not in self.implemented_tactics:
            return False
        contract = self.contracts.get(tactic_name)
        if contract is None or not contract.matches_shape(int(batch_size), int(seq_len)):
            return False
        if not contract.matches_tensor(tensor):
            return False
        return bool(
            self.lib.kudacuda_can_dispatch(self.engine_handle, tactic_name.encode("utf-8"), int(batch_size), int(seq_len))
        )

    def _qwen_symbol(self, tactic_name: str) -> Any:
        for fragment, symbol in _GQA_ROUTES:
            if fragment in tactic_name:
                return self._symbol(symbol)
        return self._symbol("kudacuda_qwen2_gqa_decode")

    def tactic_status(self, tactic_name: str) -> str:
        if tactic_name.startswith("qwen2_gqa_decode_") and self._qwen_symbol(tactic_name) is None:
            return "unavailable"
        if tactic_name.startswith("qwen2_fused_rmsnorm_qkv_"):
            suffix = "_v3" if tactic_name.endswith("_v3") else "_v2" if tactic_name.endswith("_v2") else ""
            if self._symbol(_QKV_SYMBOLS[suffix]) is None:
                return "unavailable"
        if tactic_name.startswith("qwen2_swiglu_"):
            symbol = "kudacuda_qwen2_swiglu_nf4_bf16" if "_bf16_" in tactic_name else "kudacuda_qwen2_swiglu_nf4"
            if self._symbol(symbol) is None:
                return "unavailable"
        for status, names in (
            ("implemented", self.implemented_tactics),
            ("experimental", self.experimental_tactics),
            ("planned", self.planned_tactics),
        ):
            if tactic_name in names:
                return status
        return "unknown"

    # ---------------------------------------------------------------- small reference ops
    def vector_add(self, a: Any, b: Any, output: Any, *, stream_ptr: int) -> None:
        self._check_open()
        if self._qwen2_gqa_decode is None:
            # python/kudacuda_sidecar.py:507-508 -- the bridge requires a Qwen2-capable library
            raise NativeCudaError("native library does not export kudacuda_qwen2_gqa_decode")
        contract = self.contracts.get("vector_add")
        if "vector_add" not in self.implemented_tactics or contract is None:
            raise NativeCudaError("vector_add is not implemented by this manifest")
        named = (("a", a), ("b", b), ("output", output))
        for label, t in named:
            if not contract.matches_tensor(t):
                raise ValueError(f"{label} does not satisfy the vector_add CUDA contract")
        sizes = [int(t.numel()) for _, t in named]
        if len(set(sizes)) != 1:
            raise ValueError(f"vector_add tensors must have equal sizes, got {sizes}")
        status = self.lib.kudacuda_vector_add(
            self.engine_handle,
            self._tensor_pointer(a, "a"),
            self._tensor_pointer(b, "b"),
            self._tensor_pointer(output, "output"),
            sizes[0],
            _normalize_cuda_handle(stream_ptr),
        )
        self._raise_if_failed(status, "kudacuda_vector_add")

    def rmsnorm(self, input_tensor: Any, weight: Any, output: Any, *, epsilon: float = 1.0e-5, stream_ptr: int) -> None:
        self._check_open()
        contract = self.contracts.get("rmsnorm")
        if "rmsnorm" not in self.implemented_tactics or contract is None:
            raise NativeCudaError("rmsnorm is not implemented by this manifest")
        if not contract.matches_tensor(input_tensor) or not contract.matches_tensor(output):
            raise ValueError("input and output do not satisfy the RMSNorm CUDA contract")
        if not self._tensor_contract_matches(weight, dtype=contract.dtype, rank=1):
            raise ValueError("weight does not satisfy the RMSNorm CUDA contract")
        shape = _shape(input_tensor)
        if len(shape) != 2 or _shape(output) != shape:
            raise ValueError("RMSNorm input and output must have the same 2D shape")
        if _shape(weight) != (shape[1],):
            raise ValueError("RMSNorm weight must match the input hidden dimension")
        if epsilon <= 0.0:
            raise ValueError("epsilon must be positive")
        status = self.lib.kudacuda_rmsnorm(
            self.engine_handle,
            self._tensor_pointer(input_tensor, "input"),
            self._tensor_pointer(weight, "weight"),
            self._tensor_pointer(output, "output"),
            shape[0],
            shape[1],
            float(epsilon),
            _normalize_cuda_handle(stream_ptr),
        )
        self._raise_if_failed(status, "kudacuda_rmsnorm")

    def fused_rmsnorm_qkv(self, input_tensor: Any, norm_weight: Any, qkv_weight: Any, bias: Any, output: Any, *,
                          epsilon: float = 1.0e-5, stream_ptr: int) -> None:
        """Dense fp16 RMSNorm + [3H, H] QKV (kernels/common/rmsnorm_qkv_reference.cuh)."""

        self._check_open()
        fn = self._symbol("kudacuda_fused_rmsnorm_qkv")
        if fn is None:
            raise NativeCudaError("native library does not export kudacuda_fused_rmsnorm_qkv")
        for label, t, rank in (("input", input_tensor, 2), ("norm_weight", norm_weight, 1),
                               ("qkv_weight", qkv_weight, 2), ("bias", bias, 1), ("output", output, 2)):
            if not self._tensor_contract_matches(t, dtype="float16", rank=rank):
                raise ValueError(f"{label} does not satisfy the fused RMSNorm-QKV CUDA contract")
        rows, hidden = _shape(input_tensor)
        if _shape(norm_weight) != (hidden,):
            raise ValueError("norm_weight must match the input hidden dimension")
        if _shape(qkv_weight) != (hidden * 3, hidden):
            raise ValueError("qkv_weight must have shape (3 * hidden, hidden)")
        if _shape(bias) != (hidden * 3,):
            raise ValueError("bias must have shape (3 * hidden,)")
        if _shape(output) != (rows, hidden * 3):
            raise ValueError("output must have shape (rows, 3 * hidden)")
        if epsilon <= 0.0:
            raise ValueError("epsilon must be positive")
        status = fn(self.engine_handle, self._tensor_pointer(input_tensor, "input"),
                    self._tensor_pointer(norm_weight, "norm_weight"), self._tensor_pointer(qkv_weight, "qkv_weight"),
                    self._tensor_pointer(bias, "bias"), self._tensor_pointer(output, "output"), rows, hidden,
                    float(epsilon), _normalize_cuda_handle(stream_ptr))
        self._raise_if_failed(status, "kudacuda_fused_rmsnorm_qkv")

    # ---------------------------------------------------------------- GQA (reference ABI)
    def _check_qwen_tensors(self, contract: Qwen2GqaContract, tensors: tuple, kv_extent: int, what: str,
                            batch: int = 1) -> None:
        shapes = (
            (batch, contract.query_heads, 1, contract.head_dim),
            (batch, contract.kv_heads, int(kv_extent), contract.head_dim),
            (batch, contract.kv_heads, int(kv_extent), contract.head_dim),
            (batch, contract.query_heads, 1, contract.head_dim),
        )
        for label, t, shape in zip(("query", "key_cache", "value_cache", "output"), tensors, shapes):
            if not contract.matches_tensor(t, shape):
                raise ValueError(f"{label} does not satisfy the Qwen2 {what} CUDA contract")

    def dispatch_qwen2_gqa_decode(self, query: Any, key_cache: Any, value_cache: Any, output: Any, *, kv_len: int,
                                  stream_ptr: int, tactic_name: str = "qwen2_gqa_decode_sm100_fp16") -> None:
        self._check_open()
        if "graph_v1" in tactic_name:
            raise NativeCudaError("graph tactic requires an active static decode graph context")
        contract = self.qwen_contracts.get(tactic_name)
        if not self._enabled(tactic_name) or contract is None:
            raise NativeCudaError(f"{tactic_name} is not implemented by this manifest")
        fn = self._qwen_symbol(tactic_name)
        if fn is None:
            raise NativeCudaError(f"native library does not export the {tactic_name} dispatcher")
        if not contract.matches(1, 1, kv_len):
            raise ValueError(f"Qwen2 GQA decode contract does not accept kv_len={kv_len}")
        self._check_qwen_tensors(contract, (query, key_cache, value_cache, output), kv_len, "GQA")
        scale = 1.0 / math.sqrt(contract.head_dim)
        if "splitkv" in tactic_name:
            self._dispatch_splitkv(query, key_cache, value_cache, output, contract, batch=1, kv_len=int(kv_len),
                                   kv_stride=int(kv_len), kv_len_device=None, scale=scale, stream_ptr=stream_ptr,
                                   label=tactic_name)
        else:
            status = fn(self.engine_handle, self._tensor_pointer(query, "query"),
                        self._tensor_pointer(key_cache, "key_cache"), self._tensor_pointer(value_cache, "value_cache"),
                        self._tensor_pointer(output, "output"), 1, 1, int(kv_len), contract.query_heads,
                        contract.kv_heads, contract.head_dim, scale, _normalize_cuda_handle(stream_ptr))
            self._raise_if_failed(status, tactic_name)
        self.native_attention_dispatches += 1

    def configure_qwen2_graph_dispatch(self, *, kv_len_device: Any, kv_capacity: int, workspace: Any = None) -> None:
        if self._qwen2_gqa_decode_graph is None:
            raise NativeCudaError("native library does not export kudacuda_qwen2_gqa_decode_graph")
        if int(kv_capacity) < 1 or int(kv_capacity) > 4096:
            raise ValueError("kv_capacity must be in the range 1..4096")
        self._graph_kv_len_device = kv_len_device
        self._graph_kv_capacity = int(kv_capacity)
        self._graph_workspace = workspace

    def clear_qwen2_graph_dispatch(self) -> None:
        self._graph_kv_len_device = None
        self._graph_kv_capacity = None
        self._graph_workspace = None

    def _check_kv_len_device(self, kv_len_device: Any, what: str) -> None:
        if not self._tensor_contract_matches(kv_len_device, dtype="int32", rank=1):
            raise ValueError(f"kv_len_device does not satisfy the Qwen2 {what} CUDA contract")
        if _shape(kv_len_device) != (1,):
            raise ValueError("kv_len_device must have shape (1,)")

    def dispatch_qwen2_gqa_decode_workspace(self, query: Any, key_cache: Any, value_cache: Any, output: Any, *,
                                            kv_capacity: int, kv_len_device: Any, workspace: Any, stream_ptr: int,
                                            tactic_name: str = "qwen2_gqa_decode_sm100_fp16_workspace_v3") -> None:
        self._check_open()
        contract = self.qwen_contracts.get(tactic_name)
        if contract is None or self._qwen2_gqa_decode_workspace is None:
            raise NativeCudaError(f"{tactic_name} workspace contract or dispatcher is unavailable")
        if not self._enabled(tactic_name):
            raise NativeCudaError(f"{tactic_name} is not enabled by this manifest")
        if int(kv_capacity) != 512:
            raise ValueError("workspace GQA requires kv_capacity=512")
        self._check_qwen_tensors(contract, (query, key_cache, value_cache, output), kv_capacity, "workspace")
        self._check_kv_len_device(kv_len_device, "workspace")
        need = contract.query_heads * 8 * (2 + contract.head_dim)
        if not self._tensor_contract_matches(workspace, dtype="float32", rank=1):
            raise ValueError("workspace does not satisfy the Qwen2 workspace CUDA contract")
        if int(workspace.numel()) < need:
            raise ValueError(f"workspace must contain at least {need} float32 values")
        status = self._qwen2_gqa_decode_workspace(
            self.engine_handle, self._tensor_pointer(query, "query"), self._tensor_pointer(key_cache, "key_cache"),
            self._tensor_pointer(value_cache, "value_cache"), self._tensor_pointer(output, "output"),
            self._tensor_pointer(workspace, "workspace"), self._tensor_pointer(kv_len_device, "kv_len_device"),
            1, 1, int(kv_capacity), contract.query_heads, contract.kv_heads, contract.head_dim,
            1.0 / math.sqrt(contract.head_dim), _normalize_cuda_handle(stream_ptr))
        self._raise_if_failed(status, tactic_name)
        self.native_attention_dispatches += 1

    def dispatch_qwen2_gqa_decode_graph(self, query: Any, key_cache: Any, value_cache: Any, output: Any, *,
                                        kv_capacity: int, kv_len_device: Any, stream_ptr: int,
                                        tactic_name: str = "qwen2_gqa_decode_sm100_fp16_graph_v1") -> None:
        self._check_open()
        contract = self.qwen_contracts.get(tactic_name)
        if contract is None or self._qwen_symbol(tactic_name) is None:
            raise NativeCudaError(f"{tactic_name} graph contract or dispatcher is unavailable")
        self._check_qwen_tensors(contract, (query, key_cache, value_cache, output), kv_capacity, "graph")
        self._check_kv_len_device(kv_len_device, "graph")
        scale = 1.0 / math.sqrt(contract.head_dim)
        if "splitkv" in tactic_name:
            self._dispatch_splitkv(query, key_cache, value_cache, output, contract, batch=1, kv_len=int(kv_capacity),
                                   kv_stride=int(kv_capacity), kv_len_device=kv_len_device, scale=scale,
                                   stream_ptr=stream_ptr, label=tactic_name)
        else:
            args = (self.engine_handle, self._tensor_pointer(query, "query"),
                    self._tensor_pointer(key_cache, "key_cache"), self._tensor_pointer(value_cache, "value_cache"),
                    self._tensor_pointer(output, "output"), 1, 1, int(kv_capacity), contract.query_heads,
                    contract.kv_heads, contract.head_dim, scale, self._tensor_pointer(kv_len_device, "kv_len_device"),
                    _normalize_cuda_handle(stream_ptr))
            try:
                status = self._qwen2_gqa_decode_graph(*args)
            except OverflowError as error:
                raise NativeCudaError(f"graph dispatcher argument conversion failed: {args}") from error
            self._raise_if_failed(status, tactic_name)
        self.native_attention_dispatches += 1

    # ---------------------------------------------------------------- sm100 split-KV GQA
    def gqa_workspace(self, *, batch: int, query_heads: int, kv_heads: int, kv_extent: int, device: Any = None,
                      torch_module: Any = None) -> tuple[Any, Any, int]:
        """Stable (workspace, tickets, nbytes) for the split-KV kernel; cached
        per shape so graph capture sees fixed pointers.  Allocated once, before
        capture, through torch (the caller's allocator)."""

        key = (int(batch), int(query_heads), int(kv_heads), int(kv_extent), str(device))
        cached = self._gqa_scratch.get(key)
        if cached is not None:
            return cached
        if torch_module is None:
            import torch as torch_module
        nbytes = int(self.lib.kudacuda_sm100_gqa_workspace_bytes(batch, query_heads, kv_heads, kv_extent, 128))
        if nbytes <= 0:
            raise NativeCudaError("kudacuda_sm100_gqa_workspace_bytes rejected the shape")
        ws = torch_module.empty((nbytes // 4,), dtype=torch_module.float32, device=device or "cuda")
        tickets = torch_module.zeros((batch * kv_heads,), dtype=torch_module.int32, device=device or "cuda")
        self._gqa_scratch[key] = (ws, tickets, nbytes)
        return ws, tickets, nbytes

    def _dispatch_splitkv(self, query, key_cache, value_cache, output, contract: Qwen2GqaContract, *, batch: int,
                          kv_len: int, kv_stride: int, kv_len_device: Any, scale: float, stream_ptr: int,
                          label: str) -> None:
        ws, tickets, nbytes = self.gqa_workspace(batch=batch, query_heads=contract.query_heads,
                                                 kv_heads=contract.kv_heads, kv_extent=kv_stride,
                                                 device=getattr(query, "device", None))
        self.dispatch_gqa_decode_splitkv(query, key_cache, value_cache, output, ws, tickets, kv_len_device=kv_len_device,
                                         batch=batch, kv_len=kv_len, kv_stride=kv_stride,
                                         query_heads=contract.query_heads, kv_heads=contract.kv_heads,
                                         scale=scale, stream_ptr=stream_ptr, workspace_bytes=nbytes, label=label)

    def dispatch_gqa_decode_splitkv(self, query: Any, key_cache: Any, value_cache: Any, output: Any, workspace: Any,
                                    tickets: Any, *, kv_len_device: Any = None, batch: int = 1, kv_len: int,
                                    kv_stride: int, query_heads: int, kv_heads: int, scale: float | None = None,
                                    stream_ptr: int, workspace_bytes: int | None = None,
                                    label: str = "qwen2_gqa_decode_sm100_bf16_splitkv_v1") -> None:
        """kudacuda_sm100_gqa_decode: split-KV flash-decode over [B, kv_heads, stride, 128] caches."""

        self._check_open()
        dtype = _dtype_name(getattr(query, "dtype", ""))
        if dtype not in ("float16", "bfloat16"):
            raise ValueError("split-KV GQA requires float16 or bfloat16 tensors")
        for label_, t in (("query", query), ("key_cache", key_cache), ("value_cache", value_cache), ("output", output)):
            if not _is_cuda_contiguous(t) or _dtype_name(getattr(t, "dtype", "")) != dtype:
                raise ValueError(f"{label_} must be contiguous CUDA {dtype}")
        nbytes = int(workspace_bytes if workspace_bytes is not None else workspace.numel() * 4)
        status = self.lib.kudacuda_sm100_gqa_decode(
            self.engine_handle, self._tensor_pointer(query, "query"), self._tensor_pointer(key_cache, "key_cache"),
            self._tensor_pointer(value_cache, "value_cache"), self._tensor_pointer(output, "output"),
            self._tensor_pointer(workspace, "workspace"), nbytes, self._tensor_pointer(tickets, "tickets"),
            self._optional_pointer(kv_len_device, "kv_len_device"), _DTYPE_CODE[dtype], int(batch), int(kv_len),
            int(kv_stride), int(query_heads), int(kv_heads), 128,
            float(scale if scale is not None else 1.0 / math.sqrt(128)), _normalize_cuda_handle(stream_ptr))
        self._raise_if_failed(status, label)
        self.native_sm100_dispatches += 1

    # ---------------------------------------------------------------- Transformers attention hook
    def dispatch_qwen2_attention(self, module: Any, hidden_states: Any, *args: Any,
                                 tactic_name: str = "qwen2_gqa_decode_sm100_fp16", **kwargs: Any) -> Any:
        """Native decode attention for one Qwen2 attention module, or None.

        Transformers keeps the projections, RoPE and the cache update; the
        native kernel does the single-token GQA over the cache.  None means
        "fall back to the framework" (the caller then runs the original
        forward); a framework-computed result with a reason string is returned
        when the cache was already updated, so it is never updated twice.
        Mirrors python/kudacuda_sidecar.py:767-958.
        """

        import torch

        self.last_qwen2_dispatch_reason = "started"

        def decline(reason: str) -> None:
            self.last_qwen2_dispatch_reason = reason
            return None

        shape = _shape(hidden_states)
        if len(shape) != 3 or shape[0] != 1 or shape[1] != 1:
            return decline(f"shape:{shape}")
        if bool(kwargs.get("output_attentions", False)):
            return decline("output_attentions")
        contract = self.qwen_contracts.get(tactic_name)
        q_heads, kv_heads, head_dim = _qwen2_attention_dimensions(module)
        if contract is not None and contract.any_heads:
            if head_dim != 128 or kv_heads <= 0 or q_heads % kv_heads or (q_heads // kv_heads) not in (1, 2, 4, 8):
                return decline(f"heads:{q_heads}/{kv_heads}/{head_dim}")
        else:
            if q_heads != 16:
                return decline(f"query_heads:{q_heads}")
            if kv_heads != 2:
                return decline(f"kv_heads:{kv_heads}")
            if head_dim != 128:
                return decline(f"head_dim:{head_dim}")

        rest = list(args)
        position_embeddings = kwargs.get("position_embeddings")
        attention_mask = kwargs.get("attention_mask")
        past_key_values = kwargs.get("past_key_values")
        if position_embeddings is None and rest:
            position_embeddings = rest.pop(0)
        if attention_mask is None and rest:
            attention_mask = rest.pop(0)
        if past_key_values is None and rest:
            past_key_values = rest.pop(0)
        if position_embeddings is None:
            return decline("missing_position_embeddings")

        from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb

        cache_updated = False
        graph_mode = False
        q_states = k_states = v_states = None
        input_shape = hidden_states.shape[:-1]

        def framework_attention(reason: str) -> Any:
            self.last_qwen2_dispatch_reason = reason
            rep = q_heads // kv_heads
            keys = k_states.repeat_interleave(rep, dim=1)
            values = v_states.repeat_interleave(rep, dim=1)
            scores = torch.matmul(q_states, keys.transpose(-1, -2)) * float(
                getattr(module, "scaling", 1.0 / math.sqrt(head_dim)))
            if attention_mask is not None:
                scores = scores + attention_mask
            probs = torch.softmax(scores, dim=-1, dtype=torch.float32).to(q_states.dtype)
            ctx = torch.matmul(probs, values).transpose(1, 2).reshape(*input_shape, -1).contiguous()
            return module.o_proj(ctx), None

        try:
            hidden_shape = (*input_shape, -1, module.head_dim)
            prefused = getattr(module, "_kudacuda_prefused_qkv", None)
            if prefused is not None:
                q_flat, k_flat, v_flat = prefused
                q_states = q_flat.view(hidden_shape).transpose(1, 2)
                k_states = k_flat.view(hidden_shape).transpose(1, 2)
                v_states = v_flat.view(hidden_shape).transpose(1, 2)
            else:
                q_states = module.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
                k_states = module.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
                v_states = module.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            cos, sin = position_embeddings
            q_states, k_states = apply_rotary_pos_emb(q_states, k_states, cos, sin)
            if past_key_values is not None:
                cache_kwargs = {"sin": sin, "cos": cos}
                if kwargs.get("cache_position") is not None:
                    cache_kwargs["cache_position"] = kwargs["cache_position"]
                try:
                    k_states, v_states = past_key_values.update(k_states, v_states, module.layer_idx, cache_kwargs)
                except TypeError:
                    k_states, v_states = past_key_values.update(k_states, v_states, module.layer_idx)
                cache_updated = True
            if k_states.dim() != 4 or v_states.shape != k_states.shape:
                return decline(f"cache_shape:{tuple(k_states.shape)}:{tuple(v_states.shape)}")
            graph_mode = (
                ("graph_v1" in tactic_name or "workspace_v3" in tactic_name or "splitkv" in tactic_name)
                and self._graph_kv_len_device is not None
                and self._graph_kv_capacity is not None
            )
            kv_len = int(k_states.shape[-2])
            if graph_mode:
                if kv_len != self._graph_kv_capacity:
                    return decline(f"graph_cache_capacity:{kv_len}:{self._graph_kv_capacity}")
                if getattr(module, "sliding_window", None) is not None:
                    return decline("graph_sliding_window_unsupported")
            if attention_mask is not None and not graph_mode:
                if attention_mask.dim() != 4 or int(attention_mask.shape[-1]) != kv_len:
                    return decline(f"attention_mask_shape:{tuple(attention_mask.shape)}:kv={kv_len}")
                if not bool(torch.all(attention_mask == 0)):
                    return framework_attention("framework_fallback:attention_mask_values")
            if graph_mode:
                q_states = q_states.contiguous()
                k_states = k_states.contiguous()
                v_states = v_states.contiguous()
            elif not bool(q_states.is_contiguous()) or not bool(k_states.is_contiguous()):
                return framework_attention(f"non_contiguous:q={q_states.stride()}:k={k_states.stride()}")

            out = torch.empty_like(q_states)
            stream_ptr = int(torch.cuda.current_stream(hidden_states.device).cuda_stream)
            try:
                if "workspace_v3" in tactic_name:
                    if self._graph_workspace is None:
                        raise NativeCudaError("workspace GQA tactic requires a configured workspace")
                    self.dispatch_qwen2_gqa_decode_workspace(
                        q_states, k_states, v_states, out, kv_capacity=int(self._graph_kv_capacity),
                        kv_len_device=self._graph_kv_len_device, workspace=self._graph_workspace,
                        stream_ptr=stream_ptr, tactic_name=tactic_name)
                elif graph_mode:
                    self.dispatch_qwen2_gqa_decode_graph(
                        q_states, k_states, v_states, out, kv_capacity=int(self._graph_kv_capacity),
                        kv_len_device=self._graph_kv_len_device, stream_ptr=stream_ptr, tactic_name=tactic_name)
                else:
                    self.dispatch_qwen2_gqa_decode(q_states, k_states, v_states, out, kv_len=kv_len,
                                                   stream_ptr=stream_ptr, tactic_name=tactic_name)
            except Exception as error:
                if graph_mode:
                    raise
                return framework_attention(f"framework_fallback:native_exception:{type(error).__name__}:{error}")
            ctx = out.transpose(1, 2).reshape(*input_shape, -1).contiguous()
            self.last_qwen2_dispatch_reason = "native"
            return module.o_proj(ctx), None
        except Exception as error:
            if graph_mode:
                raise
            if cache_updated and q_states is not None and k_states is not None:
                try:
                    return framework_attention(f"framework_fallback:exception:{type(error).__name__}:{error}")
                except Exception:
                    pass
            return decline(f"exception:{type(error).__name__}:{error}")

    # ---------------------------------------------------------------- NF4 reference ABI
    @staticmethod
    def _validate_nf4_weight(weight: Any, absmax: Any, *, expected_shape: tuple[int, int], label: str) -> int:
        """bitsandbytes Params4bit checks (python/kudacuda_sidecar.py:1017-1049):
        nf4, blocksize 64, not nested, packed (N*K/2, 1) uint8, fp32 absmax."""

        state = getattr(weight, "quant_state", None)
        if state is None:
            raise ValueError(f"{label} is missing quant_state")
        if str(getattr(state, "quant_type", "")) != "nf4":
            raise ValueError(f"{label} quant_type must be nf4")
        blocksize = int(getattr(state, "blocksize", 0))
        if blocksize != 64:
            raise ValueError(f"{label} blocksize must be 64")
        if bool(getattr(state, "nested", False)):
            raise ValueError(f"{label} nested quantization is unsupported")
        if tuple(int(v) for v in getattr(state, "shape", ())) != expected_shape:
            raise ValueError(f"{label} logical shape must be {expected_shape}")
        if not KudaCudaBridge._tensor_contract_matches(weight, dtype="uint8", rank=2):
            raise ValueError(f"{label} packed storage must be contiguous CUDA uint8")
        packed = (expected_shape[0] * expected_shape[1] + 1) // 2
        if _shape(weight) != (packed, 1):
            raise ValueError(f"{label} packed shape must be {(packed, 1)}")
        if not KudaCudaBridge._tensor_contract_matches(absmax, dtype="float32", rank=1):
            raise ValueError(f"{label} absmax must be contiguous CUDA float32")
        blocks = (expected_shape[0] * expected_shape[1] + blocksize - 1) // blocksize
        if int(absmax.numel()) != blocks:
            raise ValueError(f"{label} absmax must contain {blocks} blocks")
        return blocksize

    def dispatch_qwen2_fused_rmsnorm_qkv_nf4(self, input_tensor: Any, norm_weight: Any, q_weight: Any, q_absmax: Any,
                                             q_bias: Any, k_weight: Any, k_absmax: Any, k_bias: Any, v_weight: Any,
                                             v_absmax: Any, v_bias: Any, q_output: Any, k_output: Any, v_output: Any,
                                             *, normalized_workspace: Any = None, epsilon: float = 1.0e-5,
                                             stream_ptr: int,
                                             tactic_name: str = "qwen2_fused_rmsnorm_qkv_sm100_nf4_v1") -> None:
        """Qwen2.5-3B fp16 RMSNorm + NF4 Q/K/V (+bias); v2/v3 also fill the fp32
        normalised workspace."""

        self._check_open()
        suffix = "_v3" if tactic_name.endswith("_v3") else "_v2" if tactic_name.endswith("_v2") else ""
        fn = self._symbol(_QKV_SYMBOLS[suffix])
        if fn is None:
            raise NativeCudaError("native library does not export the requested NF4 fused QKV ABI")
        if not self._enabled(tactic_name):
            raise NativeCudaError(f"{tactic_name} is not enabled by this manifest")
        if not self._tensor_contract_matches(input_tensor, dtype="float16", rank=2):
            raise ValueError("input must be contiguous CUDA float16 rank-2")
        if not self._tensor_contract_matches(norm_weight, dtype="float16", rank=1):
            raise ValueError("norm_weight must be contiguous CUDA float16 rank-1")
        rows, hidden = _shape(input_tensor)
        if (rows, hidden) != (1, 2048) or _shape(norm_weight) != (2048,):
            raise ValueError("NF4 fused QKV requires input (1, 2048) and norm_weight (2048,)")
        sizes = []
        sizes.append(self._validate_nf4_weight(q_weight, q_absmax, expected_shape=(2048, 2048), label="q_weight"))
        for label, bias, shape in (("q_bias", q_bias, (2048,)), ("k_bias", k_bias, (256,)), ("v_bias", v_bias, (256,))):
            if not self._tensor_contract_matches(bias, dtype="float16", rank=1):
                raise ValueError(f"{label} must be contiguous CUDA float16 rank-1")
            if _shape(bias) != shape:
                raise ValueError(f"{label} must have shape {shape}")
        sizes.append(self._validate_nf4_weight(k_weight, k_absmax, expected_shape=(256, 2048), label="k_weight"))
        sizes.append(self._validate_nf4_weight(v_weight, v_absmax, expected_shape=(256, 2048), label="v_weight"))
        if sizes != [64, 64, 64]:
            raise ValueError("all NF4 projection block sizes must be 64")
        for label, t, shape in (("q_output", q_output, (rows, 2048)), ("k_output", k_output, (rows, 256)),
                                ("v_output", v_output, (rows, 256))):
            if not self._tensor_contract_matches(t, dtype="float16", rank=2):
                raise ValueError(f"{label} must be contiguous CUDA float16 rank-2")
            if _shape(t) != shape:
                raise ValueError(f"{label} must have shape {shape}")
        if suffix:
            if not self._tensor_contract_matches(normalized_workspace, dtype="float32", rank=2):
                raise ValueError("normalized_workspace must be contiguous CUDA float32 rank-2")
            if _shape(normalized_workspace) != (rows, hidden):
                raise ValueError(f"normalized_workspace must have shape {(rows, hidden)}")
        if epsilon <= 0.0:
            raise ValueError("epsilon must be positive")
        ptr = self._tensor_pointer
        args = [self.engine_handle, ptr(input_tensor, "input"), ptr(norm_weight, "norm_weight"),
                ptr(q_weight, "q_weight"), ptr(q_absmax, "q_absmax"), ptr(q_bias, "q_bias"),
                ptr(k_weight, "k_weight"), ptr(k_absmax, "k_absmax"), ptr(k_bias, "k_bias"),
                ptr(v_weight, "v_weight"), ptr(v_absmax, "v_absmax"), ptr(v_bias, "v_bias")]
        if suffix:
            args.append(ptr(normalized_workspace, "normalized_workspace"))
        args += [ptr(q_output, "q_output"), ptr(k_output, "k_output"), ptr(v_output, "v_output"), rows, hidden, 2048,
                 256, 64, float(epsilon), _normalize_cuda_handle(stream_ptr)]
        self._raise_if_failed(fn(*args), tactic_name)
        self.native_fused_qkv_dispatches += 1
        if suffix == "_v2":
            self.native_fused_qkv_v2_dispatches += 1
        if suffix == "_v3":
            self.native_fused_qkv_v3_dispatches += 1

    def dispatch_qwen2_fused_rmsnorm_qkv_nf4_v2(self, *args: Any, normalized_workspace: Any, epsilon: float = 1.0e-5,
                                                stream_ptr: int,
                                                tactic_name: str = "qwen2_fused_rmsnorm_qkv_sm100_nf4_v2") -> None:
        self.dispatch_qwen2_fused_rmsnorm_qkv_nf4(*args, normalized_workspace=normalized_workspace, epsilon=epsilon,
                                                  stream_ptr=stream_ptr, tactic_name=tactic_name)

    def dispatch_qwen2_fused_rmsnorm_qkv_nf4_v3(self, *args: Any, normalized_workspace: Any, epsilon: float = 1.0e-5,
                                                stream_ptr: int,
                                                tactic_name: str = "qwen2_fused_rmsnorm_qkv_sm100_nf4_v3") -> None:
        self.dispatch_qwen2_fused_rmsnorm_qkv_nf4(*args, normalized_workspace=normalized_workspace, epsilon=epsilon,
                                                  stream_ptr=stream_ptr, tactic_name=tactic_name)

    def _swiglu(self, dtype: str, symbol: str, counter: Optional[str], input_tensor, norm_weight, gate_weight,
                gate_absmax, up_weight, up_absmax, output, epsilon, stream_ptr, tactic_name) -> None:
        self._check_open()
        fn = self._symbol(symbol)
        if fn is None:
            what = "BF16 NF4 SwiGLU" if dtype == "bfloat16" else "NF4 SwiGLU"
            raise NativeCudaError(f"native library does not export the {what} ABI")
        if not self._enabled(tactic_name):
            raise NativeCudaError(f"{tactic_name} is not enabled by this manifest")
        if not self._tensor_contract_matches(input_tensor, dtype=dtype, rank=2):
            raise ValueError(f"input must be contiguous CUDA {dtype} rank-2")
        if not self._tensor_contract_matches(norm_weight, dtype=dtype, rank=1):
            raise ValueError(f"norm_weight must be contiguous CUDA {dtype} rank-1")
        rows, hidden = _shape(input_tensor)
        if (rows, hidden) != (1, 2048) or _shape(norm_weight) != (2048,):
            prefix = "BF16 NF4 SwiGLU" if dtype == "bfloat16" else "NF4 SwiGLU"
            raise ValueError(f"{prefix} requires input (1, 2048) and norm_weight (2048,)")
        g = self._validate_nf4_weight(gate_weight, gate_absmax, expected_shape=(11008, 2048), label="gate_weight")
        u = self._validate_nf4_weight(up_weight, up_absmax, expected_shape=(11008, 2048), label="up_weight")
        if g != 64 or u != 64:
            raise ValueError("NF4 SwiGLU block sizes must be 64")
        if not self._tensor_contract_matches(output, dtype=dtype, rank=2):
            raise ValueError(f"output must be contiguous CUDA {dtype} rank-2")
        if _shape(output) != (rows, 11008):
            raise ValueError("output must have shape (1, 11008)")
        if epsilon <= 0.0:
            raise ValueError("epsilon must be positive")
        ptr = self._tensor_pointer
        status = fn(self.engine_handle, ptr(input_tensor, "input"), ptr(norm_weight, "norm_weight"),
                    ptr(gate_weight, "gate_weight"), ptr(gate_absmax, "gate_absmax"), ptr(up_weight, "up_weight"),
                    ptr(up_absmax, "up_absmax"), ptr(output, "output"), rows, hidden, 11008, 64, float(epsilon),
                    _normalize_cuda_handle(stream_ptr))
        self._raise_if_failed(status, tactic_name)
        self.native_swiglu_dispatches += 1
        if counter:
            setattr(self, counter, getattr(self, counter) + 1)

    def dispatch_qwen2_swiglu_nf4(self, input_tensor: Any, norm_weight: Any, gate_weight: Any, gate_absmax: Any,
                                  up_weight: Any, up_absmax: Any, output: Any, *, epsilon: float = 1.0e-5,
                                  stream_ptr: int, tactic_name: str = "qwen2_swiglu_sm100_nf4_v1") -> None:
        self._swiglu("float16", "kudacuda_qwen2_swiglu_nf4", None, input_tensor, norm_weight, gate_weight,
                     gate_absmax, up_weight, up_absmax, output, epsilon, stream_ptr, tactic_name)

    def dispatch_qwen2_swiglu_nf4_bf16(self, input_tensor: Any, norm_weight: Any, gate_weight: Any, gate_absmax: Any,
                                       up_weight: Any, up_absmax: Any, output: Any, *, epsilon: float = 1.0e-6,
                                       stream_ptr: int, tactic_name: str = "qwen2_swiglu_sm100_bf16_nf4_v1") -> None:
        self._swiglu("bfloat16", "kudacuda_qwen2_swiglu_nf4_bf16", "native_swiglu_bf16_dispatches", input_tensor,
                     norm_weight, gate_weight, gate_absmax, up_weight, up_absmax, output, epsilon, stream_ptr,
                     tactic_name)

    # ---------------------------------------------------------------- sm100 bf16 model blocks
    def _call(self, symbol: str, *args: Any) -> None:
        self._check_open()
        fn = self._symbol(symbol)
        if fn is None:
            raise NativeCudaError(f"native library does not export {symbol}")
        self._raise_if_failed(fn(self.engine_handle, *args), symbol)
        self.native_sm100_dispatches += 1

    def dispatch_nf4_gemv(self, x: Any, weight_packed: Any, absmax: Any, output: Any, *, rows: int, k: int,
                          bias: Any = None, stream_ptr: int) -> None:
        """output[r] = x . W[r] (+ bias): any rows, k % 64 == 0, bf16/f16/f32 io."""

        xd = _DTYPE_CODE.get(_dtype_name(getattr(x, "dtype", "")))
        od = _DTYPE_CODE.get(_dtype_name(getattr(output, "dtype", "")))
        if xd is None or od is None:
            raise ValueError("x and output must be float32, float16 or bfloat16")
        if int(x.numel()) != int(k) or int(output.numel()) != int(rows):
            raise ValueError("x must hold k values and output rows values")
        self._call("kudacuda_sm100_nf4_gemv", self._tensor_pointer(x, "x"), xd,
                   self._tensor_pointer(weight_packed, "weight_packed"), self._tensor_pointer(absmax, "absmax"),
                   self._optional_pointer(bias, "bias"), self._tensor_pointer(output, "output"), od, int(rows), int(k),
                   64, _normalize_cuda_handle(stream_ptr))

    def dispatch_nf4_linear_residual(self, x: Any, weight_packed: Any, absmax: Any, residual: Any, *, rows: int,
                                     k: int, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_nf4_linear_residual_bf16", self._tensor_pointer(x, "x"),
                   self._tensor_pointer(weight_packed, "weight_packed"), self._tensor_pointer(absmax, "absmax"),
                   self._tensor_pointer(residual, "residual"), int(rows), int(k), 64, _normalize_cuda_handle(stream_ptr))

    def dispatch_nf4_dequantize(self, weight_packed: Any, absmax: Any, output: Any, *, n: int, stream_ptr: int) -> None:
        od = _DTYPE_CODE[_dtype_name(output.dtype)]
        self._call("kudacuda_sm100_nf4_dequantize", self._tensor_pointer(weight_packed, "weight_packed"),
                   self._tensor_pointer(absmax, "absmax"), self._tensor_pointer(output, "output"), od, int(n), 64,
                   _normalize_cuda_handle(stream_ptr))

    def dispatch_nf4_quantize(self, weight: Any, weight_packed: Any, absmax: Any, *, stream_ptr: int) -> None:
        it = _DTYPE_CODE[_dtype_name(weight.dtype)]
        self._call("kudacuda_sm100_nf4_quantize", self._tensor_pointer(weight, "weight"), it,
                   self._tensor_pointer(weight_packed, "weight_packed"), self._tensor_pointer(absmax, "absmax"),
                   int(weight.numel()), 64, _normalize_cuda_handle(stream_ptr))

    def dispatch_attention_input(self, x: Any, norm_weight: Any, q: tuple, k: tuple, v: tuple, rope_cos: Any,
                                 rope_sin: Any, position_device: Any, q_output: Any, key_cache: Any, value_cache: Any,
                                 *, q_heads: int, kv_heads: int, head_dim: int, kv_capacity: int, epsilon: float,
                                 stream_ptr: int) -> None:
        """RMSNorm + NF4 q/k/v (+bias) + RoPE + KV append; q/k/v = (packed, absmax, bias or None)."""

        p = self._tensor_pointer
        self._call("kudacuda_sm100_rmsnorm_qkv_rope_nf4_bf16", p(x, "x"), p(norm_weight, "norm_weight"),
                   p(q[0], "q_weight"), p(q[1], "q_absmax"), self._optional_pointer(q[2], "q_bias"),
                   p(k[0], "k_weight"), p(k[1], "k_absmax"), self._optional_pointer(k[2], "k_bias"),
                   p(v[0], "v_weight"), p(v[1], "v_absmax"), self._optional_pointer(v[2], "v_bias"),
                   p(rope_cos, "rope_cos"), p(rope_sin, "rope_sin"), p(position_device, "position_device"),
                   p(q_output, "q_output"), p(key_cache, "key_cache"), p(value_cache, "value_cache"),
                   int(x.numel()), int(q_heads), int(kv_heads), int(head_dim), int(kv_capacity),
                   int(rope_cos.shape[0]), 64, float(epsilon), _normalize_cuda_handle(stream_ptr))

    def dispatch_swiglu_bf16(self, x: Any, norm_weight: Any, gate: tuple, up: tuple, output: Any, *, epsilon: float,
                             stream_ptr: int) -> None:
        p = self._tensor_pointer
        self._call("kudacuda_sm100_swiglu_nf4_bf16", p(x, "x"), p(norm_weight, "norm_weight"), p(gate[0], "gate"),
                   p(gate[1], "gate_absmax"), p(up[0], "up"), p(up[1], "up_absmax"), p(output, "output"),
                   int(x.numel()), int(output.numel()), 64, float(epsilon), _normalize_cuda_handle(stream_ptr))

    def dispatch_lm_head_argmax(self, hidden: Any, final_norm: Any, embedding: Any, token_out: Any, workspace: Any,
                                ticket: Any, *, logits: Any = None, epsilon: float, stream_ptr: int) -> None:
        vocab, h = _shape(embedding)
        p = self._tensor_pointer
        self._call("kudacuda_sm100_lm_head_argmax_bf16", p(hidden, "hidden"), p(final_norm, "final_norm"),
                   p(embedding, "embedding"), self._optional_pointer(logits, "logits"), p(token_out, "token_out"),
                   p(workspace, "workspace"), int(workspace.numel()) * int(workspace.element_size()),
                   p(ticket, "ticket"), vocab, h, float(epsilon), _normalize_cuda_handle(stream_ptr))

    def dispatch_embedding(self, embedding: Any, token_device: Any, output: Any, *, stream_ptr: int) -> None:
        vocab, h = _shape(embedding)
        p = self._tensor_pointer
        self._call("kudacuda_sm100_embedding_bf16", p(embedding, "embedding"), p(token_device, "token_device"),
                   p(output, "output"), vocab, h, _normalize_cuda_handle(stream_ptr))

    def dispatch_decode_advance(self, step_state: Any, next_token: Any, *, history: Any = None,
                                stream_ptr: int) -> None:
        self._call("kudacuda_sm100_decode_advance", self._tensor_pointer(step_state, "step_state"),
                   self._tensor_pointer(next_token, "next_token"), self._optional_pointer(history, "history"),
                   int(history.numel()) if history is not None else 0, _normalize_cuda_handle(stream_ptr))

    def lm_head_workspace_bytes(self) -> int:
        return int(self.lib.kudacuda_sm100_lm_head_workspace_bytes())

    # ---------------------------------------------------------------- tensor-parallel step ops
    def dispatch_rmsnorm_nf4_gemv(self, x: Any, norm_weight: Any, weight: tuple, output: Any, *, epsilon: float,
                                  stream_ptr: int) -> None:
        packed, absmax = weight[0], weight[1]
        rows = int(output.numel())
        od = _DTYPE_CODE[_dtype_name(output.dtype)]
        self._call("kudacuda_sm100_rmsnorm_nf4_gemv", self._tensor_pointer(x, "input"),
                   self._tensor_pointer(norm_weight, "norm_weight"), self._tensor_pointer(packed, "weight_packed"),
                   self._tensor_pointer(absmax, "absmax"), self._tensor_pointer(output, "output"), od, rows,
                   int(x.numel()), float(epsilon), _normalize_cuda_handle(stream_ptr))

    def dispatch_residual_add_f32(self, partial_sum: Any, residual: Any, *, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_residual_add_f32", self._tensor_pointer(partial_sum, "partial_sum"),
                   self._tensor_pointer(residual, "residual"), int(residual.numel()),
                   _normalize_cuda_handle(stream_ptr))

    def argmax_workspace_bytes(self) -> int:
        return int(self.lib.kudacuda_sm100_argmax_workspace_bytes())

    def dispatch_argmax_shard(self, logits: Any, workspace: Any, ticket: Any, out_pair: Any, *, index_base: int,
                              stream_ptr: int) -> None:
        self._call("kudacuda_sm100_argmax_shard_f32", self._tensor_pointer(logits, "logits"), int(logits.numel()),
                   int(index_base), self._tensor_pointer(workspace, "workspace"),
                   int(workspace.numel()) * int(workspace.element_size()), self._tensor_pointer(ticket, "ticket"),
                   self._tensor_pointer(out_pair, "out_pair"), _normalize_cuda_handle(stream_ptr))

    def dispatch_select_token(self, pairs: Any, next_token: Any, *, count: int, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_select_token", self._tensor_pointer(pairs, "pairs"), int(count),
                   self._tensor_pointer(next_token, "next_token"), _normalize_cuda_handle(stream_ptr))

    # ---------------------------------------------------------------- persistent decode of all layers
    RETILE_PLAIN, RETILE_SWIGLU, RETILE_QKV_ROPE = 0, 1, 2

    def retile_groups(self, mode: int, rows: tuple[int, int, int], head_dim: int = 0) -> int:
        """Row groups of the persistent stream layout, or -1 for an unsupported shape."""

        self._check_open()
        return int(self.lib.kudacuda_sm100_nf4_retile_groups(int(mode), int(rows[0]), int(rows[1]), int(rows[2]),
                                                             int(head_dim)))

    def dispatch_nf4_retile(self, mode: int, mats: list[tuple[Any, Any, int]], out_codes: Any, out_absmax: Any, *,
                            k: int, head_dim: int = 0, stream_ptr: int) -> None:
        """Copy bitsandbytes NF4 matrices ``(packed, absmax, rows)`` into the
        persistent kernel's group-tile stream layout."""

        args: list[int] = []
        for i in range(3):
            if i < len(mats):
                packed, absmax, rows = mats[i]
                args += [self._tensor_pointer(packed, "packed"), self._tensor_pointer(absmax, "absmax"), int(rows)]
            else:
                args += [0, 0, 0]
        self._call("kudacuda_sm100_nf4_retile", int(mode), *args, int(k), int(head_dim),
                   self._tensor_pointer(out_codes, "out_codes"), self._tensor_pointer(out_absmax, "out_absmax"),
                   _normalize_cuda_handle(stream_ptr))

    def retile16_tiles(self, mode: int, rows: tuple[int, int, int], head_dim: int = 0) -> int:
        """16-row tiles of the row-split persistent layout, or -1 for an unsupported shape."""

        self._check_open()
        return int(self.lib.kudacuda_sm100_nf4_retile16_tiles(int(mode), int(rows[0]), int(rows[1]), int(rows[2]),
                                                              int(head_dim)))

    def dispatch_nf4_retile16(self, mode: int, mats: list[tuple[Any, Any, int]], out_units: Any, *, k: int,
                              head_dim: int = 0, stream_ptr: int) -> None:
        """Copy bitsandbytes NF4 matrices ``(packed, absmax, rows)`` into the
        row-split persistent kernel's 576-byte units (tile-major)."""

        args: list[int] = []
        for i in range(3):
            if i < len(mats):
                packed, absmax, rows = mats[i]
                args += [self._tensor_pointer(packed, "packed"), self._tensor_pointer(absmax, "absmax"), int(rows)]
            else:
                args += [0, 0, 0]
        self._call("kudacuda_sm100_nf4_retile16", int(mode), *args, int(k), int(head_dim),
                   self._tensor_pointer(out_units, "out_units"), int(out_units.numel()) * int(out_units.element_size()),
                   _normalize_cuda_handle(stream_ptr))

    def rows_scratch_bytes(self, *, layers: int, hidden: int, q_heads: int, kv_heads: int, head_dim: int,
                           intermediate: int, kv_capacity: int) -> int:
        self._check_open()
        n = int(self.lib.kudacuda_sm100_decode_rows_scratch_bytes(
            self.engine_handle, int(layers), int(hidden), int(q_heads), int(kv_heads), int(head_dim),
            int(intermediate), int(kv_capacity)))
        if n < 0:
            raise NativeCudaError(f"kudacuda_sm100_decode_rows_scratch_bytes: {self._native_error()}")
        return n

    def dispatch_decode_layers_rows(self, layer_table: Any, x: Any, state: Any, rope_cos: Any, rope_sin: Any,
                                    scratch: Any, *, layers: int, max_pos: int, hidden: int, q_heads: int,
                                    kv_heads: int, head_dim: int, intermediate: int, kv_capacity: int, epsilon: float,
                                    scale: float, stream_ptr: int, taps: Any = None, spin_limit: int = 0,
                                    stall_counter: int = -1) -> None:
        tp = 0 if taps is None else self._tensor_pointer(taps, "taps")
        tb = 0 if taps is None else int(taps.numel()) * int(taps.element_size())
        self._call("kudacuda_sm100_decode_layers_rows", self._tensor_pointer(layer_table, "layer_table"), int(layers),
                   self._tensor_pointer(x, "x"), self._tensor_pointer(state, "state"),
                   self._tensor_pointer(rope_cos, "rope_cos"), self._tensor_pointer(rope_sin, "rope_sin"),
                   int(max_pos), self._tensor_pointer(scratch, "scratch"),
                   int(scratch.numel()) * int(scratch.element_size()), int(hidden), int(q_heads), int(kv_heads),
                   int(head_dim), int(intermediate), int(kv_capacity), float(epsilon), float(scale), tp, tb,
                   int(spin_limit), int(stall_counter), _normalize_cuda_handle(stream_ptr))

    def dispatch_decode_layers_rows_tp(self, layer_table: Any, x: Any, state: Any, rope_cos: Any, rope_sin: Any,
                                       scratch: Any, *, layers: int, max_pos: int, hidden: int, q_heads: int,
                                       kv_heads: int, head_dim: int, intermediate: int, kv_capacity: int,
                                       epsilon: float, scale: float, world: int, rank: int, peers: Any,
                                       stream_ptr: int) -> None:
        """The row-split kernel over this rank's tensor-parallel shard; o_proj
        and down partials are exchanged with the other ranks inside the kernel
        (``peers``: device int64 [world] exchange-buffer addresses)."""

        self._call("kudacuda_sm100_decode_layers_rows_tp", self._tensor_pointer(layer_table, "layer_table"),
                   int(layers), self._tensor_pointer(x, "x"), self._tensor_pointer(state, "state"),
                   self._tensor_pointer(rope_cos, "rope_cos"), self._tensor_pointer(rope_sin, "rope_sin"),
                   int(max_pos), self._tensor_pointer(scratch, "scratch"),
                   int(scratch.numel()) * int(scratch.element_size()), int(hidden), int(q_heads), int(kv_heads),
                   int(head_dim), int(intermediate), int(kv_capacity), float(epsilon), float(scale), int(world),
                   int(rank), self._tensor_pointer(peers, "peers"), _normalize_cuda_handle(stream_ptr))

    def tp_exchange_bytes(self, world: int, hidden: int) -> int:
        self._check_open()
        n = int(self.lib.kudacuda_sm100_tp_exchange_bytes(int(world), int(hidden)))
        if n < 0:
            raise NativeCudaError("kudacuda_sm100_tp_exchange_bytes: unsupported world or hidden")
        return n

    def ipc_alloc(self, nbytes: int) -> tuple[int, bytes]:
        """A zeroed device allocation of its own and its 64-byte CUDA IPC handle."""

        import ctypes

        ptr = ctypes.c_uint64(0)
        buf = ctypes.create_string_buffer(64)
        self._check_open()
        fn = self._symbol("kudacuda_sm100_ipc_alloc")
        if fn is None:
            raise NativeCudaError("native library does not export kudacuda_sm100_ipc_alloc")
        self._raise_if_failed(fn(self.engine_handle, int(nbytes), ctypes.byref(ptr), buf, 64), "kudacuda_sm100_ipc_alloc")
        return int(ptr.value), bytes(buf.raw)

    def ipc_open(self, handle: bytes) -> int:
        import ctypes

        ptr = ctypes.c_uint64(0)
        buf = ctypes.create_string_buffer(bytes(handle), 64)
        self._check_open()
        fn = self._symbol("kudacuda_sm100_ipc_open")
        if fn is None:
            raise NativeCudaError("native library does not export kudacuda_sm100_ipc_open")
        self._raise_if_failed(fn(self.engine_handle, buf, 64, ctypes.byref(ptr)), "kudacuda_sm100_ipc_open")
        return int(ptr.value)

    def ipc_close(self, ptr: int, *, owned: bool) -> None:
        self._check_open()
        fn = self._symbol("kudacuda_sm100_ipc_close")
        if fn is None:
            raise NativeCudaError("native library does not export kudacuda_sm100_ipc_close")
        self._raise_if_failed(fn(self.engine_handle, int(ptr), 1 if owned else 0), "kudacuda_sm100_ipc_close")

    def persistent_scratch_bytes(self, *, layers: int, hidden: int, q_heads: int, kv_heads: int, head_dim: int,
                                 intermediate: int, kv_capacity: int) -> int:
        self._check_open()
        n = int(self.lib.kudacuda_sm100_decode_persistent_scratch_bytes(
            self.engine_handle, int(layers), int(hidden), int(q_heads), int(kv_heads), int(head_dim),
            int(intermediate), int(kv_capacity)))
        if n < 0:
            raise NativeCudaError(f"kudacuda_sm100_decode_persistent_scratch_bytes: {self._native_error()}")
        return n

    def dispatch_decode_layers_persistent(self, layer_table: Any, x: Any, state: Any, rope_cos: Any, rope_sin: Any,
                                          scratch: Any, *, layers: int, max_pos: int,
                                          hidden: int, q_heads: int, kv_heads: int, head_dim: int, intermediate: int,
                                          kv_capacity: int, epsilon: float, scale: float, stream_ptr: int,
                                          taps: Any = None, spin_limit: int = 0, stall_counter: int = -1) -> None:
        args = [self._tensor_pointer(layer_table, "layer_table"), int(layers), self._tensor_pointer(x, "x"),
                self._tensor_pointer(state, "state"), self._tensor_pointer(rope_cos, "rope_cos"),
                self._tensor_pointer(rope_sin, "rope_sin"), int(max_pos), self._tensor_pointer(scratch, "scratch"),
                int(scratch.numel()) * int(scratch.element_size()), int(hidden), int(q_heads), int(kv_heads),
                int(head_dim), int(intermediate), int(kv_capacity), float(epsilon), float(scale)]
        if taps is None and not spin_limit and stall_counter < 0:
            self._call("kudacuda_sm100_decode_layers_persistent", *args, _normalize_cuda_handle(stream_ptr))
            return
        tp = 0 if taps is None else self._tensor_pointer(taps, "taps")
        tb = 0 if taps is None else int(taps.numel()) * int(taps.element_size())
        self._call("kudacuda_sm100_decode_layers_persistent_debug", *args, tp, tb, int(spin_limit),
                   int(stall_counter), _normalize_cuda_handle(stream_ptr))

    def persistent_tap_elements(self, *, layers: int, hidden: int, q_heads: int, kv_heads: int, head_dim: int,
                                intermediate: int) -> int:
        n = int(self.lib.kudacuda_sm100_decode_persistent_tap_elements(int(layers), int(hidden), int(q_heads),
                                                                         int(kv_heads), int(head_dim),
                                                                         int(intermediate)))
        if n < 0:
            raise NativeCudaError("kudacuda_sm100_decode_persistent_tap_elements: unsupported shapes")
        return n

    # ---------------------------------------------------------------- batched decode (B sequences per step)
    def batch_gemm_ksplit(self, rows: int, k: int) -> int:
        n = int(self.lib.kudacuda_sm100_batch_gemm_ksplit(int(rows), int(k)))
        if n < 1:
            raise ValueError(f"batch_gemm_ksplit: unsupported shape rows={rows} k={k}")
        return n

    def batch_retile_bytes(self, rows: int, k: int) -> int:
        n = int(self.lib.kudacuda_sm100_batch_retile_bytes(int(rows), int(k)))
        if n < 0:
            raise ValueError(f"batch_retile_bytes: unsupported shape rows={rows} k={k}")
        return n

    def dispatch_batch_retile(self, packed: Any, absmax: Any, out: Any, *, rows: int, k: int, stream_ptr: int) -> None:
        """bitsandbytes NF4 -> the batched GEMM's streaming form (weight_type 2)."""

        self._call("kudacuda_sm100_batch_retile", self._tensor_pointer(packed, "packed"),
                   self._tensor_pointer(absmax, "absmax"), int(rows), int(k), self._tensor_pointer(out, "out"),
                   int(out.numel()) * int(out.element_size()), _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_gemm(self, weight: Any, absmax: Any, x: Any, partials: Any, *, weight_type: int, rows: int,
                            k: int, n_pad: int, ksplit: int, row_offset: int = 0, total_rows: int | None = None,
                            stream_ptr: int) -> None:
        """fp32 split-K partials of W . x^T for a padded batch on the tensor cores
        (weight_type 0: NF4 + absmax, 1: bf16, 2: NF4 re-tiled by dispatch_batch_retile)."""

        total = int(rows if total_rows is None else total_rows)
        if int(x.numel()) != int(n_pad) * int(k):
            raise ValueError("x must be [n_pad, k]")
        if int(partials.numel()) < int(ksplit) * total * int(n_pad):
            raise ValueError("partials must hold ksplit * total_rows * n_pad floats")
        self._call("kudacuda_sm100_batch_gemm", int(weight_type), self._tensor_pointer(weight, "weight"),
                   self._optional_pointer(absmax, "absmax"), int(rows), int(k), self._tensor_pointer(x, "x"),
                   int(n_pad), int(ksplit), self._tensor_pointer(partials, "partials"), int(row_offset), total,
                   _normalize_cuda_handle(stream_ptr))

    def _fused_gemm_common(self, weight: Any, absmax: Any, x: Any, partials: Any, tickets: Any) -> list:
        return [self._tensor_pointer(weight, "weight"), self._optional_pointer(absmax, "absmax")], \
            [self._tensor_pointer(x, "x")], [self._tensor_pointer(partials, "partials"),
                                             int(partials.numel()) * int(partials.element_size()),
                                             self._tensor_pointer(tickets, "tickets")]

    def dispatch_batch_gemm_residual(self, weight: Any, absmax: Any, x: Any, partials: Any, tickets: Any, resid: Any, *,
                                     weight_type: int, rows: int, k: int, n_pad: int, ksplit: int, batch: int,
                                     stream_ptr: int) -> None:
        """GEMM + fused residual epilogue: resid[b][r] = bf16(resid + bf16(W . x[b]))."""

        w, xx, pt = self._fused_gemm_common(weight, absmax, x, partials, tickets)
        self._call("kudacuda_sm100_batch_gemm_residual", int(weight_type), *w, int(rows), int(k), *xx, int(n_pad),
                   int(ksplit), int(batch), *pt, self._tensor_pointer(resid, "resid"),
                   _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_gemm_swiglu(self, weight: Any, absmax: Any, x: Any, partials: Any, tickets: Any, out: Any, *,
                                   weight_type: int, intermediate: int, k: int, n_pad: int, ksplit: int, batch: int,
                                   stream_ptr: int) -> None:
        """GEMM over gate|up weights in 64-row gate/up tiles + fused SwiGLU."""

        w, xx, pt = self._fused_gemm_common(weight, absmax, x, partials, tickets)
        self._call("kudacuda_sm100_batch_gemm_swiglu", int(weight_type), *w, int(intermediate), int(k), *xx,
                   int(n_pad), int(ksplit), int(batch), *pt, self._tensor_pointer(out, "out"),
                   _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_gemm_qkv_rope(self, weight: Any, absmax: Any, x: Any, partials: Any, tickets: Any,
                                     q_bias: Any, k_bias: Any, v_bias: Any, rope_cos: Any, rope_sin: Any, pos: Any,
                                     q_out: Any, key_cache: Any, value_cache: Any, *, weight_type: int, k: int,
                                     n_pad: int, ksplit: int, batch: int, q_heads: int, kv_heads: int, head_dim: int,
                                     max_pos: int, kv_capacity: int, shared_cache: bool = False,
                                     stream_ptr: int) -> None:
        """GEMM over q|k|v weights + fused bias, RoPE and K/V append per head."""

        w, xx, pt = self._fused_gemm_common(weight, absmax, x, partials, tickets)
        self._call("kudacuda_sm100_batch_gemm_qkv_rope", int(weight_type), *w, int(k), *xx, int(n_pad), int(ksplit),
                   int(batch), *pt, int(q_heads), int(kv_heads), int(head_dim),
                   self._optional_pointer(q_bias, "q_bias"), self._optional_pointer(k_bias, "k_bias"),
                   self._optional_pointer(v_bias, "v_bias"), self._tensor_pointer(rope_cos, "rope_cos"),
                   self._tensor_pointer(rope_sin, "rope_sin"), int(max_pos), self._tensor_pointer(pos, "pos"),
                   self._tensor_pointer(q_out, "q_out"), self._tensor_pointer(key_cache, "key_cache"),
                   self._tensor_pointer(value_cache, "value_cache"), int(kv_capacity), 1 if shared_cache else 0,
                   _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_rmsnorm(self, x: Any, weight: Any, out: Any, *, batch: int, hidden: int, epsilon: float,
                               stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_rmsnorm", self._tensor_pointer(x, "x"), self._tensor_pointer(weight, "weight"),
                   self._tensor_pointer(out, "out"), int(batch), int(hidden), float(epsilon),
                   _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_qkv_rope(self, partials: Any, q_bias: Any, k_bias: Any, v_bias: Any, rope_cos: Any,
                                rope_sin: Any, pos: Any, q_out: Any, key_cache: Any, value_cache: Any, *, ksplit: int,
                                n_pad: int, batch: int, q_heads: int, kv_heads: int, head_dim: int, max_pos: int,
                                kv_capacity: int, shared_cache: bool = False, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_qkv_rope", self._tensor_pointer(partials, "partials"), int(ksplit), int(n_pad),
                   int(batch), int(q_heads), int(kv_heads), int(head_dim), self._optional_pointer(q_bias, "q_bias"),
                   self._optional_pointer(k_bias, "k_bias"), self._optional_pointer(v_bias, "v_bias"),
                   self._tensor_pointer(rope_cos, "rope_cos"), self._tensor_pointer(rope_sin, "rope_sin"), int(max_pos),
                   self._tensor_pointer(pos, "pos"), self._tensor_pointer(q_out, "q_out"),
                   self._tensor_pointer(key_cache, "key_cache"), self._tensor_pointer(value_cache, "value_cache"),
                   int(kv_capacity), 1 if shared_cache else 0, _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_residual(self, partials: Any, x: Any, *, ksplit: int, rows: int, n_pad: int, batch: int,
                                stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_residual", self._tensor_pointer(partials, "partials"), int(ksplit), int(rows),
                   int(n_pad), int(batch), self._tensor_pointer(x, "x"), _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_swiglu(self, partials: Any, out: Any, *, ksplit: int, intermediate: int, n_pad: int,
                              batch: int, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_swiglu", self._tensor_pointer(partials, "partials"), int(ksplit),
                   int(intermediate), int(n_pad), int(batch), self._tensor_pointer(out, "out"),
                   _normalize_cuda_handle(stream_ptr))

    def batch_argmax_workspace_bytes(self, batch: int) -> int:
        n = int(self.lib.kudacuda_sm100_batch_argmax_workspace_bytes(int(batch)))
        if n < 0:
            raise ValueError(f"batch_argmax_workspace_bytes: unsupported batch {batch}")
        return n

    def dispatch_batch_argmax_advance(self, partials: Any, workspace: Any, state: Any, history: Any = None, *,
                                      ksplit: int, vocab: int, n_pad: int, batch: int, stream_ptr: int) -> None:
        hist_len = int(history.shape[-1]) if history is not None else 0
        self._call("kudacuda_sm100_batch_argmax_advance", self._tensor_pointer(partials, "partials"), int(ksplit),
                   int(vocab), int(n_pad), int(batch), self._tensor_pointer(workspace, "workspace"),
                   int(workspace.numel()) * int(workspace.element_size()), self._tensor_pointer(state, "state"),
                   self._optional_pointer(history, "history"), hist_len, _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_embedding(self, embedding: Any, state: Any, x: Any, *, batch: int, hidden: int, vocab: int,
                                 stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_embedding", self._tensor_pointer(embedding, "embedding"),
                   self._tensor_pointer(state, "state"), self._tensor_pointer(x, "x"), int(batch), int(hidden),
                   int(vocab), _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_state_views(self, state: Any, pos: Any, kv_len: Any, *, batch: int, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_state_views", self._tensor_pointer(state, "state"), int(batch),
                   self._tensor_pointer(pos, "pos"), self._tensor_pointer(kv_len, "kv_len"),
                   _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_split_sum(self, partials: Any, out: Any, *, ksplit: int, rows: int, n_pad: int,
                                 stream_ptr: int) -> None:
        if int(out.numel()) < int(rows) * int(n_pad):
            raise ValueError("out must hold rows * n_pad floats")
        self._call("kudacuda_sm100_batch_split_sum", self._tensor_pointer(partials, "partials"), int(ksplit), int(rows),
                   int(n_pad), self._tensor_pointer(out, "out"), _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_argmax_pairs(self, partials: Any, workspace: Any, pairs: Any, *, ksplit: int, vocab: int,
                                    n_pad: int, batch: int, index_base: int, stream_ptr: int) -> None:
        self._call("kudacuda_sm100_batch_argmax_pairs", self._tensor_pointer(partials, "partials"), int(ksplit),
                   int(vocab), int(n_pad), int(batch), self._tensor_pointer(workspace, "workspace"),
                   int(workspace.numel()) * int(workspace.element_size()), int(index_base),
                   self._tensor_pointer(pairs, "pairs"), _normalize_cuda_handle(stream_ptr))

    def dispatch_batch_select_advance(self, gathered: Any, state: Any, history: Any = None, *, world: int, batch: int,
                                      stream_ptr: int) -> None:
        hist_len = int(history.shape[-1]) if history is not None else 0
        self._call("kudacuda_sm100_batch_select_advance", self._tensor_pointer(gathered, "gathered"), int(world),
                   int(batch), self._tensor_pointer(state, "state"), self._optional_pointer(history, "history"),
                   hist_len, _normalize_cuda_handle(stream_ptr))

    def gqa_batch_workspace(self, *, batch: int, query_heads: int, kv_heads: int, kv_stride: int, device: Any,
                            torch_module: Any = None) -> tuple[Any, Any]:
        """(workspace, tickets) for dispatch_gqa_decode_batch, allocated once
        through torch (tickets zero; the kernels leave them zero)."""

        if torch_module is None:
            import torch as torch_module
        n = int(self.lib.kudacuda_sm100_gqa_batch_workspace_bytes(int(batch), int(query_heads), int(kv_heads),
                                                                   int(kv_stride)))
        if n <= 0:
            raise NativeCudaError("kudacuda_sm100_gqa_batch_workspace_bytes rejected the shape")
        ws = torch_module.empty((n // 4,), dtype=torch_module.float32, device=device)
        tickets = torch_module.zeros((int(batch) * int(kv_heads),), dtype=torch_module.int32, device=device)
        return ws, tickets

    def dispatch_gqa_decode_batch(self, query: Any, key_cache: Any, value_cache: Any, output: Any, workspace: Any,
                                  tickets: Any, kv_len: Any, *, batch: int, kv_stride: int, query_heads: int,
                                  kv_heads: int, head_dim: int = 128, scale: float | None = None,
                                  shared_cache: bool = False, stream_ptr: int) -> None:
        """Split-KV GQA decode of B sequences with per-sequence lengths kv_len (int32 [B])."""

        sc = float(scale) if scale is not None else 1.0 / math.sqrt(head_dim)
        self._call("kudacuda_sm100_gqa_decode_batch", self._tensor_pointer(query, "query"),
                   self._tensor_pointer(key_cache, "key_cache"), self._tensor_pointer(value_cache, "value_cache"),
                   self._tensor_pointer(output, "output"), self._tensor_pointer(workspace, "workspace"),
                   int(workspace.numel()) * int(workspace.element_size()), self._tensor_pointer(tickets, "tickets"),
                   self._tensor_pointer(kv_len, "kv_len"), int(batch), int(kv_stride), int(query_heads),
                   int(kv_heads), int(head_dim), sc, 1 if shared_cache else 0, _normalize_cuda_handle(stream_ptr))

    def error_word(self, *, clear: bool = True) -> int:
        word = ctypes.c_int(0)
        self._raise_if_failed(self.lib.kudacuda_sm100_error_word(self.engine_handle, ctypes.byref(word), int(clear)),
                              "kudacuda_sm100_error_word")
        return int(word.value)

    # ---------------------------------------------------------------- graphs
    def begin_capture(self, *, stream_ptr: int) -> None:
        self._raise_if_failed(self.lib.kudacuda_begin_capture(self.engine_handle, _normalize_cuda_handle(stream_ptr)),
                              "kudacuda_begin_capture")

    def end_capture(self, *, stream_ptr: int) -> None:
        self._raise_if_failed(self.lib.kudacuda_end_capture(self.engine_handle, _normalize_cuda_handle(stream_ptr)),
                              "kudacuda_end_capture")

    def replay_graph(self, *, stream_ptr: int) -> None:
        self._raise_if_failed(self.lib.kudacuda_replay_graph(self.engine_handle, _normalize_cuda_handle(stream_ptr)),
                              "kudacuda_replay_graph")

    def reset_graph(self) -> None:
        self._raise_if_failed(self.lib.kudacuda_reset_graph(self.engine_handle), "kudacuda_reset_graph")

    def graph_step_host(self, host_in: Any, device_in: Any, host_out: Any, device_out: Any, *, stream_ptr: int) -> None:
        """One replay with host input/output copies (kudacuda_sm100_graph_step_host); synchronises."""

        in_bytes = int(host_in.numel()) * int(host_in.element_size())
        out_bytes = int(host_out.numel()) * int(host_out.element_size())
        status = self.lib.kudacuda_sm100_graph_step_host(
            self.engine_handle, ctypes.c_void_p(int(host_in.data_ptr())), self._tensor_pointer(device_in, "device_in"),
            in_bytes, ctypes.c_void_p(int(host_out.data_ptr())), self._tensor_pointer(device_out, "device_out"),
            out_bytes, _normalize_cuda_handle(stream_ptr))
        self._raise_if_failed(status, "kudacuda_sm100_graph_step_host")

    def bind_graph_step_host(self, host_in: Any, device_in: Any, host_out: Any, device_out: Any, *,
                             stream_ptr: int) -> Any:
        """graph_step_host with its four buffers and the stream resolved once,
        for a decode loop.

        Returns a callable that runs one step through the same C entry
        (kudacuda_sm100_graph_step_host: H2D of host_in, graph replay, D2H into
        host_out, stream synchronise) and raises on a non-zero status.  The
        callable keeps the tensors alive; write each step's input into host_in
        (``host_in.numpy()`` is a view of pinned memory) before the call and
        read host_out after it.  The graph itself is looked up at each call, so
        a re-instantiated graph needs no new binding.
        """

        in_bytes = int(host_in.numel()) * int(host_in.element_size())
        out_bytes = int(host_out.numel()) * int(host_out.element_size())
        args = (self.engine_handle, ctypes.c_void_p(int(host_in.data_ptr())),
                self._tensor_pointer(device_in, "device_in"), in_bytes, ctypes.c_void_p(int(host_out.data_ptr())),
                self._tensor_pointer(device_out, "device_out"), out_bytes, _normalize_cuda_handle(stream_ptr))
        fn = self.lib.kudacuda_sm100_graph_step_host
        buffers = (host_in, device_in, host_out, device_out)

        def step() -> None:
            status = fn(*args)
            if status != 0:
                self._raise_if_failed(status, "kudacuda_sm100_graph_step_host")

        step.buffers = buffers  # type: ignore[attr-defined]
        return step

    # ---------------------------------------------------------------- lifetime
    def shutdown(self) -> None:
        if not self._closed:
            self.lib.kudacuda_destroy(self.engine_handle)
            self._closed = True
            self.engine_handle = None

    def __enter__(self) -> "KudaCudaBridge":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.shutdown()

    def __del__(self) -> None:
        try:
            self.shutdown()
        except Exception:
            pass


# ====================================================================== hooks
def _install(cls: Any, replacement: Callable) -> Callable[[], None]:
    original = cls.forward
    cls.forward = replacement
    done = False

    def unpatch() -> None:
        nonlocal done
        if not done:
            cls.forward = original
            done = True

    return unpatch


def patch_llama_attention(bridge: Any, *, attention_cls: Any = None, tactic_name: str = "gqa8_attn") -> Callable[[], None]:
    """Guarded attention hook: dispatch to ``bridge.dispatch_attention`` only
    when the tactic's contract matches, else the original forward."""

    if attention_cls is None:
        from transformers.models.llama.modeling_llama import LlamaAttention

        attention_cls = LlamaAttention
    original = attention_cls.forward

    @wraps(original)
    def forward(self: Any, hidden_states: Any, *args: Any, **kwargs: Any) -> Any:
        try:
            shape = _shape(hidden_states)
            dispatcher = getattr(bridge, "dispatch_attention", None)
            if (
                len(shape) >= 2
                and callable(dispatcher)
                and bridge.matches_contract(tactic_name, shape[0], shape[1], tensor=hidden_states)
            ):
                return dispatcher(self, hidden_states, *args, **kwargs)
        except Exception:
            pass
        return original(self, hidden_states, *args, **kwargs)

    return _install(attention_cls, forward)


def patch_qwen2_attention(bridge: Any, *, attention_cls: Any = None,
                          tactic_name: str = "qwen2_gqa_decode_sm100_fp16") -> Callable[[], None]:
    """Route Qwen2 decode attention through the native GQA with framework fallback."""

    if attention_cls is None:
        from transformers.models.qwen2.modeling_qwen2 import Qwen2Attention

        attention_cls = Qwen2Attention
    original = attention_cls.forward

    @wraps(original)
    def forward(self: Any, hidden_states: Any, *args: Any, **kwargs: Any) -> Any:
        try:
            dispatcher = getattr(bridge, "dispatch_qwen2_attention", None)
            if len(_shape(hidden_states)) >= 2 and callable(dispatcher):
                result = dispatcher(self, hidden_states, *args, tactic_name=tactic_name, **kwargs)
                if result is not None:
                    return result
        except Exception:
            pass
        return original(self, hidden_states, *args, **kwargs)

    return _install(attention_cls, forward)


def _decoder_layers(model: Any) -> list[Any]:
    layers = getattr(getattr(model, "model", None), "layers", None)
    if layers is None:
        raise ValueError("Qwen2 model does not expose model.layers")
    return list(layers)


def prepare_qwen2_fused_qkv(model: Any, *, torch_module: Any = None) -> None:
    """One stable Q/K/V (+ fp32 normalised) buffer set per decoder layer,
    allocated before graph capture so replays see fixed addresses."""

    if torch_module is None:
        import torch as torch_module
    for layer in _decoder_layers(model):
        attention = getattr(layer, "self_attn", None)
        weight = getattr(getattr(layer, "input_layernorm", None), "weight", None)
        if attention is None or weight is None:
            raise ValueError("Qwen2 decoder layer is missing self_attn or input_layernorm")
        device, dtype = getattr(weight, "device", None), getattr(weight, "dtype", None)
        if device is None or dtype is None:
            raise ValueError("Qwen2 input layernorm weight has no device/dtype")
        attention._kudacuda_fused_qkv_state = {
            "normalized": torch_module.empty((1, 2048), device=device, dtype=torch_module.float32),
            "query": torch_module.empty((1, 2048), device=device, dtype=dtype),
            "key": torch_module.empty((1, 256), device=device, dtype=dtype),
            "value": torch_module.empty((1, 256), device=device, dtype=dtype),
        }


def prepare_qwen2_swiglu(model: Any, *, torch_module: Any = None) -> None:
    """One stable SwiGLU output buffer per decoder layer."""

    if torch_module is None:
        import torch as torch_module
    for layer in _decoder_layers(model):
        mlp = getattr(layer, "mlp", None)
        weight = getattr(getattr(layer, "post_attention_layernorm", None), "weight", None)
        if mlp is None or weight is None:
            raise ValueError("Qwen2 decoder layer is missing mlp or post-attention layernorm")
        layer._kudacuda_swiglu_state = {
            "output": torch_module.empty((1, 11008), device=weight.device, dtype=weight.dtype),
        }


def _stream_of(torch_module: Any, tensor: Any) -> int:
    if torch_module is None:
        import torch as torch_module
    return int(torch_module.cuda.current_stream(tensor.device).cuda_stream)


_MISSING = object()


def _restore_attr(obj: Any, name: str, previous: Any) -> None:
    if previous is _MISSING:
        if hasattr(obj, name):
            try:
                delattr(obj, name)
            except AttributeError:
                pass
    else:
        setattr(obj, name, previous)


def patch_qwen2_swiglu(model: Any, bridge: Any, *, tactic_name: str = "qwen2_swiglu_sm100_nf4_v1",
                       prepare: bool = True, torch_module: Any = None) -> Callable[[], None]:
    """Run each exact Qwen2.5-3B decoder layer's post-attention RMSNorm +
    gate/up SwiGLU natively (down_proj stays in the framework, as in the
    reference); anything unsupported runs the layer's original forward."""

    layers = _decoder_layers(model)
    if not layers:
        raise ValueError("Qwen2 model does not expose decoder layers")
    dispatch = bridge.dispatch_qwen2_swiglu_nf4_bf16 if "_bf16_" in tactic_name else bridge.dispatch_qwen2_swiglu_nf4
    saved = [(layer, layer.forward, getattr(layer, "_kudacuda_swiglu_state", _MISSING)) for layer in layers]
    if prepare:
        prepare_qwen2_swiglu(model, torch_module=torch_module)

    for layer, original, _ in saved:

        def forward(self: Any, hidden_states: Any, attention_mask: Any = None, position_ids: Any = None,
                    past_key_values: Any = None, use_cache: Any = False, position_embeddings: Any = None,
                    _layer: Any = layer, _original: Any = original, **kwargs: Any) -> Any:
            call = dict(attention_mask=attention_mask, position_ids=position_ids, past_key_values=past_key_values,
                        use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
            bridge.native_swiglu_hook_calls = int(getattr(bridge, "native_swiglu_hook_calls", 0)) + 1
            shape = _shape(hidden_states)
            if shape != (1, 1, 2048):
                bridge.last_swiglu_dispatch_reason = f"shape:{shape}"
                return _original(hidden_states, **call)
            state = getattr(_layer, "_kudacuda_swiglu_state", None)
            if not isinstance(state, dict) or "output" not in state:
                bridge.last_swiglu_dispatch_reason = "missing_workspace"
                return _original(hidden_states, **call)
            residual = None
            try:
                attn, _ = _layer.self_attn(hidden_states=_layer.input_layernorm(hidden_states), **call)
                residual = hidden_states + attn

                def framework_mlp(value: Any) -> Any:
                    return value + _layer.mlp(_layer.post_attention_layernorm(value))

                flat = residual.reshape(1, 2048)
                if not bool(flat.is_contiguous()):
                    bridge.last_swiglu_dispatch_reason = "non_contiguous_input"
                    return framework_mlp(residual)
                gate, up = _layer.mlp.gate_proj, _layer.mlp.up_proj
                g_state = getattr(gate.weight, "quant_state", None)
                u_state = getattr(up.weight, "quant_state", None)
                if g_state is None or u_state is None:
                    bridge.last_swiglu_dispatch_reason = "missing_quant_state"
                    return framework_mlp(residual)
                if getattr(gate, "bias", None) is not None or getattr(up, "bias", None) is not None:
                    bridge.last_swiglu_dispatch_reason = "unexpected_projection_bias"
                    return framework_mlp(residual)
                norm = _layer.post_attention_layernorm
                dispatch(flat, norm.weight, gate.weight, g_state.absmax, up.weight, u_state.absmax, state["output"],
                         epsilon=float(getattr(norm, "variance_epsilon", 1.0e-6)),
                         stream_ptr=_stream_of(torch_module, flat), tactic_name=tactic_name)
                bridge.last_swiglu_dispatch_reason = "native"
                return residual + _layer.mlp.down_proj(state["output"].reshape(1, 1, 11008))
            except Exception as error:
                bridge.last_swiglu_dispatch_reason = f"fallback:{type(error).__name__}:{error}"
                if residual is not None:
                    return residual + _layer.mlp(_layer.post_attention_layernorm(residual))
                return _original(hidden_states, **call)

        layer.forward = MethodType(forward, layer)

    done = False

    def unpatch() -> None:
        nonlocal done
        if done:
            return
        for layer, original, previous in saved:
            layer.forward = original
            _restore_attr(layer, "_kudacuda_swiglu_state", previous)
        done = True

    return unpatch


def patch_qwen2_fused_qkv(model: Any, bridge: Any, *, tactic_name: str = "qwen2_fused_rmsnorm_qkv_sm100_nf4_v1",
                          attention_tactic_name: str = "qwen2_gqa_decode_sm100_fp16", prepare: bool = True,
                          torch_module: Any = None, attention_cls: Any = None) -> Callable[[], None]:
    """Run each decoder layer's input RMSNorm + NF4 Q/K/V natively, then hand
    the pre-fused q/k/v to the (patched) attention module for RoPE, the cache
    update, GQA and o_proj.  Any unsupported case runs the original forward."""

    layers = _decoder_layers(model)
    if not layers:
        raise ValueError("Qwen2 model does not expose decoder layers")
    if attention_cls is None:
        attention_cls = type(layers[0].self_attn)
    if prepare:
        prepare_qwen2_fused_qkv(model, torch_module=torch_module)
    attention_unpatch = patch_qwen2_attention(bridge, attention_cls=attention_cls, tactic_name=attention_tactic_name)
    saved = []
    for layer in layers:
        attn = layer.self_attn
        saved.append((layer, layer.forward, getattr(attn, "_kudacuda_fused_qkv_state", _MISSING),
                      getattr(attn, "_kudacuda_prefused_qkv", _MISSING)))

        def forward(self: Any, hidden_states: Any, *args: Any, _layer: Any = layer, _attn: Any = attn,
                    _original: Any = layer.forward, **kwargs: Any) -> Any:
            bridge.native_fused_qkv_hook_calls = int(getattr(bridge, "native_fused_qkv_hook_calls", 0)) + 1
            shape = _shape(hidden_states)
            if shape != (1, 1, 2048):
                if int(getattr(bridge, "native_fused_qkv_dispatches", 0)) == 0:
                    bridge.last_qwen2_fused_qkv_dispatch_reason = f"shape:{shape}"
                return _original(hidden_states, *args, **kwargs)
            state = getattr(_attn, "_kudacuda_fused_qkv_state", None)
            if not isinstance(state, dict) or not all(k in state for k in ("query", "key", "value")):
                bridge.last_qwen2_fused_qkv_dispatch_reason = "missing_workspace"
                return _original(hidden_states, *args, **kwargs)
            before = getattr(_attn, "_kudacuda_prefused_qkv", _MISSING)
            try:
                flat = hidden_states.reshape(1, 2048)
                if not bool(flat.is_contiguous()):
                    bridge.last_qwen2_fused_qkv_dispatch_reason = "non_contiguous_input"
                    return _original(hidden_states, *args, **kwargs)
                norm = _layer.input_layernorm
                projs = (_attn.q_proj, _attn.k_proj, _attn.v_proj)
                states = [getattr(p.weight, "quant_state", None) for p in projs]
                if any(s is None for s in states):
                    bridge.last_qwen2_fused_qkv_dispatch_reason = "missing_quant_state"
                    return _original(hidden_states, *args, **kwargs)
                biases = [getattr(p, "bias", None) for p in projs]
                if any(b is None for b in biases):
                    bridge.last_qwen2_fused_qkv_dispatch_reason = "missing_projection_bias"
                    return _original(hidden_states, *args, **kwargs)
                bridge.dispatch_qwen2_fused_rmsnorm_qkv_nf4(
                    flat, norm.weight,
                    projs[0].weight, states[0].absmax, biases[0],
                    projs[1].weight, states[1].absmax, biases[1],
                    projs[2].weight, states[2].absmax, biases[2],
                    state["query"], state["key"], state["value"],
                    normalized_workspace=state.get("normalized"),
                    epsilon=float(getattr(norm, "variance_epsilon", 1.0e-6)),
                    stream_ptr=_stream_of(torch_module, hidden_states), tactic_name=tactic_name)
                bridge.last_qwen2_fused_qkv_dispatch_reason = "native"
                _attn._kudacuda_prefused_qkv = (state["query"], state["key"], state["value"])
                out = _attn(hidden_states, *args, **kwargs)
                hidden = hidden_states + (out[0] if isinstance(out, tuple) else out)
                return hidden + _layer.mlp(_layer.post_attention_layernorm(hidden))
            except Exception as error:
                bridge.last_qwen2_fused_qkv_dispatch_reason = f"fallback:{type(error).__name__}:{error}"
                return _original(hidden_states, *args, **kwargs)
            finally:
                _restore_attr(_attn, "_kudacuda_prefused_qkv", before)

        layer.forward = MethodType(forward, layer)

    done = False

    def unpatch() -> None:
        nonlocal done
        if done:
            return
        for layer, original, prev_state, prev_prefused in saved:
            layer.forward = original
            _restore_attr(layer.self_attn, "_kudacuda_fused_qkv_state", prev_state)
            _restore_attr(layer.self_attn, "_kudacuda_prefused_qkv", prev_prefused)
        attention_unpatch()
        done = True

    return unpatch
