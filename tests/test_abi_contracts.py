"""CPU tests of the drop-in boundary: the C-ABI library loads and exports every
symbol the headers declare, the tactic table and manifest agree, and the
Python sidecar applies the reference's contracts and argument order
(python/kudacuda_sidecar.py:66-165, 259-419, 1017-1049) before anything
reaches native code.  Native calls go to a recording fake, so no GPU is
needed; the same checks the reference's tests/test_contracts.py makes about
its bridge are made here about this one.
"""

import ctypes
import math
import re
from pathlib import Path
from types import SimpleNamespace

import pytest

from kudacuda_b200 import build as kbuild
from kudacuda_b200 import native
from kudacuda_b200.kudacuda_sidecar import (
    DEFAULT_MANIFEST,
    KudaCudaBridge,
    NativeCudaError,
    Qwen2GqaContract,
    TensorContract,
    _qwen2_attention_dimensions,
    load_manifest,
    select_library_name,
)

ROOT = Path(__file__).resolve().parents[1]
HEADERS = [ROOT / "include" / "kudacuda.h", ROOT / "include" / "kudacuda_registry.h"]


def _declared_symbols() -> list[str]:
    names = []
    for h in HEADERS:
        text = h.read_text()
        # C functions: "KUDACUDA_API <type> <name>(" and plain extern "C" prototypes "<type> kudacuda_<name>("
        names += re.findall(r"\b(kudacuda_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    path = kbuild.build()  # no-op when up to date; nvcc cross-compiles without a GPU
    return ctypes.CDLL(str(path))


def test_library_exports_every_declared_symbol(lib):
    declared = _declared_symbols()
    assert len(declared) >= 40
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_every_declared_symbol_has_a_ctypes_signature():
    declared = set(_declared_symbols())
    known = set(native.SIGNATURES)
    # the registry helpers are C++-class internals of KudaCudaModuleRegistry or return plain ints
    missing = sorted(n for n in declared - known if not n.startswith("kudacuda_tactic_"))
    assert not missing, f"no ctypes signature for {missing}"
    assert not (known - declared), f"signatures for undeclared symbols: {sorted(known - declared)}"


def test_reference_abi_names_are_all_present():
    # include/kudacuda.h:19-267 of the reference, by name
    reference = [
        "kudacuda_create", "kudacuda_freeze", "kudacuda_can_dispatch", "kudacuda_vector_add", "kudacuda_rmsnorm",
        "kudacuda_fused_rmsnorm_qkv", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2",
        "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3", "kudacuda_qwen2_swiglu_nf4", "kudacuda_qwen2_swiglu_nf4_bf16",
        "kudacuda_qwen2_gqa_decode_workspace_v3", "kudacuda_qwen2_gqa_decode", "kudacuda_qwen2_gqa_decode_graph",
        "kudacuda_qwen2_gqa_decode_group_tiled", "kudacuda_qwen2_gqa_decode_vectorized", "kudacuda_begin_capture",
        "kudacuda_end_capture", "kudacuda_replay_graph", "kudacuda_reset_graph", "kudacuda_last_error",
        "kudacuda_destroy",
    ]
    declared = set(_declared_symbols())
    assert [n for n in reference if n not in declared] == []


def test_library_has_no_cuda_runtime_link_dependency():
    # the CUDA runtime is linked statically: the .so must load on a box with only the driver
    import subprocess

    out = subprocess.run(["ldd", str(kbuild.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcudart" not in out and "libcuda.so" not in out


def test_target_arch_and_tactic_table(lib):
    table = native.tactic_table(native.configure(lib))
    names = {row["name"] for row in table}
    symbols = {row["symbol"] for row in table}
    lib.kudacuda_sm100_target_arch.restype = ctypes.c_char_p
    assert lib.kudacuda_sm100_target_arch() == b"sm_100a"
    # the reference's sm86 tactic names stay resolvable (aliases of the sm_100a kernels)
    for ref_name in ("qwen2_gqa_decode_sm86_fp16", "qwen2_gqa_decode_sm86_fp16_graph_v1"):
        assert ref_name in names
    # every symbol the table points at is exported
    assert all(hasattr(lib, s) for s in symbols)
    # every implemented tactic of the B200 manifest is in the table
    manifest = load_manifest(DEFAULT_MANIFEST)
    assert manifest["target_arch"] == "sm_100a"
    assert [t for t in manifest["implemented_tactics"] if t not in names] == []


# --------------------------------------------------------------------- sidecar with a recording fake
class _Fn:
    def __init__(self, impl):
        self.impl = impl
        self.argtypes = None
        self.restype = None

    def __call__(self, *args):
        return self.impl(*args)


class FakeLib:
    """Records every native call; returns `status` from the dispatch entries."""

    def __init__(self, status: int = 0):
        self.calls = []
        self.status = status
        ok = lambda *a: 0  # noqa: E731
        self.kudacuda_create = _Fn(lambda dev: 4242)
        self.kudacuda_freeze = _Fn(ok)
        self.kudacuda_destroy = _Fn(lambda h: self.calls.append(("destroy", h)))
        self.kudacuda_last_error = _Fn(lambda h: b"injected native failure")
        self.kudacuda_can_dispatch = _Fn(lambda h, name, b, s: 1)
        for name in ("kudacuda_qwen2_gqa_decode", "kudacuda_qwen2_gqa_decode_graph",
                     "kudacuda_qwen2_gqa_decode_workspace_v3", "kudacuda_qwen2_gqa_decode_group_tiled",
                     "kudacuda_qwen2_gqa_decode_vectorized", "kudacuda_qwen2_swiglu_nf4",
                     "kudacuda_qwen2_swiglu_nf4_bf16", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4",
                     "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v2", "kudacuda_qwen2_fused_rmsnorm_qkv_nf4_v3",
                     "kudacuda_vector_add", "kudacuda_rmsnorm", "kudacuda_begin_capture", "kudacuda_end_capture",
                     "kudacuda_replay_graph", "kudacuda_reset_graph"):
            setattr(self, name, _Fn(self._recorder(name)))

    def _recorder(self, name):
        def record(*args):
            self.calls.append((name,) + args)
            return self.status

        return record


class FakeTensor:
    def __init__(self, dtype, shape, pointer, *, cuda=True, contiguous=True, quant_state=None):
        self.dtype = dtype
        self.shape = tuple(shape)
        self._ptr = pointer
        self.is_cuda = cuda
        self._contiguous = contiguous
        if quant_state is not None:
            self.quant_state = quant_state

    def data_ptr(self):
        return self._ptr

    def dim(self):
        return len(self.shape)

    def numel(self):
        return math.prod(self.shape)

    def is_contiguous(self):
        return self._contiguous


def _bridge(status=0):
    fake = FakeLib(status)
    return KudaCudaBridge(native_lib=fake), fake


def _gqa_tensors(dtype="float16", kv=128):
    return (FakeTensor(dtype, (1, 16, 1, 128), 11), FakeTensor(dtype, (1, 2, kv, 128), 22),
            FakeTensor(dtype, (1, 2, kv, 128), 33), FakeTensor(dtype, (1, 16, 1, 128), 44))


def test_attention_dimensions_follow_transformers_config_layout():
    module = SimpleNamespace(config=SimpleNamespace(num_attention_heads=16, num_key_value_heads=2), head_dim=128)
    assert _qwen2_attention_dimensions(module) == (16, 2, 128)


def test_qwen2_contract_accepts_only_the_decode_profile():
    c = Qwen2GqaContract.from_mapping(dict(dtype="float16", layout="contiguous", batch_size=1, query_len=1,
                                           kv_len_min=1, kv_len_max=512, query_heads=16, kv_heads=2, head_dim=128))
    assert c.matches(1, 1, 128) and c.matches(1, 1, 512)
    assert not c.matches(2, 1, 128) and not c.matches(1, 2, 128) and not c.matches(1, 1, 513)
    wrong_heads = Qwen2GqaContract.from_mapping(dict(dtype="float16", layout="contiguous", batch_size=1, query_len=1,
                                                     kv_len_min=1, kv_len_max=512, query_heads=32, kv_heads=8,
                                                     head_dim=128))
    assert not wrong_heads.matches(1, 1, 128)  # reference profile is fixed to 16/2/128


def test_b200_manifest_direct_profile_is_long_and_graph_profile_bounded():
    m = load_manifest(DEFAULT_MANIFEST)
    assert m["contracts"]["qwen2_gqa_decode_sm100_fp16"]["kv_len_max"] == 2048
    assert m["contracts"]["qwen2_gqa_decode_sm100_fp16_graph_v1"]["kv_len_max"] == 512
    assert Qwen2GqaContract.from_mapping(m["contracts"]["qwen2_gqa_decode_sm100_fp16"]).matches(1, 1, 585)


def test_gqa_dispatch_passes_pointers_dimensions_scale_and_stream_in_reference_order():
    bridge, fake = _bridge()
    bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(), kv_len=128, stream_ptr=77)
    call = fake.calls[-1]
    assert call[0] == "kudacuda_qwen2_gqa_decode"
    assert call[1:6] == (4242, 11, 22, 33, 44)
    assert call[6:12] == (1, 1, 128, 16, 2, 128)
    assert call[12] == pytest.approx(1.0 / math.sqrt(128.0))
    assert call[13] == 77
    assert bridge.native_attention_dispatches == 1


def test_native_failure_surfaces_the_native_message():
    bridge, _ = _bridge(status=1)
    with pytest.raises(NativeCudaError, match="injected native failure"):
        bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(), kv_len=128, stream_ptr=77)


def test_gqa_dispatch_rejects_wrong_dtype_shape_and_host_tensors_before_native():
    bridge, fake = _bridge()
    before = len(fake.calls)
    with pytest.raises(ValueError):
        bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(dtype="bfloat16"), kv_len=128, stream_ptr=1)
    q, k, v, o = _gqa_tensors()
    with pytest.raises(ValueError):
        bridge.dispatch_qwen2_gqa_decode(q, FakeTensor("float16", (1, 2, 64, 128), 22), v, o, kv_len=128,
                                         stream_ptr=1)
    with pytest.raises(ValueError):
        bridge.dispatch_qwen2_gqa_decode(FakeTensor("float16", (1, 16, 1, 128), 11, cuda=False), k, v, o,
                                         kv_len=128, stream_ptr=1)
    with pytest.raises(ValueError):
        bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(kv=4096), kv_len=4096, stream_ptr=1)
    assert len(fake.calls) == before  # nothing reached native code


def test_graph_tactic_needs_a_graph_context():
    bridge, _ = _bridge()
    with pytest.raises(NativeCudaError, match="graph"):
        bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(), kv_len=128, stream_ptr=1,
                                         tactic_name="qwen2_gqa_decode_sm100_fp16_graph_v1")


def test_unknown_tactic_is_rejected_and_status_reported():
    bridge, _ = _bridge()
    with pytest.raises(NativeCudaError):
        bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(), kv_len=128, stream_ptr=1, tactic_name="no_such_tactic")
    assert bridge.tactic_status("qwen2_gqa_decode_sm100_fp16") == "implemented"
    assert bridge.tactic_status("no_such_tactic") == "unknown"


def test_tensor_contract_requires_exact_batch_and_sequence_when_declared():
    c = TensorContract.from_mapping(dict(dtype="float32", layout="contiguous", batch_size=1, seq_len=1))
    assert c.matches_shape(1, 1)
    assert not c.matches_shape(2, 1) and not c.matches_shape(1, 2) and not c.matches_shape(0, 1)
    assert c.matches_tensor(FakeTensor("float32", (4,), 1))
    assert not c.matches_tensor(FakeTensor("float16", (4,), 1))
    assert not c.matches_tensor(FakeTensor("float32", (4,), 1, contiguous=False))


class _QuantState:
    def __init__(self, shape, blocksize=64, nested=False, quant_type="nf4"):
        self.shape = shape
        self.blocksize = blocksize
        self.nested = nested
        self.quant_type = quant_type


def test_nf4_weight_validation_follows_bitsandbytes_storage():
    n, k = 256, 2048
    packed = FakeTensor("uint8", (n * k // 2, 1), 5, quant_state=_QuantState((n, k)))
    absmax = FakeTensor("float32", (n * k // 64,), 6)
    assert KudaCudaBridge._validate_nf4_weight(packed, absmax, expected_shape=(n, k), label="w") == 64
    for bad in (_QuantState((n, k), blocksize=128), _QuantState((n, k), nested=True),
                _QuantState((n, k), quant_type="fp4"), _QuantState((n, 1024))):
        with pytest.raises(ValueError):
            KudaCudaBridge._validate_nf4_weight(FakeTensor("uint8", (n * k // 2, 1), 5, quant_state=bad), absmax,
                                                expected_shape=(n, k), label="w")
    with pytest.raises(ValueError):  # wrong absmax block count
        KudaCudaBridge._validate_nf4_weight(packed, FakeTensor("float32", (n * k // 128,), 6), expected_shape=(n, k),
                                            label="w")


def test_graph_lifecycle_calls_reach_native_with_the_stream():
    bridge, fake = _bridge()
    bridge.begin_capture(stream_ptr=5)
    bridge.end_capture(stream_ptr=5)
    bridge.replay_graph(stream_ptr=5)
    bridge.reset_graph()
    names = [c[0] for c in fake.calls]
    assert names[-4:] == ["kudacuda_begin_capture", "kudacuda_end_capture", "kudacuda_replay_graph",
                          "kudacuda_reset_graph"]
    assert fake.calls[-2][2] == 5


def test_shutdown_destroys_the_handle_once():
    bridge, fake = _bridge()
    bridge.shutdown()
    bridge.shutdown()
    assert [c for c in fake.calls if c[0] == "destroy"] == [("destroy", 4242)]
    with pytest.raises(NativeCudaError):
        bridge.dispatch_qwen2_gqa_decode(*_gqa_tensors(), kv_len=128, stream_ptr=1)


def test_platform_library_name():
    assert select_library_name("Linux").endswith(".so")


# ------------------------------------------------------------------ the reference's own bridge on this library
def _reference_checkout():
    import os

    env = os.environ.get("KUDACUDA_REFERENCE")
    for cand in ([Path(env)] if env else []) + [Path(__file__).resolve().parents[2] / "reference"]:
        if (cand / "python" / "kudacuda_sidecar.py").is_file():
            return cand
    return None


def test_reference_bridge_binds_this_library_and_manifest():
    """The reference's unmodified KudaCudaBridge (python/kudacuda_sidecar.py:
    185-431) loads this repository's manifest with its own loader and contract
    parsers, binds this library with its own ctypes argtypes (every symbol it
    binds resolves), gets a handle from kudacuda_create, and -- in a container
    without a GPU -- fails only at kudacuda_freeze, with this library's error
    message through its own error path."""

    import importlib.util
    import sys

    ref = _reference_checkout()
    if ref is None:
        pytest.skip("no reference checkout at hand (KUDACUDA_REFERENCE)")
    spec = importlib.util.spec_from_file_location("reference_kudacuda_sidecar", ref / "python" / "kudacuda_sidecar.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # its dataclasses look their module up
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.modules.pop(spec.name, None)
    manifest = Path(native.PACKAGE_DIR) / "manifests" / "b200-sm100.json"
    lib = ctypes.CDLL(str(native.DEFAULT_LIBRARY))
    assert mod.load_manifest(manifest)["target_arch"] == "sm_100a"
    try:
        bridge = mod.KudaCudaBridge(manifest=manifest, native_lib=lib, device_id=0)
    except mod.NativeCudaError as exc:  # no GPU here: the handle exists, freeze reports the device
        assert "kudacuda_freeze" in str(exc) and "cudaSetDevice" in str(exc), str(exc)
        return
    assert bridge.engine_handle  # on a machine with a GPU the bridge is fully usable
    bridge.shutdown()
