"""CPU tests of the decode-graph static contract (python/kudacuda_graph_plan.py
semantics): replay only under the captured key and stream, no nested capture,
invalidation clears the graph."""

import pytest

from kudacuda_b200.kudacuda_graph_plan import DecodeGraphKey, GraphContractError, KudaCudaGraphPlan


class RecordingBridge:
    def __init__(self, fail_end=False):
        self.calls = []
        self.fail_end = fail_end

    def begin_capture(self, *, stream_ptr):
        self.calls.append(("begin", stream_ptr))

    def end_capture(self, *, stream_ptr):
        self.calls.append(("end", stream_ptr))
        if self.fail_end:
            raise RuntimeError("capture failed")

    def replay_graph(self, *, stream_ptr):
        self.calls.append(("replay", stream_ptr))


def key(seed=100, bucket=512, rank=0):
    return DecodeGraphKey(device_id=0, tactic_name="decode_step_sm100_v1", layer_count=36,
                          query_shape=(1, 16, 1, 128), key_shape=(1, 2, bucket, 128),
                          value_shape=(1, 2, bucket, 128), output_shape=(1, 16, 1, 128), kv_bucket=bucket,
                          pointers=(seed, seed + 1, seed + 2), tp_rank=rank)


def test_capture_then_replay_under_the_same_key():
    br = RecordingBridge()
    plan = KudaCudaGraphPlan(br)
    plan.begin_capture(key(), stream_ptr=7)
    assert plan.capturing and not plan.captured
    plan.end_capture(key(), stream_ptr=7)
    plan.replay(key(), stream_ptr=7)
    assert br.calls == [("begin", 7), ("end", 7), ("replay", 7)]


@pytest.mark.parametrize("other", [key(seed=200), key(bucket=1024), key(rank=1)])
def test_changed_pointers_bucket_or_shard_is_refused(other):
    plan = KudaCudaGraphPlan(RecordingBridge())
    plan.begin_capture(key(), stream_ptr=7)
    plan.end_capture(key(), stream_ptr=7)
    assert not plan.can_replay(other, stream_ptr=7)
    with pytest.raises(GraphContractError, match="key"):
        plan.replay(other, stream_ptr=7)


def test_changed_stream_is_refused():
    plan = KudaCudaGraphPlan(RecordingBridge())
    plan.begin_capture(key(), stream_ptr=7)
    with pytest.raises(GraphContractError):
        plan.end_capture(key(), stream_ptr=8)
    plan.invalidate()
    plan.begin_capture(key(), stream_ptr=7)
    plan.end_capture(key(), stream_ptr=7)
    with pytest.raises(GraphContractError, match="stream"):
        plan.replay(key(), stream_ptr=8)


def test_nested_capture_and_recapture_are_refused_until_invalidated():
    plan = KudaCudaGraphPlan(RecordingBridge())
    plan.begin_capture(key(), stream_ptr=7)
    with pytest.raises(GraphContractError, match="capturing"):
        plan.begin_capture(key(), stream_ptr=7)
    plan.end_capture(key(), stream_ptr=7)
    with pytest.raises(GraphContractError, match="captured"):
        plan.begin_capture(key(), stream_ptr=7)
    plan.invalidate()
    with pytest.raises(GraphContractError, match="captured"):
        plan.replay(key(), stream_ptr=7)


def test_failed_native_end_capture_leaves_nothing_captured():
    plan = KudaCudaGraphPlan(RecordingBridge(fail_end=True))
    plan.begin_capture(key(), stream_ptr=7)
    with pytest.raises(RuntimeError):
        plan.end_capture(key(), stream_ptr=7)
    assert not plan.capturing and not plan.captured


# ------------------------------------------------------------------ GraphStaticCache (CPU)
def _tiny_prefilled_cache(layers=2, prompt=5):
    import torch
    from transformers import DynamicCache, Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(hidden_size=256, intermediate_size=512, num_hidden_layers=layers, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=100, max_position_embeddings=64, tie_word_embeddings=True)
    torch.manual_seed(0)
    model = Qwen2ForCausalLM(cfg).eval()
    cache = DynamicCache(config=model.config)
    with torch.no_grad():
        model(input_ids=torch.arange(1, prompt + 1).view(1, -1), past_key_values=cache, use_cache=True)
    return cache


def test_graph_static_cache_from_dynamic_cache_copies_the_prefix():
    """python/kudacuda_static_decode.py:100-145: fixed-capacity tensors, prefix
    copied, rows past it zero, device cache_position = sequence length."""

    import torch

    from kudacuda_b200.kudacuda_static_decode import GraphStaticCache

    dyn = _tiny_prefilled_cache(layers=2, prompt=5)
    gc = GraphStaticCache.from_dynamic_cache(torch, dyn, max_cache_len=16)
    assert len(gc) == 2 and gc.max_cache_len == 16 and gc.get_seq_length() == 5
    assert gc.get_max_length() == gc.get_max_cache_shape() == 16
    assert int(gc.cache_position.item()) == 5 and gc.cache_position.dtype == torch.long
    for i, layer in enumerate(dyn.layers):
        k, v = gc.key_cache[i], gc.value_cache[i]
        assert tuple(k.shape) == (1, 2, 16, 64)
        assert torch.equal(k[..., :5, :], layer.keys) and torch.equal(v[..., :5, :], layer.values)
        assert not k[..., 5:, :].any() and not v[..., 5:, :].any()
    # update writes the step's rows at cache_position and returns the full layer
    ks = torch.ones((1, 2, 1, 64))
    k_all, _ = gc.update(ks, ks * 2, 1)
    assert torch.equal(k_all[..., 5, :], ks[..., 0, :]) and k_all.shape[2] == 16


def test_graph_static_cache_rejects_a_short_capacity():
    import torch

    from kudacuda_b200.kudacuda_static_decode import GraphStaticCache

    dyn = _tiny_prefilled_cache(layers=1, prompt=9)
    with pytest.raises(GraphContractError):
        GraphStaticCache.from_dynamic_cache(torch, dyn, max_cache_len=8)


def test_runner_signatures_match_the_reference():
    """capture / replay keyword names of python/kudacuda_static_decode.py:271-287, 388-395."""

    import inspect

    from kudacuda_b200.kudacuda_static_decode import StaticDecodeGraphRunner

    cap = inspect.signature(StaticDecodeGraphRunner.capture).parameters
    for name in ("input_ids", "position_ids", "attention_mask", "cache_position", "past_key_values",
                 "logical_kv_len", "kv_bucket", "tactic_name", "stream_ptr", "stream", "device_id", "model_kwargs",
                 "workspace"):
        assert name in cap and cap[name].kind == inspect.Parameter.KEYWORD_ONLY, name
    rep = inspect.signature(StaticDecodeGraphRunner.replay).parameters
    for name in ("next_token", "position_ids", "cache_position", "logical_kv_len", "stream_ptr"):
        assert name in rep and rep[name].kind == inspect.Parameter.KEYWORD_ONLY, name
    runner = StaticDecodeGraphRunner(bridge=None, model=None, torch_module=object())
    assert not runner.captured and runner.status == "not-requested"
