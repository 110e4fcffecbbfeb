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
