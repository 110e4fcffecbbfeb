"""CPU tests of the chat loop's host logic (kudacuda_b200.chat): message
building as the reference's tools/chat_qwen2_kudacuda.py builds them, the KV
preflight and the per-turn summary."""

from kudacuda_b200.chat import DEFAULT_SYSTEM_PROMPT, build_messages, kv_preflight, summarize_turn


def test_build_messages_keeps_history_untouched():
    history = [{"role": "user", "content": "hi"}, {"role": "assistant", "content": "hello"}]
    msgs = build_messages(history, "next")
    assert msgs[0] == {"role": "system", "content": DEFAULT_SYSTEM_PROMPT}
    assert msgs[1:3] == history and msgs[3] == {"role": "user", "content": "next"}
    assert len(history) == 2


def test_kv_preflight_counts_prompt_and_generated_tokens():
    assert kv_preflight(prompt_tokens=100, requested_tokens=28, kv_bucket=128)["fits"]
    r = kv_preflight(prompt_tokens=100, requested_tokens=29, kv_bucket=128)
    assert not r["fits"] and r["budget"] == 28
    assert not kv_preflight(prompt_tokens=0, requested_tokens=1, kv_bucket=128)["fits"]


def test_summarize_turn_throughput():
    s = summarize_turn(prompt_tokens=10, generated=[1, 2, 3, 4, 5], prefill_s=0.01, decode_s=0.004, error_word=0)
    assert s["generated_tokens"] == 5 and s["decode_tokens_per_second"] == 1000.0
    assert s["ttft_ms"] == 10.0 and s["waiting_ms"] == 14.0
