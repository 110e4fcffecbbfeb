"""GPU test of the chat loop (kudacuda_b200.chat.ChatSession): batched prefill
into the persistent decode plan's cache, then greedy decode steps, on a
2-layer model with the config-1 layer shapes (random weights).

* the same prompt twice gives the same tokens (the second turn's prefill
  overwrites every cache row the first turn's decode wrote);
* a text turn through a stand-in tokenizer (chat template = word hashes)
  joins the history, and the next turn's prompt is longer;
* a turn that would overrun the KV bucket is refused before it starts;
* the device error word stays clear.
"""

import pytest

pytestmark = pytest.mark.gpu


class _WordTokenizer:
    """Stand-in tokenizer: one id per word of the rendered conversation."""

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=True):
        text = " ".join(f"<{m['role']}> {m['content']}" for m in messages) + (" <assistant>" if add_generation_prompt else "")
        return [1 + (sum(map(ord, w)) * 7919) % 4000 for w in text.split()]

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(f"t{i}" for i in ids)


def test_chat_session_turns():
    import torch

    from kudacuda_b200.chat import ChatSession
    from kudacuda_b200.decode_engine import random_weights, tiny_config
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    torch.cuda.set_device(0)
    cfg = tiny_config(layers=2, vocab=4096)
    bridge = KudaCudaBridge(device_id=0)
    w = random_weights(bridge, cfg, seed=3, device="cuda:0")
    sess = ChatSession(bridge, w, tokenizer=_WordTokenizer(), kv_bucket=256, device="cuda:0", eos_ids=[4095])
    try:
        prompt = [(i * 37 + 11) % 4000 for i in range(70)]
        a, sa = sess.generate_ids(prompt, 12)
        b, sb = sess.generate_ids(prompt, 12)
        assert a == b and all(0 <= t < cfg.vocab for t in a)
        assert sa["device_error_word"] == 0 and sb["device_error_word"] == 0 and sa["prompt_tokens"] == 70
        text, s1 = sess.turn("hello there", 8)
        assert len(sess.history) == 2 and sess.history[1]["content"] == text
        _, s2 = sess.turn("and again", 8)
        assert s2["prompt_tokens"] > s1["prompt_tokens"] and s2["device_error_word"] == 0
        with pytest.raises(ValueError):
            sess.generate_ids(prompt, 256 - 70 + 1)
    finally:
        sess.close()
        bridge.shutdown()
