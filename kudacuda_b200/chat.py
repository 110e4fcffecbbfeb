"""Chat over the B200 decode plan: the user-facing path of the same kernels
(the counterpart of the reference's tools/chat_qwen2_kudacuda.py).

Each turn renders the conversation with the tokenizer's chat template,
prefills it through the batched tensor-core path into the decode plan's KV
cache (default bucket 2048 tokens), then decodes greedily one token per graph
replay of the persistent all-layers step, until an end-of-sequence token or
``--max-new-tokens``.  Every turn reports its prompt length, time to the first
token, decode throughput and the device error word.  Unlike the reference
tool, nothing falls back to Transformers: a conversation that would overrun
the KV bucket is refused before the turn starts (``kv_preflight``).

    python -m kudacuda_b200.chat --model /path/to/Qwen2.5-3B-Instruct          # interactive
    python -m kudacuda_b200.chat --model /path/to/model --prompt "Hello" --json  # one turn
    python -m kudacuda_b200.chat --random --prompt-ids 1,2,3 --max-new-tokens 32 --json
      (the Qwen2.5-3B architecture with random-init weights, token ids in and out)
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from typing import Any, Mapping, Optional, Sequence

DEFAULT_SYSTEM_PROMPT = "You are a helpful assistant."


def build_messages(history: Sequence[Mapping[str, str]], user_text: str, *,
                   system_prompt: str = DEFAULT_SYSTEM_PROMPT) -> list[dict[str, str]]:
    """System prompt, the earlier turns, then the new user message (history is not modified)."""

    messages = [{"role": "system", "content": system_prompt}]
    messages.extend({"role": str(m["role"]), "content": str(m["content"])} for m in history)
    messages.append({"role": "user", "content": user_text})
    return messages


def kv_preflight(*, prompt_tokens: int, requested_tokens: int, kv_bucket: int) -> dict[str, Any]:
    """Whether a turn fits the KV bucket: the prompt plus every generated token
    (the last one is never fed back) must fit."""

    prompt_tokens, requested_tokens = max(0, int(prompt_tokens)), max(0, int(requested_tokens))
    budget = max(0, int(kv_bucket) - prompt_tokens)
    return {"prompt_tokens": prompt_tokens, "requested_tokens": requested_tokens, "kv_bucket": int(kv_bucket),
            "budget": budget, "fits": prompt_tokens >= 1 and prompt_tokens + requested_tokens <= int(kv_bucket)}


def summarize_turn(*, prompt_tokens: int, generated: Sequence[int], prefill_s: float, decode_s: float,
                   error_word: int) -> dict[str, Any]:
    """Waiting time and throughput of one response."""

    n = len(generated)
    return {
        "prompt_tokens": int(prompt_tokens),
        "generated_tokens": n,
        "ttft_ms": round(prefill_s * 1e3, 3),
        "decode_ms": round(decode_s * 1e3, 3),
        "waiting_ms": round((prefill_s + decode_s) * 1e3, 3),
        "decode_tokens_per_second": round((n - 1) / decode_s, 2) if n > 1 and decode_s > 0 else 0.0,
        "device_error_word": int(error_word),
    }


class ChatSession:
    """One model on one device: the persistent decode plan (KV bucket
    ``kv_bucket``), its batched prefill, and the conversation so far."""

    def __init__(self, bridge: Any, weights: Any, *, tokenizer: Any = None, kv_bucket: int = 2048,
                 device: Any = "cuda:0", system_prompt: str = DEFAULT_SYSTEM_PROMPT,
                 eos_ids: Sequence[int] = (), torch_module: Any = None) -> None:
        if torch_module is None:
            import torch as torch_module
        from .decode_engine import BatchedPrefill, StaticDecodePlan

        self.torch = torch_module
        self.bridge = bridge
        self.tokenizer = tokenizer
        self.system_prompt = system_prompt
        self.eos_ids = {int(e) for e in eos_ids}
        self.history: list[dict[str, str]] = []
        self.plan = StaticDecodePlan(bridge, weights, kv_bucket=int(kv_bucket), max_tokens=int(kv_bucket),
                                     device=device, torch_module=torch_module, persistent=True)
        # the prefill's chunk step is captured before the cache holds anything
        self.prefill = BatchedPrefill(self.plan, chunk=64)
        self.stream = torch_module.cuda.Stream(device=device)
        self.plan.capture(self.stream)

    @property
    def kv_bucket(self) -> int:
        return self.plan.kv_bucket

    def generate_ids(self, prompt_ids: Sequence[int], max_new_tokens: int) -> tuple[list[int], dict[str, Any]]:
        """Greedy continuation of ``prompt_ids``: the prompt through the batched
        prefill, then one persistent decode step per token."""

        pre = kv_preflight(prompt_tokens=len(prompt_ids), requested_tokens=max_new_tokens, kv_bucket=self.kv_bucket)
        if not pre["fits"]:
            raise ValueError(f"turn does not fit the KV bucket: {pre}")
        # the batched prefill pads the prompt to whole 64-token chunks
        if -(-len(prompt_ids) // self.prefill.chunk) * self.prefill.chunk > self.kv_bucket:
            raise ValueError("prompt padded to whole prefill chunks does not fit the KV bucket")
        torch = self.torch
        torch.cuda.synchronize(self.plan.device)
        t0 = time.perf_counter()
        tok = int(self.prefill.prefill([int(t) for t in prompt_ids], self.stream))
        t1 = time.perf_counter()
        out = [tok]
        pos = len(prompt_ids)
        while len(out) < int(max_new_tokens) and out[-1] not in self.eos_ids:
            out.append(int(self.plan.step_host(out[-1], pos, self.stream)))
            pos += 1
        t2 = time.perf_counter()
        stats = summarize_turn(prompt_tokens=len(prompt_ids), generated=out, prefill_s=t1 - t0, decode_s=t2 - t1,
                               error_word=self.bridge.error_word(clear=True))
        return out, stats

    def turn(self, user_text: str, max_new_tokens: int) -> tuple[str, dict[str, Any]]:
        """One chat turn; the reply joins the history."""

        if self.tokenizer is None:
            raise ValueError("a text turn needs a tokenizer (use generate_ids with token ids)")
        messages = build_messages(self.history, user_text, system_prompt=self.system_prompt)
        ids = self.tokenizer.apply_chat_template(messages, add_generation_prompt=True, tokenize=True)
        if isinstance(ids, Mapping):  # newer tokenizers return a BatchEncoding
            ids = ids["input_ids"]
        ids = list(ids[0]) if ids and isinstance(ids[0], (list, tuple)) else list(ids)
        out, stats = self.generate_ids(ids, max_new_tokens)
        reply_ids = [t for t in out if t not in self.eos_ids]
        text = self.tokenizer.decode(reply_ids, skip_special_tokens=True)
        self.history.append({"role": "user", "content": user_text})
        self.history.append({"role": "assistant", "content": text})
        return text, stats

    def close(self) -> None:
        self.prefill.plan.release()
        self.prefill.bridge.shutdown()
        self.bridge.reset_graph()


def _load(args: argparse.Namespace) -> tuple[Any, Any, Any, list[int]]:
    import torch

    from .decode_engine import QWEN25_3B, random_weights
    from .kudacuda_sidecar import KudaCudaBridge

    bridge = KudaCudaBridge(device_id=torch.device(args.device).index or 0)
    if args.random:
        return bridge, random_weights(bridge, QWEN25_3B, seed=args.seed, device=args.device), None, []
    from transformers import AutoModelForCausalLM, AutoTokenizer

    from .kudacuda_static_decode import weights_from_transformers

    tok = AutoTokenizer.from_pretrained(args.model)
    model = AutoModelForCausalLM.from_pretrained(args.model, dtype=torch.bfloat16).to(args.device).eval()
    weights = weights_from_transformers(bridge, model, device=args.device, torch_module=torch)
    eos = model.generation_config.eos_token_id if model.generation_config is not None else tok.eos_token_id
    eos_ids = [eos] if isinstance(eos, int) else list(eos or [])
    del model
    torch.cuda.empty_cache()
    return bridge, weights, tok, eos_ids


def main(argv: Optional[Sequence[str]] = None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    src = p.add_mutually_exclusive_group(required=True)
    src.add_argument("--model", help="Transformers model directory (Qwen2/Llama; dense or bitsandbytes NF4)")
    src.add_argument("--random", action="store_true", help="Qwen2.5-3B architecture, random-init weights")
    p.add_argument("--prompt", help="one user turn (text), then exit")
    p.add_argument("--prompt-ids", help="one turn of comma-separated token ids, then exit")
    p.add_argument("--max-new-tokens", type=int, default=128)
    p.add_argument("--kv-bucket", type=int, default=2048)
    p.add_argument("--system-prompt", default=DEFAULT_SYSTEM_PROMPT)
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--seed", type=int, default=20260824)
    p.add_argument("--json", action="store_true", help="print one JSON line per turn")
    args = p.parse_args(argv)
    import torch

    torch.cuda.set_device(torch.device(args.device))
    bridge, weights, tok, eos_ids = _load(args)
    session = ChatSession(bridge, weights, tokenizer=tok, kv_bucket=args.kv_bucket, device=args.device,
                          system_prompt=args.system_prompt, eos_ids=eos_ids)
    try:
        if args.prompt_ids is not None:
            ids = [int(v) for v in args.prompt_ids.split(",") if v.strip()]
            out, stats = session.generate_ids(ids, args.max_new_tokens)
            print(json.dumps({"tokens": out, **stats}) if args.json else f"{out}\n{stats}", flush=True)
            return 0 if stats["device_error_word"] == 0 else 1
        if args.prompt is not None:
            text, stats = session.turn(args.prompt, args.max_new_tokens)
            print(json.dumps({"reply": text, **stats}) if args.json else f"{text}\n{stats}", flush=True)
            return 0 if stats["device_error_word"] == 0 else 1
        while True:  # interactive
            try:
                user = input("you> ").strip()
            except EOFError:
                return 0
            if user in ("", "/exit", "/quit"):
                return 0
            text, stats = session.turn(user, args.max_new_tokens)
            print(f"assistant> {text}\n  [{stats['prompt_tokens']} prompt tokens, ttft {stats['ttft_ms']:.1f} ms, "
                  f"{stats['decode_tokens_per_second']:.1f} tok/s, {stats['generated_tokens']} tokens]", flush=True)
    finally:
        session.close()


if __name__ == "__main__":
    sys.exit(main())
