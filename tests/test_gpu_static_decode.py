"""GPU test of the Transformers-model runner (kudacuda_static_decode): a
2-layer Qwen2 model with the config-1 layer shapes is converted to NF4 and
decoded through one captured graph per token; greedy top-1 agreement is
measured teacher-forced against Transformers' eager bf16 forward on the same
dequantised NF4 weights -- the restatement of the reference's eager NF4 path
(Transformers + bitsandbytes Linear4bit, which computes with weights
dequantised to bf16; bitsandbytes itself is absent here).  Both sides see the
same token history at every position, so a disagreement is a per-step
numerical near-tie, not compounding drift."""

import pytest

pytestmark = pytest.mark.gpu

PROMPT_LEN, NEW_TOKENS = 16, 128
# A random-init model has many near-tied logits: Transformers' own bf16 eager
# forward agrees with its fp32 eager forward on only ~97.7% of positions here,
# so the bar is relative to that floor (at most 4 of 128 more disagreements)
# plus an absolute minimum.
AGREEMENT = 0.94
FLOOR_MARGIN = 4 / 128


def _tiny_qwen2(torch):
    from transformers import Qwen2Config, Qwen2ForCausalLM

    cfg = Qwen2Config(hidden_size=2048, intermediate_size=11008, num_hidden_layers=2, num_attention_heads=16,
                      num_key_value_heads=2, vocab_size=4096, max_position_embeddings=1024, rope_theta=1.0e6,
                      rms_norm_eps=1.0e-6, tie_word_embeddings=True)
    torch.manual_seed(20260824)
    model = Qwen2ForCausalLM(cfg)
    return model.to(device="cuda:0", dtype=torch.bfloat16).eval()


def test_runner_matches_transformers_eager_on_the_same_nf4_weights():
    import copy

    import torch

    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge
    from kudacuda_b200.kudacuda_static_decode import StaticDecodeGraphRunner

    model = _tiny_qwen2(torch)
    bridge = KudaCudaBridge(device_id=0)
    runner = StaticDecodeGraphRunner(bridge, model, torch)
    runner.capture(kv_bucket=256)
    assert runner.captured

    # eager models computing with the runner's NF4 weights: fp32 with the exact
    # dequantised values, and bf16 with them rounded to bf16 (the reference's
    # eager NF4 path: bitsandbytes dequantises to the compute dtype)
    w = runner._weights
    sp = int(torch.cuda.current_stream().cuda_stream)

    def deq(lin, dtype):
        out = torch.empty((lin.rows, lin.k), dtype=dtype, device="cuda:0")
        bridge.dispatch_nf4_dequantize(lin.packed, lin.absmax, out, n=lin.rows * lin.k, stream_ptr=sp)
        return out

    m32 = copy.deepcopy(model).float()
    with torch.no_grad():
        for mdl, dt in ((model, torch.bfloat16), (m32, torch.float32)):
            for layer, L in zip(mdl.model.layers, w.layers):
                a, m = layer.self_attn, layer.mlp
                for mod, lin in ((a.q_proj, L.q), (a.k_proj, L.k), (a.v_proj, L.v), (a.o_proj, L.o),
                                 (m.gate_proj, L.gate), (m.up_proj, L.up), (m.down_proj, L.down)):
                    mod.weight.copy_(deq(lin, dt))
            mdl.config._attn_implementation = "eager"
    torch.cuda.synchronize()

    g = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, 4096, (PROMPT_LEN,), generator=g).tolist()
    with torch.no_grad():
        ids = torch.tensor([prompt], device="cuda:0")
        seq = m32.generate(ids, max_new_tokens=NEW_TOKENS, do_sample=False, min_new_tokens=NEW_TOKENS,
                           pad_token_id=0, eos_token_id=None)[0].tolist()
        full = torch.tensor([seq[:-1]], device="cuda:0")
        p32 = m32(full).logits[0].float().argmax(-1).tolist()[PROMPT_LEN - 1:]
        p16 = model(full).logits[0].float().argmax(-1).tolist()[PROMPT_LEN - 1:]
    # teacher-forced: our next-token prediction at every generated position
    runner.plan.reset_cache()
    ours = []
    for pos in range(len(seq) - 1):
        nxt = runner.replay(seq[pos], pos)
        if pos >= PROMPT_LEN - 1:
            ours.append(nxt)

    def agree(a, b):
        return sum(int(x == y) for x, y in zip(a, b)) / len(a)

    a32, a16, ref_noise = agree(ours, p32), agree(ours, p16), agree(p16, p32)
    print(f"teacher-forced top-1 agreement over {len(ours)} tokens: ours vs fp32-eager {a32:.4f}, "
          f"ours vs bf16-eager {a16:.4f}, bf16-eager vs fp32-eager {ref_noise:.4f}")
    assert bridge.error_word(clear=True) == 0
    msg = f"ours/fp32 {a32:.4f} ours/bf16 {a16:.4f} bf16/fp32 {ref_noise:.4f}"
    assert a32 >= AGREEMENT and a16 >= AGREEMENT, msg
    assert a32 >= ref_noise - FLOOR_MARGIN, msg
    # free-running greedy generation through the runner also starts with the same token
    gen = runner.generate(prompt, 8)
    assert gen[0] == seq[PROMPT_LEN] or gen[0] == p16[0]

    # the batched tensor-core path on the same weights (one sequence): its
    # arithmetic is the bf16 eager path's (weights dequantised to bf16, bf16
    # matmul with fp32 accumulation), so it tracks the bf16 forward closely
    from kudacuda_b200.decode_engine import BatchedDecodePlan

    bbridge = KudaCudaBridge(device_id=0)
    bplan = BatchedDecodePlan(bbridge, w, batch=1, kv_bucket=256, max_tokens=256, device="cuda:0")
    bstream = torch.cuda.Stream()
    bplan.capture(bstream)
    bplan.reset_cache()
    batched = []
    for pos in range(len(seq) - 1):
        nxt = bplan.step_tokens([seq[pos]], [pos], bstream)[0]
        if pos >= PROMPT_LEN - 1:
            batched.append(nxt)
    b32, b16 = agree(batched, p32), agree(batched, p16)
    print(f"batched path: vs fp32-eager {b32:.4f}, vs bf16-eager {b16:.4f}")
    assert bbridge.error_word(clear=True) == 0
    bmsg = f"batched/fp32 {b32:.4f} batched/bf16 {b16:.4f} bf16/fp32 {ref_noise:.4f}"
    assert b32 >= AGREEMENT and b16 >= AGREEMENT, bmsg
    assert b32 >= ref_noise - FLOOR_MARGIN, bmsg
    bplan.release()
    bbridge.reset_graph()
    bbridge.shutdown()
    runner.invalidate("test done")
    assert not runner.captured
