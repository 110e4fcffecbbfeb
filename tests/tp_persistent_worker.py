"""Worker of tests/test_gpu_tp_persistent.py (one process per GPU, launched by
torch.distributed.run): the tensor-parallel row-split persistent kernel
(o_proj / down partials exchanged inside the kernel over peer memory) against
the tensor-parallel per-op path (NCCL allreduce) on the same shards of a
2-layer Llama-3-8B-architecture model, and against the unsharded model on one
GPU.  Rank 0 writes the measurements as JSON to argv[1]."""

from __future__ import annotations

import json
import os
import sys
from dataclasses import replace
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main() -> int:
    import datetime

    import torch
    import torch.distributed as dist

    from kudacuda_b200.decode_engine import LLAMA3_8B, StaticDecodePlan, random_weights
    from kudacuda_b200.kudacuda_sidecar import KudaCudaBridge

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = f"cuda:{local}"
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    group = dist.group.WORLD
    cfg = replace(LLAMA3_8B, name="llama-3-8b-2l", layers=2, vocab=4096)
    bridge = KudaCudaBridge(device_id=local)
    w = random_weights(bridge, cfg, seed=7, device=dev, shard=(rank, world))
    stream = torch.cuda.Stream(device=dev)
    tp = StaticDecodePlan(bridge, w, kv_bucket=64, max_tokens=64, device=dev, allreduce=(rank, world, group),
                          persistent=True)
    tp.capture(stream)
    ref = StaticDecodePlan(bridge, w, kv_bucket=64, max_tokens=64, device=dev, allreduce=(rank, world, group))
    ref.capture(stream)

    # one step from the same state: the final hidden state of both paths
    xs = []
    for plan in (tp, ref):
        plan.reset_cache()
        plan.set_state(77, 0, stream)
        plan.replay(stream)
        stream.synchronize()
        xs.append(plan.buffers.x.float().clone())
    rel = float((xs[0] - xs[1]).norm() / xs[1].norm())

    # teacher-forced greedy: both paths predict from the per-op path's tokens
    seq = [5, 17, 300, 4000]
    tp.reset_cache()
    ref.reset_cache()
    preds_tp, preds_ref = [], []
    for pos in range(16):
        tok = seq[pos]
        a = tp.step_host(tok, pos, stream)
        b = ref.step_host(tok, pos, stream)
        preds_tp.append(a)
        preds_ref.append(b)
        if pos + 1 >= len(seq):
            seq.append(b)
    err = bridge.error_word(clear=True)
    mine = torch.tensor(preds_tp, dtype=torch.int32, device=dev)
    gathered = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine, group=group)
    ranks_agree = all(torch.equal(g, gathered[0]) for g in gathered)
    x_tp = xs[0]
    # timing of the two paths (device, max over ranks)
    def time_steps(plan, n=32):
        plan.reset_cache()
        plan.set_state(5, 0, stream)
        for _ in range(3):
            plan.replay(stream)
        stream.synchronize()
        dist.barrier(group=group)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(n):
            plan.replay(stream)
        e.record(stream)
        e.synchronize()
        t = torch.tensor([s.elapsed_time(e) / n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        return float(t.item())

    ms_tp, ms_ref = time_steps(tp), time_steps(ref)
    tp.graph_plan.invalidate()
    ref.graph_plan.invalidate()
    for plan in (tp, ref):
        if plan._torch_graph is not None:
            plan._torch_graph.reset()
    tp.tp_exchange.close()

    # the unsharded model on rank 0's GPU: one step from the same state
    rel_full = None
    if rank == 0:
        bridge1 = KudaCudaBridge(device_id=local)
        w1 = random_weights(bridge1, cfg, seed=7, device=dev)
        one = StaticDecodePlan(bridge1, w1, kv_bucket=64, max_tokens=64, device=dev, allreduce=(0, 1, None),
                               persistent=True)
        one.capture(stream)
        one.reset_cache()
        one.set_state(77, 0, stream)
        one.replay(stream)
        stream.synchronize()
        x1 = one.buffers.x.float()
        rel_full = float((x_tp - x1).norm() / x1.norm())
        err |= bridge1.error_word(clear=True)
        bridge1.reset_graph()
        bridge1.shutdown()
    dist.barrier(group=group)
    if rank == 0:
        agree = sum(int(a == b) for a, b in zip(preds_tp, preds_ref)) / len(preds_ref)
        Path(sys.argv[1]).write_text(json.dumps(dict(
            world=world, rel_x_tp_vs_per_op=rel, rel_x_tp_vs_one_gpu=rel_full, teacher_forced_agreement=agree,
            ranks_agree=ranks_agree, device_error_word=int(err), ms_per_step_tp_persistent=ms_tp,
            ms_per_step_tp_per_op=ms_ref, preds_tp=preds_tp, preds_ref=preds_ref)))
    dist.barrier(group=group)
    dist.destroy_process_group()
    bridge.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
