"""Worker of tests/test_gpu_tp_persistent.py's failure test (one process per
GPU, launched by torch.distributed.run): a rank that misses one step of the
tensor-parallel persistent kernel.  Rank 0 launches the kernel alone (outside
the step graph, so no collective library call can wait on the absent rank);
its waits for rank 1's partials run out, the launch returns with error bit 4
set and nothing hangs.  Then the ranks agree on a fresh launch epoch over the
host process group and a normal step runs on both, identical and error-free.
Rank 1 stays alive throughout (its exchange buffer stays mapped).  Rank 0
writes the result as JSON to argv[1]."""

from __future__ import annotations

import json
import os
import sys
import time
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
    plan = StaticDecodePlan(bridge, w, kv_bucket=64, max_tokens=64, device=dev, allreduce=(rank, world, group),
                            persistent=True)
    plan.capture(stream)

    def step(tok, pos):
        return plan.step_host(tok, pos, stream)

    before = [step(11, 0), step(12, 1)]
    err0 = bridge.error_word(clear=True)

    # rank 0 alone: the persistent kernel waits for rank 1's partials, which never come
    seconds = None
    err_missed = 0
    dist.barrier(group=group)
    if rank == 0:
        plan.set_state(13, 2, stream)
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            plan.persistent.record(int(stream.cuda_stream))
        stream.synchronize()
        seconds = time.perf_counter() - t0
        err_missed = bridge.error_word(clear=True)
    dist.barrier(group=group)

    # recovery: one fresh epoch on every rank, then a normal step from a known state
    e = torch.tensor([plan.persistent.epoch()], dtype=torch.int64, device=dev)
    dist.all_reduce(e, op=dist.ReduceOp.MAX, group=group)
    plan.persistent.set_epoch(int(e.item()) + 1)
    plan.reset_cache()
    after = [step(11, 0), step(12, 1)]
    err_after = bridge.error_word(clear=True)
    mine = torch.tensor(after, dtype=torch.int32, device=dev)
    got = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(got, mine, group=group)
    ranks_agree = all(torch.equal(g, got[0]) for g in got)

    plan.graph_plan.invalidate()
    if plan._torch_graph is not None:
        plan._torch_graph.reset()
    plan.tp_exchange.close()
    dist.barrier(group=group)
    if rank == 0:
        Path(sys.argv[1]).write_text(json.dumps(dict(
            err_before=err0, err_missed_step=err_missed, missed_step_seconds=seconds, err_after=err_after,
            tokens_before=before, tokens_after=after, ranks_agree_after=ranks_agree)))
    dist.barrier(group=group)
    dist.destroy_process_group()
    bridge.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
