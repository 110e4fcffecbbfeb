"""Per-op microbenchmark of the sm_100a kernels (device time per launch).

Each op is launched ``--launches`` times inside one CUDA graph, cycling over
``--copies`` independent weight sets so the bytes read per graph replay exceed
the 126 MB L2 (every launch streams from HBM); the graph is replayed
``--reps`` times between two CUDA events on its stream.  Algorithmic bytes are
those the op must read/write once (NF4 packed + absmax + activations, or the
KV rows for attention).

    python -m kudacuda_b200.microbench --op swiglu [--copies 12 --launches 36 --reps 20]
    ops: gemv_11008x2048 gemv_2048x11008 qkv_rope oproj down swiglu gqa512 gqa2048 lm_head all
         bgemm_<rows>x<k>_n<n_pad>[_ks<ksplit>][_bf16|_rt]  (batched tensor-core GEMM; _rt: re-tiled NF4)

    python -m kudacuda_b200.microbench --op persistent --layers 36 --kv 512 [--launches 3 --reps 20]
      the persistent all-layers kernel alone (Qwen2.5-3B layer shapes, random
      NF4 weights), launched directly on its stream at position kv - 1

    python -m kudacuda_b200.microbench --op refcompare [--launches 36 --reps 20]
      the reference's own kernels (oracle/_ref, built for sm_100a from its
      sources) against this library's through the same reference ABI entries

    python -m kudacuda_b200.microbench --op prefill --prompt 512
      time to first token: batched prefill (64-token chunks on the tensor
      cores) against the decode-loop prefill, full Qwen2.5-3B architecture

The same command with ``--reps 1 --launches 4`` is the small case used for ncu
captures (see profiles/).
"""

from __future__ import annotations

import argparse
import json
import math
import sys
from typing import Any, Callable

from .kudacuda_sidecar import KudaCudaBridge


def _peak() -> float:
    import json as _j
    from pathlib import Path

    p = Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    return float(_j.loads(p.read_text())["hbm_gbs"]) if p.exists() else 6650.0


class OpCase:
    def __init__(self, name: str, nbytes: int, launch: Callable[[int, int], None]) -> None:
        self.name = name
        self.nbytes = nbytes
        self.launch = launch  # launch(copy_index, stream_ptr)


def _nf4(torch, rows: int, k: int, copies: int, device: str) -> list[tuple[Any, Any]]:
    out = []
    for _ in range(copies):
        packed = torch.randint(0, 256, (rows * k // 2, 1), dtype=torch.uint8, device=device)
        absmax = torch.rand(rows * k // 64, device=device) * 0.05 + 0.01
        out.append((packed, absmax))
    return out


def build_cases(torch, bridge: KudaCudaBridge, names: list[str], copies: int, device: str) -> list[OpCase]:
    bf16 = torch.bfloat16
    cases = []
    H, I, V = 2048, 11008, 151936

    def vec(n, scale=1.0):
        return (torch.randn(n, device=device) * scale).to(bf16)

    for name in names:
        if name.startswith("gemv_"):
            rows, k = (int(v) for v in name[5:].split("x"))
            W = _nf4(torch, rows, k, copies, device)
            x, y = vec(k), torch.empty(rows, dtype=bf16, device=device)
            nb = rows * k // 2 + rows * k // 16 + 2 * k + 2 * rows

            def f(i, sp, W=W, x=x, y=y, rows=rows, k=k):
                p, a = W[i % len(W)]
                bridge.dispatch_nf4_gemv(x, p, a, y, rows=rows, k=k, stream_ptr=sp)

            cases.append(OpCase(name, nb, f))
        elif name in ("oproj", "down"):
            rows, k = (H, H) if name == "oproj" else (H, I)
            W = _nf4(torch, rows, k, copies, device)
            x, r = vec(k), vec(rows)
            nb = rows * k // 2 + rows * k // 16 + 2 * k + 4 * rows

            def f(i, sp, W=W, x=x, r=r, rows=rows, k=k):
                p, a = W[i % len(W)]
                bridge.dispatch_nf4_linear_residual(x, p, a, r, rows=rows, k=k, stream_ptr=sp)

            cases.append(OpCase(name, nb, f))
        elif name == "swiglu":
            G = _nf4(torch, I, H, copies, device)
            U = _nf4(torch, I, H, copies, device)
            x, nw, h = vec(H), (1 + vec(H, 0.02).float()).to(bf16), torch.empty(I, dtype=bf16, device=device)
            nb = 2 * (I * H // 2 + I * H // 16) + 4 * H + 2 * I

            def f(i, sp, G=G, U=U, x=x, nw=nw, h=h):
                bridge.dispatch_swiglu_bf16(x, nw, G[i % len(G)], U[i % len(U)], h, epsilon=1e-6, stream_ptr=sp)

            cases.append(OpCase(name, nb, f))
        elif name == "qkv_rope":
            from .decode_engine import rope_tables

            Q = _nf4(torch, 2048, H, copies, device)
            K = _nf4(torch, 256, H, copies, device)
            Vv = _nf4(torch, 256, H, copies, device)
            x, nw = vec(H), (1 + vec(H, 0.02).float()).to(bf16)
            qb, kb, vb = vec(2048, 0.02), vec(256, 0.02), vec(256, 0.02)
            cos, sin = rope_tables(torch, 1024, 128, 1e6, device)
            pos = torch.tensor([100], dtype=torch.int32, device=device)
            qo = torch.empty(2048, dtype=bf16, device=device)
            kc = torch.zeros((2, 512, 128), dtype=bf16, device=device)
            vc = torch.zeros((2, 512, 128), dtype=bf16, device=device)
            nb = 2560 * H // 2 + 2560 * H // 16 + 4 * H + 2 * 2560 * 2

            def f(i, sp, Q=Q, K=K, Vv=Vv):
                j = i % len(Q)
                bridge.dispatch_attention_input(x, nw, (*Q[j], qb), (*K[j], kb), (*Vv[j], vb), cos, sin, pos, qo, kc, vc,
                                                q_heads=16, kv_heads=2, head_dim=128, kv_capacity=512, epsilon=1e-6,
                                                stream_ptr=sp)

            cases.append(OpCase(name, nb, f))
        elif name.startswith("gqa"):
            L = int(name[3:])
            KC = [torch.randn((2, L, 128), device=device).to(bf16) for _ in range(copies)]
            VC = [torch.randn((2, L, 128), device=device).to(bf16) for _ in range(copies)]
            q, out = vec(16 * 128), torch.empty(16 * 128, dtype=bf16, device=device)
            kvl = torch.tensor([L], dtype=torch.int32, device=device)
            ws, tk, nbytes = bridge.gqa_workspace(batch=1, query_heads=16, kv_heads=2, kv_extent=L, device=device,
                                                  torch_module=torch)
            nb = 2 * 2 * L * 128 * 2 + 2 * 2 * 16 * 128

            def f(i, sp, KC=KC, VC=VC, L=L, q=q, out=out, kvl=kvl, ws=ws, tk=tk, nbytes=nbytes):
                j = i % len(KC)
                bridge.dispatch_gqa_decode_splitkv(q, KC[j], VC[j], out, ws, tk, kv_len_device=kvl, kv_len=L,
                                                   kv_stride=L, query_heads=16, kv_heads=2, stream_ptr=sp,
                                                   workspace_bytes=nbytes)

            cases.append(OpCase(name, nb, f))
        elif name.startswith("bgemm_"):
            # batched tensor-core GEMM: bgemm_<rows>x<k>_n<n_pad>[_ks<ksplit>][_bf16]
            parts = name.split("_")
            rows, k = (int(v) for v in parts[1].split("x"))
            npad = int(parts[2][1:])
            ks = next((int(p[2:]) for p in parts[3:] if p.startswith("ks")), 0) or bridge.batch_gemm_ksplit(rows, k)
            wt = 1 if "bf16" in parts[3:] else (2 if "rt" in parts[3:] else 0)
            if wt == 0:
                W = _nf4(torch, rows, k, copies, device)
            elif wt == 2:  # re-tiled streaming form
                W = []
                for p_, a_ in _nf4(torch, rows, k, copies, device):
                    rt = torch.empty(bridge.batch_retile_bytes(rows, k), dtype=torch.uint8, device=device)
                    bridge.dispatch_batch_retile(p_, a_, rt, rows=rows, k=k, stream_ptr=0)
                    W.append((rt, None))
                torch.cuda.synchronize()
            else:
                W = [(torch.randn((rows, k), device=device).to(bf16), None) for _ in range(copies)]
            xb = torch.randn((npad, k), device=device).to(bf16)
            part = torch.empty(ks * rows * npad, dtype=torch.float32, device=device)
            nb = (rows * k // 2 + rows * k // 16 if wt == 0 else rows * k * 2) + npad * k * 2 + npad * rows * 2

            def f(i, sp, W=W, xb=xb, part=part, rows=rows, k=k, npad=npad, ks=ks, wt=wt):
                p, a = W[i % len(W)]
                bridge.dispatch_batch_gemm(p, a, xb, part, weight_type=wt, rows=rows, k=k, n_pad=npad, ksplit=ks,
                                           stream_ptr=sp)

            cases.append(OpCase(f"{name}(ks{ks})", nb, f))
        elif name == "lm_head":
            n_emb = max(1, min(copies, 2))
            E = [torch.randn((V, H), device=device).to(bf16) for _ in range(n_emb)]
            x, fn = vec(H), (1 + vec(H, 0.02).float()).to(bf16)
            tok = torch.zeros(1, dtype=torch.int32, device=device)
            lg = torch.empty(V, dtype=bf16, device=device)
            ws = torch.zeros(bridge.lm_head_workspace_bytes() // 4, device=device)
            tk = torch.zeros(1, dtype=torch.int32, device=device)
            nb = V * H * 2 + 2 * V

            def f(i, sp, E=E):
                bridge.dispatch_lm_head_argmax(x, fn, E[i % len(E)], tok, ws, tk, logits=lg, epsilon=1e-6, stream_ptr=sp)

            cases.append(OpCase(name, nb, f))
        else:
            raise SystemExit(f"unknown op {name}")
    return cases


def time_case(torch, bridge: KudaCudaBridge, case: OpCase, launches: int, reps: int, stream) -> dict:
    sp = int(stream.cuda_stream)
    with torch.cuda.stream(stream):
        for i in range(launches):  # eager warm-up (lazy per-kernel set-up)
            case.launch(i, sp)
    stream.synchronize()
    bridge.begin_capture(stream_ptr=sp)
    for i in range(launches):
        case.launch(i, sp)
    bridge.end_capture(stream_ptr=sp)
    bridge.replay_graph(stream_ptr=sp)
    stream.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        bridge.replay_graph(stream_ptr=sp)
    e.record(stream)
    e.synchronize()
    us = s.elapsed_time(e) * 1e3 / (reps * launches)
    gbs = case.nbytes / (us * 1e-6) / 1e9
    bridge.reset_graph()
    return {"op": case.name, "us_per_launch": round(us, 3), "bytes": case.nbytes, "gbs": round(gbs, 1),
            "frac_of_measured_hbm": round(gbs / _peak(), 4)}


def time_persistent(torch, layers: int, kv: int, launches: int, reps: int, device: str) -> dict:
    from .decode_engine import StaticDecodePlan, random_weights, tiny_config

    cfg = tiny_config(layers=layers, vocab=4096)
    bridge = KudaCudaBridge(device_id=torch.device(device).index or 0)
    w = random_weights(bridge, cfg, seed=20260824, device=device)
    plan = StaticDecodePlan(bridge, w, kv_bucket=max(kv, 16), max_tokens=max(kv, 16), device=device, persistent=True)
    stream = torch.cuda.Stream()
    sp = int(stream.cuda_stream)
    plan.set_state(1, kv - 1, stream)
    with torch.cuda.stream(stream):
        for _ in range(launches):
            plan.persistent.record(sp)
    stream.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(reps):
            plan.persistent.record(sp)
    e.record(stream)
    e.synchronize()
    us = s.elapsed_time(e) * 1e3 / max(reps, 1)
    wb = cfg.weight_bytes_per_token()
    nbytes = (wb["nf4_absmax"] + wb["norms_bias"] - cfg.hidden * 2 + 2 * cfg.hidden * 2 +
              layers * 2 * plan.kv_heads * cfg.head_dim * 2 * kv)
    gbs = nbytes / (us * 1e-6) / 1e9
    err = bridge.error_word(clear=True)
    return {"op": f"persistent_{layers}l_kv{kv}", "us_per_launch": round(us, 3), "us_per_layer": round(us / layers, 3),
            "bytes": nbytes, "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / _peak(), 4),
            "device_error_word": err}


def time_prefill(torch, prompt_len: int, device: str) -> dict:
    """Time to first token for a ``prompt_len``-token prompt on the Qwen2.5-3B
    architecture (36 layers, full vocabulary): the batched prefill (chunks of 64
    tokens through the tensor-core path into the decode plan's cache) against
    the decode-loop prefill (one persistent-kernel step per prompt token).
    Host-synchronous end to end, wall clock, after one warm-up of each."""

    import time

    from .decode_engine import QWEN25_3B, BatchedPrefill, StaticDecodePlan, random_weights

    bridge = KudaCudaBridge(device_id=torch.device(device).index or 0)
    w = random_weights(bridge, QWEN25_3B, seed=20260824, device=device)
    cap = max(512, ((prompt_len + 64 + 63) // 64) * 64)
    plan = StaticDecodePlan(bridge, w, kv_bucket=cap, max_tokens=cap, device=device, persistent=True)
    pre = BatchedPrefill(plan, chunk=64)
    stream = torch.cuda.Stream()
    plan.capture(stream)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, QWEN25_3B.vocab, (prompt_len,), generator=g).tolist()
    out = {"op": f"prefill_qwen25_3b_T{prompt_len}"}
    for name, fn in (("batched", lambda: pre.prefill(prompt, stream)), ("decode_loop", lambda: plan.prefill(prompt, stream))):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        tok = fn()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        out[f"{name}_ms"] = round(dt * 1e3, 2)
        out[f"{name}_prompt_tok_s"] = round(prompt_len / dt, 1)
        out[f"{name}_first_token"] = int(tok)
    out["device_error_word"] = bridge.error_word(clear=True)
    pre.plan.release()
    pre.bridge.shutdown()
    bridge.reset_graph()
    return out


def time_refcompare(torch, device: str, launches: int, reps: int) -> list[dict]:
    """The reference's own kernels (oracle/_ref/libkudacuda_ref.so, compiled
    for sm_100a from its sources) against this library's, through the same
    reference ABI entries on the same inputs: fused RMSNorm + NF4 QKV (v1,
    v3), NF4 SwiGLU (f16, bf16), GQA decode (direct at kv 512 / 1024 / 2048,
    graph and workspace_v3 at capacity 512).  Each library's calls are
    captured ``launches`` times into one torch CUDA graph, cycling over enough
    input copies that a replay reads more than the 126 MB L2; device time per
    call from CUDA events around ``reps`` replays."""

    import ctypes
    from pathlib import Path

    from . import native

    ref_path = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libkudacuda_ref.so"
    if not ref_path.exists():
        raise FileNotFoundError(f"{ref_path} not built (make -C oracle ref REFERENCE=...)")
    libs = {"reference": native.configure(ctypes.CDLL(str(ref_path))), "b200": native.load_library()}
    handles = {}
    for name, lib in libs.items():
        h = lib.kudacuda_create(torch.device(device).index or 0)
        assert h and lib.kudacuda_freeze(h) == 0, lib.kudacuda_last_error(h)
        handles[name] = h
    f16 = torch.float16
    l2 = 160 << 20

    def copies_for(nbytes: int) -> int:
        return max(2, min(64, -(-l2 // max(nbytes, 1))))

    def nf4(rows, k, n):
        return [(torch.randint(0, 256, (rows * k // 2,), dtype=torch.uint8, device=device),
                 torch.rand(rows * k // 64, device=device) * 0.05 + 0.01) for _ in range(n)]

    cases = []
    # fused RMSNorm + NF4 QKV (hidden 2048, q 2048, k/v 256)
    qkv_bytes = (2560 * 2048) // 2 + (2560 * 2048) // 16 + 2 * 2048 * 2 + 2 * 2560 * 2
    nq = copies_for(qkv_bytes)
    Q, K, V = nf4(2048, 2048, nq), nf4(256, 2048, nq), nf4(256, 2048, nq)
    x = torch.randn(2048, device=device).to(f16)
    nw = (1 + 0.02 * torch.randn(2048, device=device)).to(f16)
    bq, bk, bv = (torch.randn(n, device=device).mul(0.02).to(f16) for n in (2048, 256, 256))
    qo, ko, vo = (torch.empty(n, dtype=f16, device=device) for n in (2048, 256, 256))
    ws_norm = torch.empty(2048, dtype=torch.float32, device=device)
    for variant in ("", "_v3"):
        def f(lib, h, i, sp, variant=variant):
            j = i % nq
            args = [h, x.data_ptr(), nw.data_ptr(), Q[j][0].data_ptr(), Q[j][1].data_ptr(), bq.data_ptr(),
                    K[j][0].data_ptr(), K[j][1].data_ptr(), bk.data_ptr(), V[j][0].data_ptr(), V[j][1].data_ptr(),
                    bv.data_ptr()]
            if variant:
                args.append(ws_norm.data_ptr())
            args += [qo.data_ptr(), ko.data_ptr(), vo.data_ptr(), 1, 2048, 2048, 256, 64, 1e-6, sp]
            return getattr(lib, "kudacuda_qwen2_fused_rmsnorm_qkv_nf4" + variant)(*args)
        cases.append((f"qkv_nf4{variant or '_v1'}", qkv_bytes, f))
    # NF4 SwiGLU (hidden 2048, intermediate 11008)
    sw_bytes = 2 * ((11008 * 2048) // 2 + (11008 * 2048) // 16) + 2 * 2048 * 2 + 11008 * 2
    ns = copies_for(sw_bytes)
    G, U = nf4(11008, 2048, ns), nf4(11008, 2048, ns)
    h_out = torch.empty(11008, dtype=f16, device=device)
    xb, nwb = x.to(torch.bfloat16), nw.to(torch.bfloat16)
    for dt, sym, xi, ni in (("f16", "kudacuda_qwen2_swiglu_nf4", x, nw),
                            ("bf16", "kudacuda_qwen2_swiglu_nf4_bf16", xb, nwb)):
        def f(lib, h, i, sp, sym=sym, xi=xi, ni=ni):
            j = i % ns
            return getattr(lib, sym)(h, xi.data_ptr(), ni.data_ptr(), G[j][0].data_ptr(), G[j][1].data_ptr(),
                                     U[j][0].data_ptr(), U[j][1].data_ptr(), h_out.data_ptr(), 1, 2048, 11008, 64,
                                     1e-6, sp)
        cases.append((f"swiglu_nf4_{dt}", sw_bytes, f))
    # GQA decode (16 / 2 / 128 heads)
    q = torch.randn(16 * 128, device=device).to(f16)
    o = torch.empty(16 * 128, dtype=f16, device=device)
    scale = 1.0 / math.sqrt(128)
    for kv in (512, 1024, 2048):
        nbytes = 2 * 2 * kv * 128 * 2 + 2 * 16 * 128 * 2
        nk = copies_for(nbytes)
        KC = [torch.randn(2 * kv * 128, device=device).to(f16) for _ in range(nk)]
        VC = [torch.randn(2 * kv * 128, device=device).to(f16) for _ in range(nk)]

        def f(lib, h, i, sp, KC=KC, VC=VC, kv=kv, nk=nk):
            j = i % nk
            return lib.kudacuda_qwen2_gqa_decode(h, q.data_ptr(), KC[j].data_ptr(), VC[j].data_ptr(), o.data_ptr(),
                                                 1, 1, kv, 16, 2, 128, scale, sp)
        cases.append((f"gqa_direct_kv{kv}", nbytes, f))
        if kv == 512:
            kvl = torch.tensor([kv], dtype=torch.int32, device=device)
            wsg = torch.empty(16 * 8 * 130, dtype=torch.float32, device=device)

            def fg(lib, h, i, sp, KC=KC, VC=VC, nk=nk, kvl=kvl):
                j = i % nk
                return lib.kudacuda_qwen2_gqa_decode_graph(h, q.data_ptr(), KC[j].data_ptr(), VC[j].data_ptr(),
                                                           o.data_ptr(), 1, 1, 512, 16, 2, 128, scale,
                                                           kvl.data_ptr(), sp)

            def fw(lib, h, i, sp, KC=KC, VC=VC, nk=nk, kvl=kvl, wsg=wsg):
                j = i % nk
                return lib.kudacuda_qwen2_gqa_decode_workspace_v3(h, q.data_ptr(), KC[j].data_ptr(),
                                                                  VC[j].data_ptr(), o.data_ptr(), wsg.data_ptr(),
                                                                  kvl.data_ptr(), 1, 1, 512, 16, 2, 128, scale, sp)
            cases.append(("gqa_graph_cap512", nbytes, fg))
            cases.append(("gqa_workspace_v3_cap512", nbytes, fw))

    results = []
    stream = torch.cuda.Stream()
    sp = int(stream.cuda_stream)
    for name, nbytes, fn in cases:
        row = {"op": name, "bytes": nbytes}
        for lname, lib in libs.items():
            h = handles[lname]
            with torch.cuda.stream(stream):
                for i in range(launches):
                    assert fn(lib, h, i, sp) == 0, lib.kudacuda_last_error(h)
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(launches):
                    assert fn(lib, h, i, sp) == 0, lib.kudacuda_last_error(h)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):  # replay launches on the current stream: the timed one
                graph.replay()
                stream.synchronize()
                s.record(stream)
                for _ in range(reps):
                    graph.replay()
                e.record(stream)
            e.synchronize()
            us = s.elapsed_time(e) * 1e3 / (reps * launches)
            row[f"{lname}_us"] = round(us, 3)
            row[f"{lname}_gbs"] = round(nbytes / (us * 1e-6) / 1e9, 1)
            del graph
        row["speedup"] = round(row["reference_us"] / row["b200_us"], 2)
        results.append(row)
    torch.cuda.synchronize()
    for lname, lib in libs.items():
        lib.kudacuda_destroy(handles[lname])
    return results


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--op", default="all")
    p.add_argument("--copies", type=int, default=12)
    p.add_argument("--launches", type=int, default=36)
    p.add_argument("--reps", type=int, default=20)
    p.add_argument("--device", default="cuda:0")
    p.add_argument("--layers", type=int, default=36, help="--op persistent: decoder layers")
    p.add_argument("--kv", type=int, default=512, help="--op persistent: tokens attended (kv_len)")
    p.add_argument("--prompt", type=int, default=512, help="--op prefill: prompt tokens")
    args = p.parse_args(argv)
    import torch

    torch.cuda.set_device(torch.device(args.device))
    if args.op == "refcompare":
        for r in time_refcompare(torch, args.device, args.launches, args.reps):
            print(json.dumps(r), flush=True)
        return 0
    if args.op == "prefill":
        r = time_prefill(torch, args.prompt, args.device)
        print(json.dumps(r), flush=True)
        return 1 if r["device_error_word"] else 0
    if args.op == "persistent":
        r = time_persistent(torch, args.layers, args.kv, max(args.launches, 1), args.reps, args.device)
        print(json.dumps(r), flush=True)
        return 1 if r["device_error_word"] else 0
    names = (["gemv_11008x2048", "gemv_2048x11008", "qkv_rope", "oproj", "down", "swiglu", "gqa512", "gqa2048",
              "lm_head"] if args.op == "all" else args.op.split(","))
    bridge = KudaCudaBridge(device_id=torch.device(args.device).index or 0)
    stream = torch.cuda.Stream()
    for case in build_cases(torch, bridge, names, args.copies, args.device):
        print(json.dumps(time_case(torch, bridge, case, args.launches, args.reps, stream)), flush=True)
    err = bridge.error_word(clear=True)
    if err:
        print(json.dumps({"device_error_word": err}))
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
