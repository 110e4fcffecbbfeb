"""Generate the golden fixtures in tests/golden/ from the reference's own
Python code (run in a container that has the reference checkout; the GPU box
does not, so the outputs are committed).

    python tests/golden/make_golden.py --reference /path/to/KudaCuda   (or KUDACUDA_REFERENCE=...)

Sources imported from the reference:
  harness/reference.py:9-31                        rmsnorm_reference (float64)
  tools/correctness/run_qwen2_gqa_check.py:19-28   reference_qwen2_gqa (torch FP32)
  harness/compare.py:20-95                         compare_values (its verdict is stored too)
Inputs are seeded (numpy default_rng / torch.Generator, seed 20260824).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SEED = 20260824


def import_reference(ref: Path):
    tmp = Path(tempfile.mkdtemp(prefix="kc_refpkg_"))
    (tmp / "KudaCuda").symlink_to(ref)
    sys.path.insert(0, str(tmp))
    from KudaCuda.harness.reference import rmsnorm_reference  # noqa: E402
    from KudaCuda.harness.compare import compare_values  # noqa: E402
    from KudaCuda.tools.correctness.run_qwen2_gqa_check import reference_qwen2_gqa  # noqa: E402

    return rmsnorm_reference, compare_values, reference_qwen2_gqa


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, default=os.environ.get("KUDACUDA_REFERENCE"),
                        help="path of the reference checkout (or set KUDACUDA_REFERENCE)")
    args = parser.parse_args()
    if args.reference is None:
        parser.error("give --reference PATH or set KUDACUDA_REFERENCE")
    rmsnorm_reference, compare_values, reference_qwen2_gqa = import_reference(Path(args.reference))
    import torch

    g = np.random.default_rng(SEED)
    # --- RMSNorm: 3 rows x 2048 and a ragged 1 x 37 case, eps 1e-5 / 1e-6
    cases = {}
    for name, (rows, hidden, eps) in {"rms_2048": (3, 2048, 1e-5), "rms_37": (1, 37, 1e-6)}.items():
        x = g.standard_normal((rows, hidden))
        w = 1.0 + 0.02 * g.standard_normal(hidden)
        out = np.array(rmsnorm_reference(x.tolist(), w.tolist(), eps), dtype=np.float64)
        cases[name] = dict(x=x, w=w, eps=np.float64(eps), out=out)
    np.savez_compressed(HERE / "rmsnorm_reference.npz", **{f"{k}__{f}": v for k, d in cases.items() for f, v in d.items()})

    # --- GQA: the reference check tool's seeded randn inputs at its kv lengths
    gen = torch.Generator().manual_seed(SEED)
    gqa = {}
    for kv_len in (1, 7, 128, 512, 585):
        q = torch.randn((1, 16, 1, 128), generator=gen, dtype=torch.float32).to(torch.float16)
        k = torch.randn((1, 2, kv_len, 128), generator=gen, dtype=torch.float32).to(torch.float16)
        v = torch.randn((1, 2, kv_len, 128), generator=gen, dtype=torch.float32).to(torch.float16)
        out = reference_qwen2_gqa(torch, q, k, v)
        gqa[f"kv{kv_len}__q"] = q.view(torch.int16).numpy().view(np.uint16)
        gqa[f"kv{kv_len}__k"] = k.view(torch.int16).numpy().view(np.uint16)
        gqa[f"kv{kv_len}__v"] = v.view(torch.int16).numpy().view(np.uint16)
        gqa[f"kv{kv_len}__out"] = out.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(HERE / "gqa_reference.npz", **gqa)

    # --- compare_values verdicts on fixed vectors (pins the comparison rule)
    verdicts = []
    for actual, expected, kw in (
        ([1.0, 2.0, 3.0], [1.0, 2.0, 3.0], {}),
        ([1.0, 2.001], [1.0, 2.0], {"atol": 1e-4, "rtol": 1e-4}),
        ([1.0, 2.001], [1.0, 2.0], {"atol": 2e-3, "rtol": 0.0}),
        ([float("nan")], [1.0], {}),
        ([float("inf")], [float("inf")], {}),
        ([1.0], [1.0, 2.0], {}),
    ):
        r = compare_values(actual, expected, **kw)
        verdicts.append({"actual": actual, "expected": expected, "kwargs": kw, "passed": bool(r["passed"])})
    (HERE / "compare_values.json").write_text(json.dumps(verdicts, indent=1, allow_nan=True) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")), "compare_values.json")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
