"""Extract the extended shape regression cases (real VLA operator shapes) from
the reference's research/*/benchmarks.json into extended_shapes.json.

Each benchmark case names an operator and its shapes; cases are classified by
the keys of their shape record and the largest benchmarked batch of every
(model, operator) is kept.  Run from the repository root with the reference
checked out at REFERENCE (default: the path below):

    python tests/golden/make_extended_shapes.py [REFERENCE]
"""

from __future__ import annotations

import glob
import json
import sys
from pathlib import Path


def classify(op: str, shape: dict) -> str | None:
    keys = set(shape)
    if {"experts", "top_k", "hidden"} <= keys:
        return "moe"
    if "logical_query_length" in keys:
        return "varlen"
    if {"query", "key"} <= keys:
        return "sdpa"
    if {"left", "right"} <= keys:
        return "addmm" if shape.get("bias") else "mm"
    if "output_padding" in keys:
        return "conv_transpose"
    if "groups" in keys and "padding" in keys and len(shape["input"]) == 3:
        return "depthwise_conv1d"
    if {"input", "weight", "stride"} <= keys:
        return "conv"
    if {"input", "weight"} <= keys:
        return "linear"
    if "dimension" in keys or ("dim" in keys and "mean" in op):
        return "mean"
    if "dim" in keys and "input" in keys:
        return "vector_norm"
    return None


def main() -> None:
    if len(sys.argv) != 2:
        sys.exit("usage: make_extended_shapes.py <reference checkout>")
    ref = Path(sys.argv[1])
    # one case per (model, operator): the largest benchmarked batch
    best: dict[str, dict] = {}
    for path in sorted(glob.glob(str(ref / "research" / "*" / "benchmarks.json"))):
        model = Path(path).parent.name
        for case in json.loads(Path(path).read_text()).get("cases", []):
            shape = case.get("shape") or {}
            kind = classify(case.get("operator", ""), shape)
            if kind is None:
                continue
            keep = {k: v for k, v in shape.items() if k not in ("checkpoint_boundary",
                                                                   "checkpoint_weight")}
            name = f"{model}:{case['operator']}"
            batch = int(case.get("batch_size", 1))
            if name not in best or batch > best[name]["batch"]:
                best[name] = {"id": name, "batch": batch, "kind": kind, "shape": keep}
    cases = list(best.values())
    out = Path(__file__).resolve().parent / "extended_shapes.json"
    out.write_text(json.dumps({"source": "reference research/*/benchmarks.json",
                               "cases": cases}, indent=1) + "\n")
    print(f"{len(cases)} cases -> {out}")


if __name__ == "__main__":
    main()
