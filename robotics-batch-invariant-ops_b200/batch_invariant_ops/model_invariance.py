"""Model-level batch-invariance investigation.

Runs one target sample alone and inside larger batches -- copies of itself
("duplicate") and mixed with other samples ("unrelated") -- and compares the
target's outputs bit for bit, with per-tensor diagnostics (differing element
count, first differing index, max/mean absolute difference, sha256 of the raw
bytes).  A batch size that runs out of device memory ends its composition
with an "OOM" record instead of failing the investigation.

Contract followed (field names, record layout and statuses are the report
format users of the reference parse): scripts/model_invariance/harness.py
:28-40 (adapter protocol), :43-55 (per-tensor record), :110-159
(comparison), :220-312 (investigation and report).
"""

from __future__ import annotations

import contextlib
import dataclasses
import hashlib
import json
import random
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any, Protocol

import numpy as np
import torch

DEFAULT_BATCH_SIZES = (1, 2, 3, 4, 5, 7, 8, 9, 15, 16, 17, 31, 32, 33, 64)


class ModelAdapter(Protocol):
    """What the investigation needs from a model.  Optional hooks:
    ``compose_batch(samples)`` and ``reset_model(model)``."""

    name: str

    def load_model(self) -> Any: ...

    def load_example_inputs(self, count: int) -> Sequence[Any]: ...

    def run_model(self, model: Any, batch: Any) -> Any: ...

    def extract_robot_output(self, output: Any) -> Any: ...


@dataclasses.dataclass
class TensorDifference:
    path: str
    reference_shape: tuple[int, ...]
    candidate_shape: tuple[int, ...]
    dtype: str
    exact: bool
    differing_elements: int | None
    max_abs_difference: float | None
    mean_abs_difference: float | None
    first_differing_index: tuple[int, ...] | None
    reference_hash: str
    candidate_hash: str


def seed_everything(seed: int) -> None:
    """Reset the host and device random generators before a run."""
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def tensor_sha256(tensor: torch.Tensor) -> str:
    """sha256 of the tensor's raw bytes (contiguous, host copy)."""
    data = tensor.detach().contiguous().cpu()
    return hashlib.sha256(data.reshape(-1).view(torch.uint8).numpy().tobytes()).hexdigest()


def _leaves(value: Any, path: str, out: dict[str, torch.Tensor]) -> None:
    if isinstance(value, torch.Tensor):
        out[path] = value
    elif isinstance(value, Mapping):
        for key in sorted(value, key=str):
            _leaves(value[key], f"{path}.{key}", out)
    elif isinstance(value, (list, tuple)):
        for index, item in enumerate(value):
            _leaves(item, f"{path}[{index}]", out)
    else:
        raise TypeError(f"{path} contains unsupported output type {type(value).__name__}")


def flatten_tensors(value: Any, path: str = "output") -> dict[str, torch.Tensor]:
    """Tensor leaves of a nested output, keyed by access path (mapping keys
    in sorted order)."""
    out: dict[str, torch.Tensor] = {}
    _leaves(value, path, out)
    return out


def first_sample(value: Any) -> Any:
    """The first batch entry of every tensor of a nested output (scalars kept)."""
    if isinstance(value, torch.Tensor):
        return value if value.ndim == 0 else value[:1]
    if isinstance(value, Mapping):
        return type(value)((key, first_sample(item)) for key, item in value.items())
    if isinstance(value, tuple):
        return tuple(first_sample(item) for item in value)
    if isinstance(value, list):
        return [first_sample(item) for item in value]
    raise TypeError(f"unsupported output type {type(value).__name__}")


def _diff(path: str, ref: torch.Tensor, cand: torch.Tensor) -> TensorDifference:
    comparable = ref.shape == cand.shape and ref.dtype == cand.dtype
    count = first = max_abs = mean_abs = None
    if comparable:
        mask = ref != cand
        count = int(mask.sum().item())
        hits = torch.nonzero(mask, as_tuple=False)
        first = tuple(int(i) for i in hits[0].tolist()) if hits.numel() else None
        if ref.is_floating_point() or ref.is_complex():
            delta = (ref - cand).abs().float()
            max_abs = float(delta.max().item()) if delta.numel() else 0.0
            mean_abs = float(delta.mean().item()) if delta.numel() else 0.0
    return TensorDifference(
        path=path,
        reference_shape=tuple(ref.shape),
        candidate_shape=tuple(cand.shape),
        dtype=str(ref.dtype),
        exact=bool(comparable and torch.equal(ref, cand)),
        differing_elements=count,
        max_abs_difference=max_abs,
        mean_abs_difference=mean_abs,
        first_differing_index=first,
        reference_hash=tensor_sha256(ref),
        candidate_hash=tensor_sha256(cand),
    )


def compare_outputs(reference: Any, candidate: Any) -> list[TensorDifference]:
    """Exactness and magnitude diagnostics for every output tensor; the two
    outputs must have the same nested structure."""
    ref = flatten_tensors(reference)
    cand = flatten_tensors(candidate)
    if ref.keys() != cand.keys():
        raise ValueError(
            f"output structures differ: reference={sorted(ref)}, candidate={sorted(cand)}"
        )
    return [_diff(path, ref[path], cand[path]) for path in ref]


def default_compose_batch(samples: Sequence[Any]) -> Any:
    """Stack samples into a batch: tensors along a new leading dimension,
    containers element-wise; non-tensor metadata must agree across samples."""
    head = samples[0]
    if isinstance(head, torch.Tensor):
        return torch.stack(list(samples))
    if isinstance(head, Mapping):
        return type(head)((k, default_compose_batch([s[k] for s in samples])) for k in head)
    if isinstance(head, (tuple, list)):
        parts = [default_compose_batch([s[i] for s in samples]) for i in range(len(head))]
        return tuple(parts) if isinstance(head, tuple) else parts
    if isinstance(head, (bool, int, float, str)):
        if any(s != head for s in samples):
            raise ValueError("non-tensor metadata differs; provide adapter.compose_batch")
        return head
    raise TypeError(f"cannot batch {type(head).__name__}; provide adapter.compose_batch")


def _compose(adapter: ModelAdapter, samples: Sequence[Any]) -> Any:
    return getattr(adapter, "compose_batch", default_compose_batch)(samples)


def _infer(adapter: ModelAdapter, model: Any, batch: Any, seed: int) -> Any:
    seed_everything(seed)
    reset = getattr(adapter, "reset_model", None)
    if reset is not None:
        reset(model)
    with torch.inference_mode():
        out = adapter.run_model(model, batch)
    return adapter.extract_robot_output(out)


def is_out_of_memory(error: BaseException) -> bool:
    if isinstance(error, torch.OutOfMemoryError):
        return True
    return "out of memory" in str(error).lower()


def _record(diffs: list[TensorDifference]) -> dict[str, Any]:
    return {"exact": all(d.exact for d in diffs), "tensors": [dataclasses.asdict(d) for d in diffs]}


def run_investigation(
    adapter: ModelAdapter,
    *,
    batch_sizes: Sequence[int] = DEFAULT_BATCH_SIZES,
    invariant_ops: bool = False,
    seed: int = 0,
    output_path: str | Path | None = None,
) -> dict[str, Any]:
    """Repeatability, then duplicate and unrelated compositions at every batch
    size; ``invariant_ops`` runs everything under set_batch_invariant_mode.
    Returns (and optionally writes as JSON) the report."""
    sizes = tuple(sorted(set(int(b) for b in batch_sizes)))
    if not sizes or sizes[0] != 1:
        raise ValueError("batch_sizes must be positive and include 1")

    seed_everything(seed)
    model = adapter.load_model()
    if hasattr(model, "eval"):
        model.eval()
    examples = list(adapter.load_example_inputs(max(sizes)))
    if not examples:
        raise ValueError("adapter returned no example inputs")
    if max(sizes) > 1 and len(examples) < 2:
        raise ValueError("unrelated composition requires at least two example inputs")
    target = examples[0]

    report: dict[str, Any] = {
        "model": adapter.name,
        "batch_invariant_ops": invariant_ops,
        "seed": seed,
        "requested_batch_sizes": list(sizes),
        "repeatability": None,
        "composition_results": {"duplicate": [], "unrelated": []},
        "maximum_tested_batch": None,
        "end_to_end_exact": False,
    }
    if invariant_ops:
        from .batch_invariant_ops import set_batch_invariant_mode

        mode = set_batch_invariant_mode()
    else:
        mode = contextlib.nullcontext()
    with mode:
        single = _compose(adapter, [target])
        reference = _infer(adapter, model, single, seed)
        report["repeatability"] = _record(
            compare_outputs(reference, _infer(adapter, model, single, seed))
        )
        if not report["repeatability"]["exact"]:
            report["failure"] = "same-batch inference is not repeatable"
        else:
            largest = 1
            others = examples[1:]
            for kind in ("duplicate", "unrelated"):
                for size in sizes:
                    if kind == "duplicate":
                        samples = [target] * size
                    else:
                        samples = [target] + [others[i % len(others)] for i in range(size - 1)]
                    try:
                        out = _infer(adapter, model, _compose(adapter, samples), seed)
                    except RuntimeError as error:
                        if not is_out_of_memory(error):
                            raise
                        if torch.cuda.is_available():
                            torch.cuda.empty_cache()
                        report["composition_results"][kind].append(
                            {"batch_size": size, "status": "OOM"}
                        )
                        break
                    diffs = compare_outputs(reference, first_sample(out))
                    entry = {
                        "batch_size": size,
                        "status": "PASS" if all(d.exact for d in diffs) else "FAIL",
                    }
                    entry.update(_record(diffs))
                    report["composition_results"][kind].append(entry)
                    largest = max(largest, size)
            report["maximum_tested_batch"] = largest
            done = [
                entry
                for entries in report["composition_results"].values()
                for entry in entries
                if entry["status"] != "OOM"
            ]
            report["end_to_end_exact"] = bool(done) and all(e["status"] == "PASS" for e in done)

    if output_path is not None:
        path = Path(output_path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(report, indent=2) + "\n")
    return report
