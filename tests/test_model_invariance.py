"""Model-level invariance harness: CPU tests of the report
logic with a synthetic adapter (mirroring test_investigation_harness.py:9-70
of the reference suite), and a GPU test of the random-init pi0-style VLA
step under set_batch_invariant_mode."""

from __future__ import annotations

import json

import pytest
import torch

from batch_invariant_ops.model_invariance import compare_outputs, run_investigation


class SyntheticAdapter:
    name = "synthetic"

    def __init__(self, batch_dependent: bool = False, oom_at: int | None = None) -> None:
        self.batch_dependent = batch_dependent
        self.oom_at = oom_at

    def load_model(self):
        return torch.nn.Identity()

    def load_example_inputs(self, count: int):
        return [{"x": torch.tensor([float(i), 2.0])} for i in range(count)]

    def run_model(self, model, batch):
        if self.oom_at is not None and batch["x"].shape[0] >= self.oom_at:
            raise torch.OutOfMemoryError("CUDA out of memory (synthetic)")
        actions = model(batch["x"])
        if self.batch_dependent:
            actions = actions + actions.shape[0]
        return {"actions": actions, "trajectory": (actions[:, None, :],)}

    def extract_robot_output(self, output):
        return output


def test_compare_outputs_reports_first_difference_and_hashes():
    [d] = compare_outputs({"actions": torch.tensor([[1.0, 2.0]])},
                          {"actions": torch.tensor([[1.0, 3.0]])})
    assert not d.exact
    assert d.differing_elements == 1
    assert d.first_differing_index == (0, 1)
    assert d.max_abs_difference == 1.0
    assert d.reference_hash != d.candidate_hash


def test_compare_outputs_rejects_structure_mismatch():
    with pytest.raises(ValueError):
        compare_outputs({"a": torch.zeros(1)}, {"b": torch.zeros(1)})


def test_investigation_covers_duplicate_and_unrelated(tmp_path):
    out = tmp_path / "result.json"
    report = run_investigation(SyntheticAdapter(), batch_sizes=(1, 2, 3, 5), output_path=out)
    assert report["repeatability"]["exact"]
    assert report["end_to_end_exact"]
    assert report["maximum_tested_batch"] == 5
    assert [r["batch_size"] for r in report["composition_results"]["duplicate"]] == [1, 2, 3, 5]
    assert json.loads(out.read_text())["end_to_end_exact"]


def test_investigation_detects_batch_dependent_output():
    report = run_investigation(SyntheticAdapter(batch_dependent=True), batch_sizes=(1, 2, 3))
    assert report["repeatability"]["exact"]
    assert not report["end_to_end_exact"]
    assert report["composition_results"]["duplicate"][0]["status"] == "PASS"
    assert report["composition_results"]["duplicate"][1]["status"] == "FAIL"
    assert report["composition_results"]["unrelated"][2]["tensors"][0]["differing_elements"] == 2


def test_investigation_records_oom_and_stops_that_composition():
    report = run_investigation(SyntheticAdapter(oom_at=3), batch_sizes=(1, 2, 3, 5))
    dup = report["composition_results"]["duplicate"]
    assert [r["status"] for r in dup] == ["PASS", "PASS", "OOM"]
    assert report["maximum_tested_batch"] == 2
    assert report["end_to_end_exact"]


def test_batch_sizes_must_include_one():
    with pytest.raises(ValueError):
        run_investigation(SyntheticAdapter(), batch_sizes=(2, 3))


def test_vla_tiny_runs_through_the_harness_on_cpu():
    from batch_invariant_ops.vla import VLAAdapter, VLAConfig

    report = run_investigation(VLAAdapter(VLAConfig.tiny(), device="cpu"), batch_sizes=(1, 2))
    assert report["repeatability"]["exact"]
    paths = [t["path"] for t in report["composition_results"]["duplicate"][0]["tensors"]]
    assert paths == ["output.actions", "output.prefix"]


@pytest.mark.gpu
def test_vla_step_is_batch_invariant_under_the_mode():
    from batch_invariant_ops.vla import VLAAdapter, VLAConfig

    report = run_investigation(VLAAdapter(VLAConfig.tiny(), device="cuda"),
                               batch_sizes=(1, 2, 3, 5, 8), invariant_ops=True)
    assert report["repeatability"]["exact"]
    bad = [(k, r["batch_size"]) for k, rs in report["composition_results"].items() for r in rs
           if r["status"] != "PASS"]
    assert report["end_to_end_exact"], bad
