"""raya's kernel-bench result file written from the B200 kernel
(raya_b200/kernel_bench.py), checked field by field against the reference's
contract specs/007-block-local-kernel/contracts/bench-output.md:8-24 (paths
relative to the raya project root): the label from RAYA_TARGET_MACHINE, the
metadata keys, and one result row per (seq, mask) with its timing and the
qk/softmax/pv stage percentages of the kernel that ran.
"""
import json

import pytest

from raya_b200 import kernel_bench

pytestmark = pytest.mark.gpu

META_KEYS = {"cpu_model", "logical_cpus", "physical_cpus", "threads", "features", "backend", "rustflags", "rustc",
             "git_commit", "timestamp"}
ROW_KEYS = {"kernel", "mask", "backend", "seq", "heads", "head_dim", "threads", "mean_ms", "stddev_ms", "samples",
            "stages"}


@pytest.mark.parametrize("target,label", [("", "unlabeled machine, indicative only"),
                                          ("cloud-agent", "cloud-agent hardware, indicative only")])
def test_result_file_follows_the_bench_output_contract(cuda_device, tmp_path, monkeypatch, target, label):
    monkeypatch.setenv("RAYA_BENCH_SEQS", "2048")
    monkeypatch.setenv("RAYA_TARGET_MACHINE", target)
    path = kernel_bench.run(str(tmp_path))
    assert path.startswith(str(tmp_path / "results" / "kernel-bench"))
    doc = json.load(open(path))
    assert set(doc) == {"label", "metadata", "results"}
    assert doc["label"] == label == doc["metadata"]["label"]
    assert META_KEYS <= set(doc["metadata"])
    assert isinstance(doc["metadata"]["features"], list)
    rows = doc["results"]
    assert {(r["seq"], r["mask"]) for r in rows} == {(2048, "block3"), (2048, "window64")}
    for r in rows:
        assert ROW_KEYS <= set(r)
        assert (r["heads"], r["head_dim"], r["samples"]) == (16, 64, kernel_bench.SAMPLES)
        assert r["mean_ms"] > 0 and r["stddev_ms"] >= 0
        st = r["stages"]
        assert set(st) == {"qk_pct", "softmax_pct", "pv_pct"}
        assert abs(st["qk_pct"] + st["softmax_pct"] + st["pv_pct"] - 100.0) < 1e-6
    assert "85 ms" not in open(path).read()  # the contract: no comparison with the 85 ms figure
