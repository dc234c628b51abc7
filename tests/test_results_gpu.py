"""The measured results file (nkilab.results) in its --quick form: every section of the
reference's dashboard layout present, every timing measured, correctness rows small."""
from __future__ import annotations

import json

import pytest

pytestmark = pytest.mark.gpu


def test_results_json_quick(tmp_path):
    from nkilab import results

    out = tmp_path / "results.json"
    results.main(["--out", str(out), "--quick"])
    d = json.loads(out.read_text())
    for key in ("generated_at", "git_sha", "quick", "versions", "hardware_model", "matmul", "norm", "attention",
                "decoder_block", "correctness"):
        assert key in d
    entries = d["matmul"]["variants"] + d["norm"]["variants"] + d["attention"]["ladder"]
    assert [e["kernel"] for e in d["attention"]["ladder"]][0].startswith("naive")
    for e in entries:
        assert e["measured"] and e["measured_latency_us"] > 0 and 0 < e["pct_of_roofline"] <= 150
    assert all(p["measured_latency_us"] > 0 for p in d["decoder_block"]["parts"])
    assert d["decoder_block"]["max_abs_err_vs_pytorch"] < 1e-3
    assert all(c["vs_torch"] < 5e-2 for c in d["correctness"])
