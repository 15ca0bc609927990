"""Evidence report in the reference's dominus-ultra-evidence-v1 format (gpu_evidence.py:35,
:506-523): schema, canonical payload hash, case labels and suites (CPU); the quick suite end
to end on the GPU."""

import hashlib
import json

import pytest

from dominusultra_b200 import evidence


def test_suites_and_labels_follow_the_reference_protocol():
    assert evidence.SCHEMA_VERSION == "dominus-ultra-evidence-v1"
    assert len(evidence.QUICK_CASES) == 4 and len(evidence.FULL_CASES) == 10
    assert evidence.QUICK_CASES[1].label == "prefill:B1:Hq8:Hkv2:T257:D64"
    assert evidence.FULL_CASES[-1].label == "decode:B2:Hq8:Hkv2:T512:D128"
    assert evidence.tolerances("bfloat16") == {"atol": 2e-2, "rtol": 2e-2, "lse_atol": 5e-2}
    assert evidence.tolerances("float16") == {"atol": 6e-3, "rtol": 6e-3, "lse_atol": 2e-2}


def test_report_hash_is_over_the_canonical_payload(tmp_path):
    result = {"label": "prefill:B1:Hq8:Hkv8:T128:D64", "dtype": "bfloat16", "status": "pass",
              "kernel": {"median_ms": 1.0}, "baseline_timing": {"median_ms": 2.0},
              "speedup_median": 2.0, "extra": [1.5, "x"]}
    payload = {"verdict": "pass", "suite": "quick", "results": [result],
               "environment": {"device_name": "B200", "compute_capability": "10.0",
                               "multiprocessor_count": 148, "implementation": "x",
                               "git": {"commit": "c"}}}
    report = evidence.make_report(payload)
    blob = json.dumps(payload, sort_keys=True, separators=(",", ":"), ensure_ascii=True)
    assert report["payload_sha256"] == hashlib.sha256(blob.encode()).hexdigest()
    assert report["schema_version"] == evidence.SCHEMA_VERSION
    stats = evidence.latency_stats([1.0, 2.0, 3.0, 4.0])
    assert stats["median_ms"] == 2.5 and stats["min_ms"] == 1.0 and stats["max_ms"] == 4.0
    json_path, md_path, sha = evidence.write_report(tmp_path, payload)
    assert json.loads(json_path.read_text())["payload_sha256"] == sha
    assert "PASS" in md_path.read_text()


@pytest.mark.gpu
def test_quick_suite_passes_on_the_gpu(cuda_device, tmp_path):
    rc = evidence.main(["--suite", "quick", "--warmup", "2", "--iterations", "3",
                        "--output-dir", str(tmp_path)])
    assert rc == 0
    (json_path,) = tmp_path.glob("*.json")
    report = json.loads(json_path.read_text())
    assert report["payload"]["verdict"] == "pass"
    assert all(r["status"] == "pass" for r in report["payload"]["results"])
    assert report["payload"]["environment"]["compute_capability"] == "10.0"
