"""End-to-end evaluator runs on the B200 templates: compile -> correctness
against the oracle-backed reference templates -> CUDA-event benchmark.
Loss tolerances follow the reference's YAML configs (GMM atol 1.0,
KE/examples/gmm_fp8_blockwise.yaml:20-21; GLA atol 10.0,
KE/examples/chunk_gla.yaml:22)."""
import json
import os
import subprocess
import sys

import pytest

from glaucis_b200 import evaluate as E

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _read(*p):
    return open(os.path.join(ROOT, *p)).read()


def test_evaluate_gmm_template(cuda):
    req = {"variant_id": "gmm", "kernel_code": _read("glaucis_b200", "kernels", "gmm_fp8_blockwise.py"),
           "reference_code": _read("tests", "ref_templates", "gmm_fp8_blockwise_ref.py"),
           "shapes": [{"M": 1024, "K": 512, "N": 256, "G": 4}], "rtol": 1e-2, "atol": 1.0}
    r = E.evaluate(req)
    assert r["status"] == "SUCCESS", r.get("error")
    assert r["latency_ms"] > 0 and r["metadata"]["benchmark"]["timing_source"] == "cuda_events"


def test_evaluate_gla_template(cuda):
    req = {"variant_id": "gla", "kernel_code": _read("glaucis_b200", "kernels", "chunk_gla.py"),
           "reference_code": _read("tests", "ref_templates", "chunk_gla_ref.py"),
           "shapes": [{"B": 1, "T": 256, "H": 2, "K": 128, "V": 128, "chunk_size": 64}],
           "rtol": 1e-2, "atol": 10.0}
    r = E.evaluate(req)
    assert r["status"] == "SUCCESS", r.get("error")


def test_evaluate_cli_prints_result_line(cuda):
    req = {"variant_id": "cli", "kernel_code": _read("glaucis_b200", "kernels", "gmm_fp8_blockwise.py"),
           "reference_code": _read("tests", "ref_templates", "gmm_fp8_blockwise_ref.py"),
           "shapes": [{"M": 512, "K": 256, "N": 256, "G": 2}], "atol": 1.0}
    env = dict(os.environ, PYTHONPATH=ROOT)
    p = subprocess.run([sys.executable, "-m", "glaucis_b200.evaluate", "--eval-payload",
                        E.encode_request(req)], capture_output=True, text=True, timeout=300,
                       cwd=ROOT, env=env)
    line = [l for l in p.stdout.splitlines() if l.startswith("EVAL_RESULT:")]
    assert p.returncode == 0 and line, p.stderr[-2000:]
    assert json.loads(line[0].split(":", 1)[1])["status"] == "SUCCESS"
