"""CUDA evaluator backend: request/result contract, stages and batch dispatch
(CPU, with injected timers and fake subprocesses), plus the template
conventions of the Glaucis kernel templates."""
import ast
import json
import os
import sys

import numpy as np
import pytest

from glaucis_b200 import evaluate as E

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TEMPLATES = os.path.join(ROOT, "glaucis_b200", "kernels")


def _fake_timer(fn):
    fn()
    return 2.0


KERNEL_OK = "def optimized_compute(n=3):\n    return float(n) * 1.0\n"
REF_OK = "def simple_compute(n=3):\n    return float(n)\n"


def test_request_roundtrip():
    req = {"variant_id": "v1", "kernel_code": KERNEL_OK, "reference_code": REF_OK,
           "shapes": [{"n": 2}], "rtol": 1e-2, "atol": 0.1}
    assert E.decode_request(E.encode_request(req)) == req


def test_compile_error_status():
    r = E.evaluate({"variant_id": "bad", "kernel_code": "def (:", "reference_code": REF_OK,
                    "shapes": [{"n": 1}]}, timer=_fake_timer)
    assert r["status"] == "COMPILE_ERROR" and "Compilation error" in r["error"]


def test_incorrect_scalar_beyond_atol():
    kernel = "def optimized_compute(n=3):\n    return n + 0.5\n"
    r = E.evaluate({"kernel_code": kernel, "reference_code": REF_OK, "shapes": [{"n": 1}],
                    "atol": 0.1}, timer=_fake_timer)
    assert r["status"] == "INCORRECT" and r["max_diff"] == pytest.approx(0.5)


def test_incorrect_array_elementwise():
    kernel = "import numpy as np\ndef optimized_compute(n=3):\n    return np.array([1.0, 2.0, 3.5])\n"
    ref = "import numpy as np\ndef reference_fn(n=3):\n    return np.array([1.0, 2.0, 3.0])\n"
    r = E.evaluate({"kernel_code": kernel, "reference_code": ref, "shapes": [{"n": 1}],
                    "rtol": 1e-2, "atol": 1e-3}, timer=_fake_timer)
    assert r["status"] == "INCORRECT"


def test_success_reports_speedup_and_stats():
    r = E.evaluate({"variant_id": "ok", "kernel_code": KERNEL_OK, "reference_code": REF_OK,
                    "shapes": [{"n": 4}], "atol": 0.1}, timer=_fake_timer)
    assert r["status"] == "SUCCESS" and r["speedup"] == pytest.approx(1.0)
    b = r["metadata"]["benchmark"]
    assert b["median_ms"] == 2.0 and len(b["evaluation_times_ms"]) == 5 and b["cv"] == 0.0
    json.dumps(r)  # EVAL_RESULT must serialise


def test_missing_entry_point():
    r = E.evaluate({"kernel_code": "x = 1\n", "reference_code": REF_OK, "shapes": [{"n": 1}]},
                   timer=_fake_timer)
    assert r["status"] == "INCORRECT" and "kernel_fn" in r["error"]


def test_forward_flops():
    assert E.forward_flops({"M": 2, "K": 3, "N": 4, "G": 1}) == 48.0
    assert E.forward_flops({"B": 8, "T": 4096, "H": 16, "K": 128, "V": 128,
                            "chunk_size": 64}) == pytest.approx(51.54e9, rel=1e-3)


FAKE_EVALUATOR = r"""
import base64, json, sys, time
req = json.loads(base64.b64decode(sys.argv[2]).decode())
code = req["kernel_code"]
if "SLEEP" in code:
    time.sleep(30)
if "CRASH" in code:
    sys.stderr.write("boom: segfault-like crash\n"); sys.exit(139)
print("noise")
print("EVAL_RESULT:" + json.dumps({"status": "SUCCESS", "latency_ms": 1.0}))
"""


def test_batch_dispatch_timeout_crash_and_success():
    payload = {"batch": True, "reference_code": REF_OK, "shapes": [{"n": 1}],
               "variants": [{"variant_id": "a", "kernel_code": "ok"},
                            {"variant_id": "b", "kernel_code": "SLEEP"},
                            {"variant_id": "c", "kernel_code": "CRASH"}]}
    lines = E.batch_dispatch(payload, per_variant_timeout=3,
                             argv_prefix=[sys.executable, "-c", FAKE_EVALUATOR])
    res = [json.loads(l.split("EVAL_RESULT:", 1)[1]) for l in lines]
    assert res[0]["status"] == "SUCCESS" and res[0]["variant_id"] == "a"
    assert res[1]["status"] == "COMPILE_ERROR" and "timeout" in res[1]["error"]
    assert res[2]["status"] == "COMPILE_ERROR" and "boom" in res[2]["error"]


def test_cli_without_gpu_exits_nonzero(capsys):
    if E._has_cuda():
        pytest.skip("a B200 is present")
    rc = E.main(["--eval-payload", E.encode_request({"kernel_code": KERNEL_OK,
                                                     "reference_code": REF_OK,
                                                     "shapes": [{"n": 1}]})])
    assert rc == 1


@pytest.mark.parametrize("name", ["gmm_fp8_blockwise.py", "chunk_gla.py"])
def test_template_conventions(name):
    # KE/tests/test_chunk_gla.py:27-52 and test_init_kernel_conventions.py:
    # the EVOLVE block is extractable, holds optimized_compute, and the
    # imports and _make_test_data stay outside it.
    text = open(os.path.join(TEMPLATES, name)).read()
    ast.parse(text)
    start, end = "# EVOLVE-BLOCK-START", "# EVOLVE-BLOCK-END"
    assert text.count(start) == 1 and text.count(end) == 1
    before, rest = text.split(start)
    block, _ = rest.split(end)
    assert "def optimized_compute(" in block
    assert "def _make_test_data(" in before
    assert "import" not in block
