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


# ---------------------------------------------------------------------------
# deep profile stage (ncu counters), host logic only
# ---------------------------------------------------------------------------
_NCU_CSV = "\n".join([
    '==PROF== Connected to process 1',
    '"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size",'
    '"Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"',
] + [
    f'"{i}","1","python3","h","{k}","1","7","(384, 1, 1)","(148, 1, 1)","0","10.0",'
    f'"Command line profiler metrics","{m}","{u}","{v}"'
    for i, k, rows in [
        (0, "void gl::gmm::gmm_fp8_fwd_kernel<256>(CUtensorMap_st, CUtensorMap_st, gl::gmm::Params)",
         [("gpu__time_duration.sum", "ns", "300000"),
          ("sm__throughput.avg.pct_of_peak_sustained_elapsed", "%", "60"),
          ("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "%", "40"),
          ("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed", "%", "45"),
          ("dram__bytes_read.sum", "byte", "1,000,000")]),
        (1, "void quant::quant_kernel<0>(CUtensorMap_st, quant::Args)",
         [("gpu__time_duration.sum", "ns", "100000"),
          ("sm__throughput.avg.pct_of_peak_sustained_elapsed", "%", "20"),
          ("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "%", "80"),
          ("dram__bytes_write.sum", "Kbyte", "500")]),
    ] for m, u, v in rows])


def test_parse_ncu_csv_and_summary():
    ls = E.parse_ncu_csv(_NCU_CSV)
    assert len(ls) == 2
    assert ls[0]["duration_ns"] == 300000 and ls[0]["dram_read_bytes"] == 1e6
    assert ls[1]["dram_write_bytes"] == 5e5
    s = E.summarize_launches(ls)
    assert s["ok"] and s["hw_utilization"]["launches"] == 2
    sm = (60 * 3 + 20) / 4.0
    dram = (40 * 3 + 80) / 4.0
    assert abs(s["hw_utilization"]["sm_throughput_pct"] - sm) < 1e-9
    assert abs(s["compute_ratio"] - sm / (sm + dram)) < 1e-12
    assert abs(s["compute_ratio"] + s["memory_transfer_ratio"] - 1.0) < 1e-12
    assert s["hw_utilization"]["tensor_util_pct"] == 45.0   # only launches that report it
    assert s["hw_utilization"]["dram_bytes"] == 1.5e6
    assert abs(s["hw_utilization"]["kernel_time_ms"] - 0.4) < 1e-12


def test_stage_profile_deep_runs_plain_then_ncu():
    calls = []

    def runner(argv):
        calls.append(argv)
        return (0, _NCU_CSV, "") if argv[0] == "ncu" else (0, "", "")

    req = {"kernel_code": "def kernel_fn(n):\n    return n\n", "shapes": [{"n": 1}]}
    r = E.stage_profile_deep(req, runner=runner)
    assert r["ok"] and len(calls) == 2
    assert calls[0][1:3] == ["-m", "glaucis_b200.evaluate"] and "--profile-child" in calls[0]
    assert calls[1][0] == "ncu" and "--clock-control" in calls[1] and "none" in calls[1]
    assert "--profile-from-start" in calls[1]
    # a child that fails without ncu is never profiled
    calls.clear()
    r = E.stage_profile_deep(req, runner=lambda argv: calls.append(argv) or (1, "", "boom"))
    assert not r["ok"] and len(calls) == 1
