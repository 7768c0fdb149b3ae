"""The GPU job target (glaucis_b200/kube_job.py and the B200 Job template):
job naming and rendering as the reference's KubeEvaluator does
(KE/tests/test_kube_evaluator.py:43-70, :313-324), and the rendered Job's
GPU request, node selection, payload mount and evaluator command."""
import string

import yaml

from glaucis_b200 import evaluate, kube_job


def test_job_name_generation():
    name = kube_job.make_job_name("v001_abc123")
    assert name.startswith("kernel-eval-") and "abc123" in name and len(name) <= 63


def test_job_name_sanitizes_special_chars():
    name = kube_job.make_job_name("v001.gen5_abc123")
    assert name.startswith("kernel-eval-") and "." not in name
    assert not name.endswith("-") and len(name) <= 63
    assert len(kube_job.make_job_name("x" * 200)) <= 63


def _job(rendered):
    docs = [d for d in yaml.safe_load_all(rendered) if d]
    assert len(docs) == 1
    return docs[0]


def test_render_job_yaml_b200_target():
    target = kube_job.JobTarget(repo="sii-xinglong/Glaucis", branch="main")
    rendered = kube_job.render_job_yaml(target, "kernel-eval-v001", "v001_abc123")
    assert "${" not in rendered
    job = _job(rendered)
    assert job["kind"] == "Job" and job["metadata"]["name"] == "kernel-eval-v001"
    assert job["spec"]["activeDeadlineSeconds"] == 600 and job["spec"]["backoffLimit"] == 0
    pod = job["spec"]["template"]["spec"]
    c = pod["containers"][0]
    assert c["resources"]["limits"]["nvidia.com/gpu"] == "1"
    assert c["resources"]["requests"]["nvidia.com/gpu"] == "1"
    assert "google.com/tpu" not in c["resources"]["limits"]
    assert pod["nodeSelector"] == {"nvidia.com/gpu.product": "NVIDIA-B200"}
    script = c["command"][-1]
    assert "python -m glaucis_b200.evaluate --eval-payload-file /etc/eval-payload/payload" in script
    assert "g.build()" in script
    env = {e["name"]: e["value"] for e in c["env"]}
    assert env["REPO"] == "sii-xinglong/Glaucis" and env["VARIANT_ID"] == "v001_abc123"
    vols = {v["name"]: v for v in pod["volumes"]}
    assert vols["eval-payload"]["configMap"]["name"] == "kernel-eval-v001-payload"
    mounts = {m["name"]: m["mountPath"] for m in c["volumeMounts"]}
    assert mounts["eval-payload"] == "/etc/eval-payload"


def test_batch_deadline_and_reference_renderer_compatibility():
    target = kube_job.JobTarget(repo="o/r")
    job = _job(kube_job.render_batch_job_yaml(target, "kernel-eval-batch-2v", 2))
    assert job["spec"]["activeDeadlineSeconds"] == 900  # 2 variants x 300 + 300
    # the reference renderer fills exactly these five names: nothing else is left
    text = open(target.job_template).read()
    rendered = string.Template(text).safe_substitute(
        JOB_NAME="j", BRANCH="main", REPO="o/r", VARIANT_ID="v", ACTIVE_DEADLINE="600")
    assert "${" not in rendered and _job(rendered)["metadata"]["name"] == "j"


def test_payload_configmap_carries_an_evaluator_request():
    req = {"variant_id": "v1", "kernel_code": "def f(): pass", "reference_code": "",
           "shapes": [{"M": 128}], "rtol": 1e-2, "atol": 1.0}
    payload = evaluate.encode_request(req)
    cm = yaml.safe_load(kube_job.render_payload_configmap(kube_job.JobTarget(), "kernel-eval-v1", payload))
    assert cm["kind"] == "ConfigMap" and cm["metadata"]["name"] == "kernel-eval-v1-payload"
    assert evaluate.decode_request(cm["data"]["payload"])["variant_id"] == "v1"
