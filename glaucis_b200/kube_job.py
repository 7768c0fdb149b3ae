"""GPU job target of the kernel evaluator: the Kubernetes Job that runs the
CUDA evaluator (`python -m glaucis_b200.evaluate`) on one B200.

Mirrors the job half of KE/src/kernel_evolve/kube_evaluator.py: the job name
rule of `_make_job_name` (:33-37), the placeholder mapping of
`_render_job_yaml` (:39-49) and `_render_batch_job_yaml` (:229-239, deadline
300 s per variant + 300 s), and the payload ConfigMap of `_create_configmap`
(:62-95, name `<job>-payload`, key `payload`).  Submission, polling, log and
artifact collection stay with the caller (the reference's KubeEvaluator can
use the template as its `job_template` unchanged: it only needs the five
placeholders the reference fills).
"""
from __future__ import annotations

import re
import string
from dataclasses import dataclass
from pathlib import Path

DEFAULT_TEMPLATE = Path(__file__).with_name("kube") / "kernel-eval-b200-job.yaml"


@dataclass
class JobTarget:
    namespace: str = "default"
    job_template: str = str(DEFAULT_TEMPLATE)
    repo: str = ""
    branch: str = "main"


def make_job_name(variant_id: str) -> str:
    """`kernel-eval-<variant>`: lower case, [a-z0-9-] only, at most 63 characters."""
    safe_id = re.sub(r"[^a-z0-9-]", "-", variant_id.lower())
    safe_id = re.sub(r"-+", "-", safe_id).strip("-")
    return f"kernel-eval-{safe_id}"[:63].rstrip("-")


def _render(target: JobTarget, mapping: dict) -> str:
    return string.Template(Path(target.job_template).read_text()).safe_substitute(mapping)


def render_job_yaml(target: JobTarget, job_name: str, variant_id: str,
                    active_deadline: int = 600) -> str:
    """The Job for one variant."""
    return _render(target, {"JOB_NAME": job_name, "BRANCH": target.branch, "REPO": target.repo,
                            "VARIANT_ID": variant_id, "ACTIVE_DEADLINE": str(active_deadline)})


def render_batch_job_yaml(target: JobTarget, job_name: str, n_variants: int) -> str:
    """The Job for a batch of variants (one pod, the evaluator's batch mode)."""
    return _render(target, {"JOB_NAME": job_name, "BRANCH": target.branch, "REPO": target.repo,
                            "VARIANT_ID": f"batch-{n_variants}",
                            "ACTIVE_DEADLINE": str(300 * n_variants + 300)})


def render_payload_configmap(target: JobTarget, job_name: str, payload_b64: str) -> str:
    """The ConfigMap the Job mounts at /etc/eval-payload (key `payload`)."""
    return "\n".join([
        "apiVersion: v1",
        "kind: ConfigMap",
        "metadata:",
        f"  name: {job_name}-payload",
        f"  namespace: {target.namespace}",
        "  labels:",
        "    app: kernel-eval",
        "data:",
        f"  payload: {payload_b64}",
        "",
    ])
