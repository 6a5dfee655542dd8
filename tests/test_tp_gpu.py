"""Tensor parallel end-to-end on 2+ GPUs (NCCL baseline and fused NVLink paths)."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(n, mode, graphs="graphs", model="tiny-tp", port=29611, extra_env=None):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"),
               TORCH_SYMM_MEM_DISABLE_MULTICAST="1", **(extra_env or {}))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "tp_worker.py"), mode, graphs, model]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(lines[-1])
    assert res["ok"] and res["ranks_agree"] and res["status"] == 0, res
    assert res["bad_guard_words"] == 0, res
    return res


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tp_nccl(n):
    _run(n, "nccl", port=29611 + n)


@pytest.mark.parametrize("n", [2, 8])
def test_tp_nccl_eager(n):
    _run(n, "nccl", graphs="eager", port=29631 + n)


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tp_fused(n):
    res = _run(n, "fused", port=29651 + n)
    assert {"partial", "x", "flags", "logit_pairs", "logit_rows"} <= set(res["guards_checked"]), res


@pytest.mark.parametrize("n", [2, 8])
def test_tp_fused_eager(n):
    _run(n, "fused", graphs="eager", port=29671 + n)


@pytest.mark.parametrize("n", [2, 8])
def test_ep_moe_fused(n):
    _run(n, "fused", model="tiny-moe-tp", port=29691 + n)


@pytest.mark.parametrize("n", [2])
def test_tp_fused_pull_variant(n):
    """Row-parallel GEMMs write locally and the collective pulls (BLOOM_TP_PUSH=0)."""
    _run(n, "fused", port=29711 + n, extra_env={"BLOOM_TP_PUSH": "0"})
