"""Multi-GPU (NCCL) checks; skipped on boxes with fewer GPUs than a case needs."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
NGPU = torch.cuda.device_count() if torch.cuda.is_available() else 0


def _torchrun(n, args, timeout=600):
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"))
    cmd = ["timeout", "-k", "30", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={29700 + n}"] + args
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)


@pytest.mark.parametrize("tp,sp1,sp2", [(1, 1, 2), (2, 1, 1), (1, 2, 1), (1, 1, 1)])
def test_sharded_model_on_two_gpus(tp, sp1, sp2):
    if NGPU < 2:
        pytest.skip("needs 2 GPUs")
    r = _torchrun(2, ["tests/mp_gpu_worker.py", str(tp), str(sp1), str(sp2)])
    assert "MULTIGPU_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_bench_two_gpus_small():
    if NGPU < 2:
        pytest.skip("needs 2 GPUs")
    r = _torchrun(2, ["bench.py", "--gpus", "2", "--steps", "1", "--warmup", "1", "--depth", "2", "--no-e2e",
                      "--no-rollout"])
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert lines, r.stdout[-3000:] + r.stderr[-3000:]
    d = json.loads(lines[-1])
    assert d["n_gpus"] == 2 and d["value"] > 0


def test_fused_gemm_allreduce_two_gpus():
    """Tensor-parallel GEMM with the all-reduce in its epilogue over NVLink peer memory."""
    if NGPU < 2:
        pytest.skip("needs 2 GPUs")
    r = _torchrun(2, ["tests/mp_fused_tp_worker.py"])
    assert "FUSED_TP_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_fused_dp_matches_nccl_two_gpus():
    """Data-parallel gradient reduction over peer memory + sharded AdamW that stores the new parameters
    into every rank, against the NCCL all-reduce and the full AdamW (parameters, norms, losses, moments)."""
    if NGPU < 2:
        pytest.skip("needs 2 GPUs")
    r = _torchrun(2, ["tests/mp_dp_fused_worker.py"])
    assert "DP_FUSED_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("n", [2, 4])
def test_fused_halo_roll_matches_torch_roll(n):
    """Sharded shifted-window roll over peer memory against torch.roll of the gathered field (sp1, sp2 and,
    on 4 GPUs, 2 x 2 layouts; graph replay; the reverse roll of the backward); prints its timing against the
    NCCL roll."""
    if NGPU < n:
        pytest.skip(f"needs {n} GPUs")
    r = _torchrun(n, ["tests/mp_halo_worker.py"])
    print("\n".join(l for l in r.stdout.splitlines() if l.startswith("roll of")))
    assert "HALO_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
