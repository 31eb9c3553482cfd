"""Multi-GPU cases (cross-process NVLink PUT/GET, PXN forward, NVLS) under
torch.distributed.run; skipped on hosts with fewer than 2 GPUs."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", ["putget", "pxn", "nvls"])
def test_multigpu_case(case):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs >= 2 GPUs")
    n = min(n, 8)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(ROOT, "tests", "mp_cases.py"), case]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MPCOMM_LOG_LEVEL="1")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, f"{case} failed:\n{r.stdout[-4000:]}\n{r.stderr[-4000:]}"
    assert f"case {case} ok" in r.stdout
