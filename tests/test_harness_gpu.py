"""Target/initiator harness on the GPU fabric: HBM initiator against an HBM
target and a host-DRAM target (separate processes, CUDA IPC / pinned host
memory), every mode verified; a performance run reports JSON."""
import json

import pytest
import torch

from harness_util import TargetProc, harness_env, run_initiator

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("target_mem", ["hbm", "dram"])
def test_harness_gpu_fabric(tmp_path, target_mem):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    env = harness_env(MPCOMM_FABRIC="nvl")
    extra = ["--gpu", "0"] if target_mem == "hbm" else []
    t = TargetProc(tmp_path, "127.0.0.1:0", env, "--buffer-size", "64M", *extra)
    try:
        spec = f"127.0.0.1:127.0.0.1:{t.port}"
        r = run_initiator(env, "--targets", spec, "--mode", "all", "--gpu", "0", "--iterations", "2",
                          "--batch-size", "2", "--max-chunk-size", str(4 << 20))
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        assert "fabric=nvl" in r.stdout and "[initiator] all tests passed" in r.stdout
        r = run_initiator(env, "--targets", spec, "--mode", "put", "--gpu", "0", "--test-mode", "performance",
                          "--iterations", "3", "--warmup", "1", "--batch-size", "4", "--min-chunk-size",
                          str(8 << 20), "--max-chunk-size", str(8 << 20), "--json")
        assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
        assert json.loads(r.stdout.strip().splitlines()[-1])["results"]["put"]["gbps"] > 1.0
    finally:
        assert t.stop() == 0
