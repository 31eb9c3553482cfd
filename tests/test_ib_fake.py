"""The ibverbs fabric on CPU, against tests/native/fake_ibverbs.cc."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "tests", "native", "bin", "libfake_ibverbs.so")


def _run(extra, args=()):
    assert os.path.exists(LIB), "fake provider not built (run __graft_entry__.build())"
    env = dict(os.environ, MPCOMM_FABRIC="ib", MPCOMM_IBVERBS_LIB=LIB, MPCOMM_GID_INDEX="-1",
               MPCOMM_LOG_LEVEL="1", PYTHONPATH=ROOT, **extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "ib_fake_case.py"), *args],
                       capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0 and "ib fake ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
    return r


def test_ib_fabric_put_get_scatter():
    _run({})


@pytest.mark.parametrize("vendor,ports", [("mlx5", ""), ("bnxt_re", "60000,60051,57663,57804")])
def test_ib_udp_source_port_per_vendor(vendor, ports):
    """RTS sets each QP's RoCE UDP source port through the device vendor's
    direct-verbs call (mlx5dv or bnxt_re_dv): spread over the dynamic port
    range by default, or cycled through MPCOMM_UDP_SPORTS."""
    extra = {"MPCOMM_IBV_DV_LIB": LIB, "EXPECT_SPORT_VENDOR": vendor}
    if vendor == "bnxt_re":
        extra["FAKE_IBV_DEVICE_PREFIX"] = "bnxt_re"
    if ports:
        extra["MPCOMM_UDP_SPORTS"] = ports
    r = _run(extra)
    assert "sport calls" in r.stdout


@pytest.mark.parametrize("mode", ["single_qp", "all_qp"])
def test_ib_fault_injection_reposts_on_healthy_rail(mode):
    r = _run({"MPCOMM_FAULT_INJECT_AFTER_SEC": "0", "MPCOMM_FAULT_INJECT_NIC": "0",
              "MPCOMM_FAULT_INJECT_MODE": mode, "MPCOMM_MAX_RDMA_TRANSFER_SIZE": "65536"})
    import re

    moved = [int(x) for x in re.findall(r"fault injection \(\w+\) moved (\d+) QPs to ERR", r.stderr)]
    assert moved and max(moved) > 0, r.stderr[-2000:]
    assert "quarantined" in r.stderr


@pytest.mark.gpu
def test_ib_gpudirect_dmabuf_registration_of_hbm():
    """HBM buffers on the ib fabric are registered through dma-buf
    (cuMemGetHandleForAddressRange on the B200, ibv_reg_dmabuf_mr on every
    NIC) and PUT/GET between them round-trip bit-exact."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    r = _run({}, ["--gpu"])
    if "dma_buf_supported=1 export_rc=0)" in r.stdout:
        assert "dma-buf registrations: 6" in r.stdout, r.stdout[-2000:]
    else:
        # The driver of this machine exports no dma-buf: registration fell
        # back to ibv_reg_mr of the device range and the HBM transfers
        # still completed bit-exact; report why the dma-buf path was idle.
        print(r.stdout[-500:])
