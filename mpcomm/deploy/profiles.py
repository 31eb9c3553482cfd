"""Named sets of MPCOMM_* environment variables for benchmark runs.

    stage0     64 KiB chunks, 4 QPs, 8 outstanding (2 MB in-flight ceiling),
               PCIe-domain statistics on — the QoS-friendly RDMA setting
    legacy     1 GiB chunks, 1 QP, 256 outstanding (no in-flight ceiling)
    multinode  the multi-node bench defaults: 4 QPs, 64 KiB chunks, 16
               outstanding, poll interval 16, 128 send WRs
    pxn        NVLink proxy rails on, 2 MiB chunks, 1 outstanding per QP
    b200-qos   GPU fabric tuned for H2D QoS: 2 MiB chunks, 2 QPs x 2
               outstanding, PCIe-domain statistics on

Values of stage0 / legacy / multinode / pxn are the reference's
(user_examples/qos_bench/env_stage0.sh, env_legacy.sh,
deploy/multi_node_test.sh:50-66); b200-qos is this library's.
"""
from __future__ import annotations

import os
import shlex
from typing import Dict, Iterable, Optional

PROFILES: Dict[str, Dict[str, str]] = {
    "stage0": {"MPCOMM_MAX_RDMA_TRANSFER_SIZE": "65536", "MPCOMM_QPS_PER_CONNECTION": "4",
               "MPCOMM_MAX_OUTSTANDING_PER_QP": "8", "MPCOMM_PCIE_STAT_ENABLE": "1"},
    "legacy": {"MPCOMM_MAX_RDMA_TRANSFER_SIZE": "1073741824", "MPCOMM_QPS_PER_CONNECTION": "1",
               "MPCOMM_MAX_OUTSTANDING_PER_QP": "256"},
    "multinode": {"MPCOMM_QPS_PER_CONNECTION": "4", "MPCOMM_POLL_INTERVAL": "16", "MPCOMM_MAX_SEND_WR": "128",
                  "MPCOMM_MAX_RDMA_TRANSFER_SIZE": "65536", "MPCOMM_MAX_OUTSTANDING_PER_QP": "16",
                  "MPCOMM_PXN_ENABLE": "0"},
    "pxn": {"MPCOMM_PXN_ENABLE": "1", "MPCOMM_MAX_RDMA_TRANSFER_SIZE": "2097152",
            "MPCOMM_MAX_OUTSTANDING_PER_QP": "1"},
    "b200-qos": {"MPCOMM_NVL_CHUNK_SIZE": "2097152", "MPCOMM_NVL_OUTSTANDING_PER_QP": "2",
                 "MPCOMM_QPS_PER_CONNECTION": "2", "MPCOMM_PCIE_STAT_ENABLE": "1"},
}

# Variables forwarded from the caller's environment to every host when set.
PASSTHROUGH = ("MPCOMM_FABRIC", "MPCOMM_NIC_FILTER", "MPCOMM_GID_INDEX", "MPCOMM_LOG_LEVEL", "MPCOMM_QPS_PER_CONNECTION",
               "MPCOMM_MAX_RDMA_TRANSFER_SIZE", "MPCOMM_MAX_OUTSTANDING_PER_QP", "MPCOMM_PXN_ENABLE",
               "MPCOMM_NVL_CHUNK_SIZE", "MPCOMM_NVL_OUTSTANDING_PER_QP", "MPCOMM_NVL_CTAS_PER_QP",
               "MPCOMM_PCIE_STAT_ENABLE", "MPCOMM_CTRL_TIMEOUT_MS", "PYTHONPATH", "LD_LIBRARY_PATH")


def profile_env(name: Optional[str], overrides: Iterable[str] = (), environ=None) -> Dict[str, str]:
    """Environment for a run: caller's MPCOMM_* passthrough, then the
    profile, then KEY=VALUE overrides (later wins)."""
    environ = os.environ if environ is None else environ
    env = {k: environ[k] for k in PASSTHROUGH if k in environ}
    if name:
        if name not in PROFILES:
            raise KeyError(f"unknown profile '{name}' (have: {', '.join(sorted(PROFILES))})")
        env.update(PROFILES[name])
    for kv in overrides:
        k, sep, v = kv.partition("=")
        if not sep or not k:
            raise ValueError(f"bad override '{kv}' (want KEY=VALUE)")
        env[k] = v
    return env


def exports(env: Dict[str, str]) -> str:
    """`export K=V; ...` shell prefix."""
    return "".join(f"export {k}={shlex.quote(v)}; " for k, v in sorted(env.items()))
