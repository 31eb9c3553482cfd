"""hosts.txt and jobs.txt parsing.

hosts.txt — one host per line, ``ID IP [PORT] [NUMAS]`` ('-' or missing
fields take 12345 and "0"); '#' starts a comment. The first host is the
initiator of a multi-node run, the others are its targets. IDs are labels:
one that looks like an IPv4 address is rejected (the old IP-first format).

jobs.txt — INI-style sections for multi-initiator runs:
    [global]         defaults inherited by every job (size, iterations, ...)
    [jobs order]     optional job order (comma/space separated)
    [<job>]          initiator = HOST (exactly one), target = HOST [HOST ...]
                     (repeatable), optional size / iterations / warmup /
                     batch-size / gpu / test-type / buffer-size
HOST is ``ID`` or ``ID[NUMA]`` (NUMA may be a comma list: ``3[0,1]``).

Format parity: reference deploy/common.sh:120-190 (hosts.txt) and
deploy/jobs.txt.example (jobs.txt).
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Dict, List, Optional

DEFAULT_PORT = 12345
DEFAULT_NUMAS = "0"
JOB_KEYS = {"size", "iterations", "warmup", "batch-size", "gpu", "test-type", "buffer-size", "both"}
_IPV4 = re.compile(r"^\d+\.\d+\.\d+\.\d+$")
_HOST_REF = re.compile(r"^([^\[\]\s]+)(?:\[([0-9,\s]+)\])?$")


class HostsError(ValueError):
    pass


@dataclass
class Host:
    id: str
    ip: str
    port: int = DEFAULT_PORT
    numas: str = DEFAULT_NUMAS


@dataclass
class HostRef:
    host: Host
    numas: str  # the role's NUMA spec (override or the host default)


@dataclass
class Job:
    name: str
    initiator: HostRef
    targets: List[HostRef]
    params: Dict[str, str] = field(default_factory=dict)


def _strip(line: str) -> str:
    return line.rstrip("\r\n").split("#", 1)[0].strip()


def parse_hosts(text: str, where: str = "hosts.txt") -> List[Host]:
    hosts: List[Host] = []
    seen = set()
    for no, raw in enumerate(text.splitlines(), 1):
        line = _strip(raw)
        if not line:
            continue
        parts = line.split()
        if len(parts) < 2:
            raise HostsError(f"{where}:{no}: expected 'ID IP [PORT] [NUMAS]', got: {line}")
        hid, ip = parts[0], parts[1]
        if _IPV4.match(hid):
            raise HostsError(f"{where}:{no}: first column must be a host ID (label), not an IP "
                             f"(format: ID IP PORT NUMAS, e.g. '1 10.0.0.1 12345 0')")
        if hid in seen:
            raise HostsError(f"{where}:{no}: duplicate host ID '{hid}'")
        port = parts[2] if len(parts) > 2 and parts[2] != "-" else str(DEFAULT_PORT)
        numas = parts[3] if len(parts) > 3 and parts[3] != "-" else DEFAULT_NUMAS
        try:
            port_i = int(port)
        except ValueError:
            raise HostsError(f"{where}:{no}: bad port '{port}'") from None
        if not re.match(r"^[0-9]+(,[0-9]+)*$", numas):
            raise HostsError(f"{where}:{no}: bad NUMA list '{numas}'")
        seen.add(hid)
        hosts.append(Host(hid, ip, port_i, numas))
    if len(hosts) < 2:
        raise HostsError(f"{where}: need at least 2 hosts (1 initiator + 1 target)")
    return hosts


def load_hosts(path: str) -> List[Host]:
    with open(path) as f:
        return parse_hosts(f.read(), path)


def _ref(token: str, by_id: Dict[str, Host], where: str) -> HostRef:
    m = _HOST_REF.match(token.strip())
    if not m:
        raise HostsError(f"{where}: bad host reference '{token}' (use ID or ID[NUMA])")
    hid, numas = m.group(1), m.group(2)
    if hid not in by_id:
        raise HostsError(f"{where}: host '{hid}' is not in hosts.txt")
    h = by_id[hid]
    return HostRef(h, numas.replace(" ", "") if numas else h.numas)


def parse_jobs(text: str, hosts: List[Host], where: str = "jobs.txt") -> List[Job]:
    by_id = {h.id: h for h in hosts}
    sections: Dict[str, List[tuple]] = {}
    order_names: List[str] = []
    current: Optional[str] = None
    for no, raw in enumerate(text.splitlines(), 1):
        line = _strip(raw)
        if not line:
            continue
        if line.startswith("[") and line.endswith("]"):
            current = line[1:-1].strip()
            if current in sections:
                raise HostsError(f"{where}:{no}: duplicate section [{current}]")
            sections[current] = []
            if current not in ("global", "jobs order"):
                order_names.append(current)
            continue
        if current is None:
            raise HostsError(f"{where}:{no}: entry outside a section: {line}")
        if current == "jobs order":
            sections[current].append(("order", line, no))
            continue
        if "=" not in line:
            raise HostsError(f"{where}:{no}: expected key = value, got: {line}")
        k, v = (x.strip() for x in line.split("=", 1))
        sections[current].append((k.lower(), v, no))
    glob = {}
    for k, v, no in sections.get("global", []):
        if k not in JOB_KEYS:
            raise HostsError(f"{where}:{no}: unknown [global] key '{k}'")
        glob[k] = v
    if "jobs order" in sections:
        order = [n for _, v, _ in sections["jobs order"] for n in re.split(r"[,\s]+", v) if n]
        unknown = [n for n in order if n not in order_names]
        if unknown:
            raise HostsError(f"{where}: [jobs order] names unknown job(s) {unknown}")
        order += [n for n in order_names if n not in order]
    else:
        order = order_names
    jobs: List[Job] = []
    initiators = {}
    for name in order:
        ini, tgts, params = None, [], dict(glob)
        for k, v, no in sections[name]:
            at = f"{where}:{no}"
            if k == "initiator":
                if ini is not None:
                    raise HostsError(f"{at}: job [{name}] has more than one initiator")
                ini = _ref(v, by_id, at)
            elif k == "target":
                tgts += [_ref(t, by_id, at) for t in v.split()]
            elif k in JOB_KEYS:
                params[k] = v
            else:
                raise HostsError(f"{at}: unknown key '{k}' in job [{name}]")
        if ini is None or not tgts:
            raise HostsError(f"{where}: job [{name}] needs one initiator and at least one target")
        if ini.host.id in initiators:
            raise HostsError(f"{where}: host '{ini.host.id}' initiates both [{initiators[ini.host.id]}] and "
                             f"[{name}] (one process per host)")
        if any(t.host.id == ini.host.id for t in tgts):
            raise HostsError(f"{where}: job [{name}] targets its own initiator '{ini.host.id}'")
        initiators[ini.host.id] = name
        jobs.append(Job(name, ini, tgts, params))
    if not jobs:
        raise HostsError(f"{where}: no jobs")
    return jobs


def load_jobs(path: str, hosts: List[Host]) -> List[Job]:
    with open(path) as f:
        return parse_jobs(f.read(), hosts, path)
