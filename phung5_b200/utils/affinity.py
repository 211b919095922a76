"""CPU sets for CPU-heavy worker pools (candidate checking, CPU rendering).

Reference: docker/opt/raff/aff_list.py:1-96 and node_aff.sh:1-13 confine the render sidecars to R = floor(cgroup
CPU quota) - reserve CPUs, one hardware thread per physical core first, highest-numbered cores first (away from
CPU 0 housekeeping), so the engines' schedulers and the API server keep the remaining cores.

`worker_cpus()` computes that list from cgroup v2 `cpu.max` (v1 `cpu.cfs_quota_us` fallback), the process's
allowed CPUs and `/sys/devices/system/cpu/cpu*/topology/thread_siblings_list`; it returns None (do not pin)
when the quota cannot be read, when fewer than `min_cpus` would remain, or when pinning would not confine
anything. `pin_current_process(cpus)` applies it (used as a worker-pool initializer).
"""
from __future__ import annotations

import math
import os
from typing import Dict, List, Optional


def read_quota(cgroup_root: str = "/sys/fs/cgroup") -> Optional[float]:
    """CPUs allowed by the quota; math.inf when unlimited; None when unreadable."""
    try:
        with open(os.path.join(cgroup_root, "cpu.max")) as f:
            q, per = f.read().split()[:2]
        return math.inf if q == "max" else float(q) / float(per)
    except (OSError, ValueError):
        pass
    for d in ("cpu", "cpu,cpuacct", "cpuacct,cpu", "."):
        fq = os.path.join(cgroup_root, d, "cpu.cfs_quota_us")
        fp = os.path.join(cgroup_root, d, "cpu.cfs_period_us")
        if os.path.exists(fq):
            try:
                q = float(open(fq).read())
                if q < 0:
                    return math.inf
                return q / float(open(fp).read())
            except (OSError, ValueError):
                return None
    return None


def core_groups(allowed: List[int], sys_root: str = "/sys/devices/system/cpu") -> List[List[int]]:
    """Allowed CPUs grouped by physical core (hardware-thread siblings), cores sorted by their lowest CPU."""
    seen: Dict[int, List[int]] = {}
    for c in allowed:
        path = os.path.join(sys_root, f"cpu{c}", "topology", "thread_siblings_list")
        sib = [c]
        try:
            txt = open(path).read().strip()
            sib = []
            for part in txt.split(","):
                if "-" in part:
                    a, b = part.split("-")
                    sib += list(range(int(a), int(b) + 1))
                else:
                    sib.append(int(part))
        except (OSError, ValueError):
            pass
        key = min(sib)
        seen.setdefault(key, [])
        if c not in seen[key]:
            seen[key].append(c)
    return [sorted(v) for _, v in sorted(seen.items())]


def worker_cpus(reserve: int = 14, min_cpus: int = 8, cgroup_root: str = "/sys/fs/cgroup",
                allowed: Optional[List[int]] = None, sys_root: str = "/sys/devices/system/cpu") -> Optional[List[int]]:
    allowed = sorted(os.sched_getaffinity(0) if allowed is None else allowed)
    if not allowed:
        return None
    q = read_quota(cgroup_root)
    if q is None:
        return None
    total = len(allowed) if q == math.inf else min(len(allowed), int(math.floor(q)))
    r = total - reserve
    if r < min_cpus or r >= len(allowed):
        return None
    cores = core_groups(allowed, sys_root)[::-1]            # highest-numbered cores first
    picked = [c[0] for c in cores][:r]                      # one thread per physical core
    if len(picked) < r:                                     # then siblings
        extra = [x for c in cores for x in c[1:]]
        picked += extra[: r - len(picked)]
    return sorted(picked)


def pin_current_process(cpus: Optional[List[int]]) -> bool:
    if not cpus:
        return False
    try:
        os.sched_setaffinity(0, set(cpus))
        return True
    except OSError:
        return False
