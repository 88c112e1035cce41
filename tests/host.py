"""Host CPU sizing for the test and benchmark harness.

``os.cpu_count()`` reports every core of the machine; a container may be
confined to far fewer by its affinity mask or its cgroup CPU quota.  Letting
torch and BLAS start one thread per reported core on a small quota makes every
CPU op crawl, so the harness sizes its thread pools with ``usable_cpus()``.
"""

from __future__ import annotations

import math
import os
from pathlib import Path


def usable_cpus() -> int:
    count = os.cpu_count() or 1
    try:
        count = min(count, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        pass
    quota = Path("/sys/fs/cgroup/cpu.max")
    try:
        fields = quota.read_text().split()
        if fields and fields[0] != "max":
            count = min(count, max(1, math.floor(int(fields[0]) / int(fields[1]))))
    except (OSError, ValueError, IndexError):
        pass
    return max(1, count)


def limit_threads(threads: int | None = None) -> int:
    """Size torch's and the BLAS libraries' pools to ``threads`` (default: usable CPUs)."""
    threads = threads or usable_cpus()
    import torch
    torch.set_num_threads(threads)
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(threads)
    except ImportError:
        pass
    return threads


def cpu_model_name() -> str:
    """The host CPU's model string (``/proc/cpuinfo``), or the platform's."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or platform.machine()
