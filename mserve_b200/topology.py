"""Host-memory placement for the GPU a process drives.

Each GPU gathers its selected KV rows over its own PCIe link.  The host store it reads
should sit on the NUMA node that link attaches to, or every row crosses the inter-socket link
as well.  Pinned pages are placed on the node of the CPU that allocates them (the default
local policy), so allocating the host store while the calling thread runs only on the GPU's
local CPUs puts it on the right node.  The CPUs come from the PCI device's sysfs entry
(/sys/bus/pci/devices/<domain:bus:device.function>/local_cpulist).  Where that entry is not
visible (containers without sysfs), placement is left to the system.
"""
from __future__ import annotations

import contextlib
import os
from typing import Optional, Set

import torch


def parse_cpulist(text: str) -> Set[int]:
    """CPU numbers of a sysfs cpulist such as "0-15,32-47"."""
    cpus: Set[int] = set()
    for part in text.strip().split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            lo, hi = part.split("-", 1)
            cpus.update(range(int(lo), int(hi) + 1))
        else:
            cpus.add(int(part))
    return cpus


def pci_path(device: torch.device) -> Optional[str]:
    """sysfs directory of the GPU's PCI function, or None when it is not visible."""
    p = torch.cuda.get_device_properties(device)
    bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    path = os.path.join("/sys/bus/pci/devices", bdf)
    return path if os.path.isdir(path) else None


def local_cpus(device: torch.device) -> Set[int]:
    """CPUs local to the GPU's PCIe attachment (empty when unknown)."""
    path = pci_path(device)
    if path is None:
        return set()
    try:
        with open(os.path.join(path, "local_cpulist")) as f:
            return parse_cpulist(f.read())
    except (OSError, ValueError):
        return set()


def numa_node(device: torch.device) -> int:
    """NUMA node of the GPU's PCIe attachment (-1 when unknown)."""
    path = pci_path(device)
    if path is None:
        return -1
    try:
        with open(os.path.join(path, "numa_node")) as f:
            return int(f.read().strip())
    except (OSError, ValueError):
        return -1


@contextlib.contextmanager
def local_placement(device: torch.device):
    """Runs the body on the GPU's local CPUs (those this thread may use), then restores the
    thread's CPU set.  Host memory allocated inside lands on the GPU's NUMA node; its pages
    stay there afterwards.  Yields the CPUs used (empty: placement unchanged)."""
    before = os.sched_getaffinity(0)
    cpus = local_cpus(device) & before
    if cpus and cpus != before:
        os.sched_setaffinity(0, cpus)
        try:
            yield cpus
        finally:
            os.sched_setaffinity(0, before)
    else:
        yield set()
