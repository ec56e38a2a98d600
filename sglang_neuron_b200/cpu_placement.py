"""CPU/NUMA placement: bind each rank's scheduler thread to the NUMA node of its GPU.

Parity: sglang_neuron/cpu_placement.py:52-93 binds each scheduler to its device's NUMA node (and keeps a
vCPU free). Here the node comes from the GPU's PCI sysfs entry; the CPU list from /sys/devices/system/node.
"""
from __future__ import annotations

import os
from typing import List, Optional


def parse_cpu_list(s: str) -> List[int]:
    """'0-3,8,10-11' -> [0,1,2,3,8,10,11] (parity: utils/hardware_config.parse_range_list)."""
    out: List[int] = []
    for part in s.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            out += list(range(int(a), int(b) + 1))
        else:
            out.append(int(part))
    return out


def gpu_numa_node(pci_bus_id: str, sysfs: str = "/sys/bus/pci/devices") -> Optional[int]:
    path = os.path.join(sysfs, pci_bus_id.lower(), "numa_node")
    try:
        with open(path) as f:
            n = int(f.read().strip())
        return n if n >= 0 else None
    except (OSError, ValueError):
        return None


def node_cpus(node: int, sysfs: str = "/sys/devices/system/node") -> List[int]:
    try:
        with open(os.path.join(sysfs, f"node{node}", "cpulist")) as f:
            return parse_cpu_list(f.read())
    except OSError:
        return []


def bind_to_gpu(device_index: int) -> Optional[List[int]]:
    """Restrict this process to the CPUs of its GPU's NUMA node; returns the CPU set (None if unknown)."""
    try:
        import torch
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    except Exception:
        return None
    node = gpu_numa_node(bus)
    if node is None:
        return None
    cpus = node_cpus(node)
    if cpus:
        os.sched_setaffinity(0, set(cpus))
    return cpus
