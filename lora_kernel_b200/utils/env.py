"""Environment report: versions, GPU capabilities, NVLink topology, extension
status (the reference's CompilationValidator::print_report,
include/core/compilation_validator.hpp:8-24, checked AVX2/OpenMP/OpenSSL)."""
from __future__ import annotations

import os
import subprocess


def env_report() -> dict:
    import torch
    r = {"torch": torch.__version__, "cuda_runtime": torch.version.cuda,
         "cuda_available": torch.cuda.is_available()}
    try:
        r["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
    except Exception:
        r["nccl"] = None
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        r.update(gpu=p.name, sm_count=p.multi_processor_count, capability=f"{p.major}.{p.minor}",
                 memory_gb=round(p.total_memory / 2 ** 30, 1), device_count=torch.cuda.device_count(),
                 sm100a=(p.major == 10))
        try:
            r["nvlink_topology"] = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True,
                                                  text=True, timeout=20).stdout
        except Exception:
            r["nvlink_topology"] = None
    from .._ext import available
    r["extension_built"] = available()
    r["nvls_env"] = os.environ.get("NCCL_NVLS_ENABLE")
    return r


def parse_cpulist(text: str) -> set:
    """'0-3,8,10-11' -> {0, 1, 2, 3, 8, 10, 11} (the sysfs cpulist format)."""
    cpus = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def gpu_numa_cpus(pci_bus_id: str, sysfs: str = "/sys") -> set:
    """CPUs of the NUMA node a PCI device (e.g. '0000:1B:00.0') is attached to;
    empty when the platform reports no node."""
    bus = pci_bus_id.lower()
    if bus.count(":") == 1:  # nvidia-smi style '00000000:1B:00.0' has 8 domain digits; sysfs wants 4
        bus = "0000:" + bus
    dom, rest = bus.split(":", 1)
    bus = dom[-4:] + ":" + rest
    try:
        with open(os.path.join(sysfs, "bus", "pci", "devices", bus, "numa_node")) as f:
            node = int(f.read().strip())
        if node < 0:
            return set()
        with open(os.path.join(sysfs, "devices", "system", "node", f"node{node}", "cpulist")) as f:
            return parse_cpulist(f.read())
    except (OSError, ValueError):
        return set()


def pin_to_gpu_numa(device_index: int, sysfs: str = "/sys") -> set:
    """Restrict this process to the CPUs of its GPU's NUMA node (the launcher-side
    counterpart of the reference's NUMA binding).  Reads the bus id through NVML;
    returns the CPU set applied (empty: nothing changed)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
        bus = pynvml.nvmlDeviceGetPciInfo(h).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
    except Exception:  # noqa: BLE001 - no NVML: leave the affinity alone
        return set()
    cpus = gpu_numa_cpus(bus, sysfs) & set(os.sched_getaffinity(0))
    if cpus:
        os.sched_setaffinity(0, cpus)
    return cpus
