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
