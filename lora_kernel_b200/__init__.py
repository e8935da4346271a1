"""lora_kernel_b200: a Blackwell (B200, sm_100a) native LLM training and
inference framework with the capabilities of sudish80/Lora-Kernel-."""
from .config import (ModelConfig, ParallelConfig, QuantConfig, RunConfig, ServeConfig,  # noqa: F401
                     TrainConfig, TransformerConfig, get_preset, load_config)

__version__ = "0.1.0"
