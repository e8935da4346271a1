"""Configuration dataclasses, named presets and YAML/JSON/CLI loading.

`TransformerConfig` keeps the reference's field names (hidden_dim, num_heads,
head_dim, vocab_size, max_seq_len, num_layers, dropout, ff_dim;
include/nn/transformer_blocks.hpp:11-20) and adds what a Llama decoder needs:
num_kv_heads (GQA), rope_base, norm_eps, tie_embeddings, init_std.

Presets cover the five workloads this framework is measured on: the CPU train
demo (4 layers, d 256), Llama 1.1B ZeRO-3 training, Llama 8B TP=8 fp8
training, Llama 8B FSDP + DP with accumulation and EMA, and Llama 8B TP=8
int4 serving.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field, fields
from typing import Any, Dict, Optional


@dataclass
class TransformerConfig:
    hidden_dim: int = 256
    num_heads: int = 4
    head_dim: int = 64
    vocab_size: int = 1024
    max_seq_len: int = 128
    num_layers: int = 4
    dropout: float = 0.0
    ff_dim: int = 688
    num_kv_heads: int = 0  # 0 = same as num_heads (MHA)
    rope_base: float = 10000.0
    norm_eps: float = 1e-5
    tie_embeddings: bool = False
    init_std: float = 0.02
    # LM head + cross-entropy in vocabulary chunks of this many columns, never
    # materialising the [tokens, vocab] logits: 0 = chunks of 8192 when the
    # logits would take more than 1 GiB, -1 = never
    ce_vocab_chunk: int = 0
    # stochastic depth (training): layer l (0-based) of L skips its attention and
    # FFN branches with probability (l + 1) / L * stochastic_depth; a kept
    # layer's branch outputs are scaled by 1 / (keep probability)
    stochastic_depth: float = 0.0

    def __post_init__(self):
        if self.num_kv_heads <= 0:
            self.num_kv_heads = self.num_heads
        if self.num_heads % self.num_kv_heads != 0:
            raise ValueError("num_heads must be a multiple of num_kv_heads")

    @property
    def q_dim(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_dim(self) -> int:
        return self.q_dim + 2 * self.kv_dim

    @property
    def ff_dim_padded(self) -> int:
        """FFN width rounded up to 128 (the gate|up GEMM tile); padding is exact
        (zero rows/columns stay zero under SwiGLU, its gradients and AdamW)."""
        return ((self.ff_dim + 127) // 128) * 128

    def num_parameters(self) -> int:
        d, v = self.hidden_dim, self.vocab_size
        per_layer = (d * self.qkv_dim + self.q_dim * d + 3 * d * self.ff_dim + 2 * d)
        head = 0 if self.tie_embeddings else v * d
        return v * d + self.num_layers * per_layer + d + head

    def flops_per_token(self, seq_len: int) -> float:
        """Training FLOPs per token: 6 x matmul parameters (blocks + LM head)
        plus causal attention (QK^T and PV, forward + 2x backward)."""
        d = self.hidden_dim
        n_matmul = self.num_layers * (d * self.qkv_dim + self.q_dim * d + 3 * d * self.ff_dim)
        n_matmul += self.vocab_size * d
        attn = 6.0 * self.num_layers * self.q_dim * seq_len
        return 6.0 * n_matmul + attn


ModelConfig = TransformerConfig


@dataclass
class TrainConfig:
    lr: float = 3e-4
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    eps: float = 1e-8
    max_grad_norm: float = 1.0
    warmup_steps: int = 0
    total_steps: int = 50
    schedule: str = "constant"  # constant|linear_warmup|cosine|cosine_restarts|polynomial
    min_lr_ratio: float = 0.1
    grad_accum_steps: int = 1
    micro_batch: int = 8
    seq_len: int = 128
    dynamic_loss_scale: bool = True
    init_loss_scale: float = 65536.0
    loss_scale_growth_interval: int = 2000
    ema_decay: float = 0.0  # 0 = off
    swa_start: int = -1  # -1 = off
    grad_noise_eta: float = 0.0  # > 0: gradient noise N(0, eta / (1 + step)^gamma) before the optimizer
    grad_noise_gamma: float = 0.55
    label_smoothing: float = 0.0
    z_loss: float = 0.0
    decay_norms: bool = False
    seed: int = 1234
    lora_rank: int = 0  # > 0: train LoRA adapters of this rank on the frozen base (one GPU)
    lora_alpha: float = 16.0
    lora_targets: str = "wqkv,wo,wgu,wdown"
    init_from: str = ""  # start from pretrained weights: model.safetensors (reference names) or a HF directory
    init_format: str = "safetensors"  # safetensors | hf
    checkpoint_dir: str = ""
    checkpoint_every: int = 0
    max_consecutive_skips: int = 20
    log_every: int = 10
    metrics_file: str = ""  # rank 0 appends one JSON line per logged step (loss, grad norm, tokens/s, MFU, ...)
    curriculum_start_len: int = 0  # > 0: sequence length grows from this to seq_len over curriculum_steps
    curriculum_steps: int = 0
    fixed_batch: bool = False  # reuse one seeded batch every step (the CPU demo's data)
    data_path: str = ""  # flat uint16/uint32 token file; empty = synthetic uniform ids
    data_dtype: str = "uint16"
    loader_threads: int = 4  # native loader fill workers
    recompute_activations: bool = False  # activation checkpointing: re-run each layer's forward in the backward
    offload_optimizer: bool = False  # fp32 master + AdamW moments in pinned host memory (train/offload.py)


@dataclass
class ParallelConfig:
    dp: int = 1  # data-parallel ranks: 1 (whatever the job has) or the job's world size
    tp: int = 1
    pp: int = 1  # pipeline stages (1F1B); spans every rank of the job
    cp: int = 1  # context parallelism: ranks share each sequence; spans the job
    cp_mode: str = "ulysses"  # ulysses (heads divisible by cp) | ring (zigzag chunks, any head count)
    zero_stage: int = 0  # 0, 1, 2, 3 (3 == FSDP)
    sequence_parallel: bool = True  # the tensor-parallel model keeps activations sequence-sharded (always)
    fused_collectives: bool = True  # False: the same schedules on NCCL collectives (library baseline)
    fuse_gather: bool = False  # ZeRO-3: parameter all-gather inside the first consuming GEMM (K17)
    fp8: bool = False
    # mx: power-of-two block scales applied by the tensor core (tcgen05 block-scaled
    # MMA), e4m3 forward and e5m2 data gradients; exact: fp32 block scales promoted
    # on the CUDA cores, forward projections only
    fp8_recipe: str = "mx"


@dataclass
class QuantConfig:
    weights: str = "none"  # none|int8|int4|fp8
    group_size: int = 128
    kv_cache: str = "bf16"  # bf16|fp8|int8


@dataclass
class ServeConfig:
    host: str = "127.0.0.1"
    port: int = 8080
    max_num_seqs: int = 256
    max_num_batched_tokens: int = 8192
    block_size: int = 16
    num_kv_blocks: int = 0  # 0 = size from free memory
    enable_prefix_caching: bool = True
    max_model_len: int = 4096
    cuda_graphs: bool = True  # decode steps replayed from CUDA graphs (per batch-size bucket)
    api_keys: tuple = ()
    rate_limit_rps: float = 0.0
    max_inflight_per_client: int = 0  # > 0: 429 for a client with this many requests running


@dataclass
class RunConfig:
    model: TransformerConfig = field(default_factory=TransformerConfig)
    train: TrainConfig = field(default_factory=TrainConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    quant: QuantConfig = field(default_factory=QuantConfig)
    serve: ServeConfig = field(default_factory=ServeConfig)


def _llama_1b() -> TransformerConfig:
    return TransformerConfig(hidden_dim=2048, num_heads=32, num_kv_heads=4, head_dim=64,
                             ff_dim=5632, vocab_size=32000, num_layers=22, max_seq_len=2048)


def _llama_8b() -> TransformerConfig:
    return TransformerConfig(hidden_dim=4096, num_heads=32, num_kv_heads=8, head_dim=128,
                             ff_dim=14336, vocab_size=128256, num_layers=32, max_seq_len=4096,
                             rope_base=500000.0)


PRESETS: Dict[str, RunConfig] = {
    # 4 layers, d 256, 4 heads x 64, ffn 688, vocab 1024, seq 128, batch 8, AdamW 3e-4 / 0.1
    "cpu-demo": RunConfig(
        model=TransformerConfig(hidden_dim=256, num_heads=4, head_dim=64, ff_dim=688,
                                vocab_size=1024, num_layers=4, max_seq_len=128),
        train=TrainConfig(lr=3e-4, weight_decay=0.1, micro_batch=8, seq_len=128, total_steps=50,
                          beta2=0.999, dynamic_loss_scale=False, fixed_batch=True)),
    "llama-1.1b-zero3": RunConfig(
        model=_llama_1b(),
        train=TrainConfig(micro_batch=4, seq_len=2048, total_steps=100),
        parallel=ParallelConfig(zero_stage=3)),
    "llama-8b-tp8-fp8": RunConfig(
        model=_llama_8b(),
        train=TrainConfig(micro_batch=32, seq_len=4096, dynamic_loss_scale=False),
        parallel=ParallelConfig(tp=8, sequence_parallel=True, fp8=True)),
    "llama-8b-fsdp-dp8": RunConfig(
        model=_llama_8b(),
        train=TrainConfig(micro_batch=2, seq_len=4096, grad_accum_steps=8, ema_decay=0.999),
        parallel=ParallelConfig(zero_stage=3)),
    "llama-8b-serve-int4": RunConfig(
        model=_llama_8b(),
        parallel=ParallelConfig(tp=8),
        quant=QuantConfig(weights="int4", group_size=128, kv_cache="fp8"),
        serve=ServeConfig(max_num_seqs=256)),
    # small model used by tests and smoke runs
    "tiny": RunConfig(
        model=TransformerConfig(hidden_dim=256, num_heads=4, num_kv_heads=2, head_dim=64,
                                ff_dim=512, vocab_size=512, num_layers=2, max_seq_len=256),
        train=TrainConfig(micro_batch=2, seq_len=128, total_steps=5)),
}


def _update(dc, values: Dict[str, Any]):
    names = {f.name: f for f in fields(dc)}
    for k, v in values.items():
        if k not in names:
            raise KeyError(f"unknown config key {type(dc).__name__}.{k}")
        cur = getattr(dc, k)
        if dataclasses.is_dataclass(cur) and isinstance(v, dict):
            _update(cur, v)
        else:
            setattr(dc, k, v)
    if hasattr(dc, "__post_init__"):
        dc.__post_init__()
    return dc


def get_preset(name: str) -> RunConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; choose from {sorted(PRESETS)}")
    return dataclasses.replace(
        PRESETS[name],
        model=dataclasses.replace(PRESETS[name].model),
        train=dataclasses.replace(PRESETS[name].train),
        parallel=dataclasses.replace(PRESETS[name].parallel),
        quant=dataclasses.replace(PRESETS[name].quant),
        serve=dataclasses.replace(PRESETS[name].serve),
    )


def load_config(path: Optional[str] = None, preset: Optional[str] = None,
                overrides: Optional[Dict[str, Any]] = None) -> RunConfig:
    """Preset, then a YAML/JSON file, then dotted overrides ({"train.lr": 1e-4})."""
    cfg = get_preset(preset) if preset else RunConfig()
    if path:
        with open(path) as f:
            if path.endswith((".yaml", ".yml")):
                import yaml
                data = yaml.safe_load(f) or {}
            else:
                data = json.load(f)
        _update(cfg, data)
    for key, val in (overrides or {}).items():
        section, _, name = key.partition(".")
        _update(getattr(cfg, section), {name: val})
    return cfg


def to_dict(cfg) -> Dict[str, Any]:
    return dataclasses.asdict(cfg)


def env_flag(name: str, default: str = "") -> str:
    return os.environ.get(name, default)
