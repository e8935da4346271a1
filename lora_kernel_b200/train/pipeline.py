"""The reference's Python-module API on the B200 engine.

    cfg = TransformerConfig(); cfg.hidden_dim = 256; ...
    model = Transformer(cfg)                         # random-init N(0, 0.02)
    pipe = TrainingPipeline(model, 3e-4, 0.1, 1.0)   # lr, weight decay, clip
    loss = pipe.train_step(ids, targets)             # one micro-step
    pipe.set_learning_rate(1e-4); pipe.current_step()

Mirrors bindings/python_module.cpp:11-56 and TrainingPipeline
(include/nn/training_pipeline.hpp:15-263): set_gradient_accumulation_steps,
init_swa, init_ema and get_loss_scaler keep their names.  Semantics follow the
standard definitions rather than the reference's defects (global-norm clip
instead of per-tensor, bias correction counted in optimizer steps, EMA/SWA over
every parameter, a skip counter that resets on a good step).
"""
from __future__ import annotations

from typing import Optional, Union

import numpy as np
import torch

from ..config import TrainConfig, TransformerConfig
from ..models.llama import LlamaModel
from ..utils.profiler import ph
from .optimizer import SWA, FusedAdamW


def _as_ids(x, device) -> torch.Tensor:
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(x)
    if not isinstance(x, torch.Tensor):
        x = torch.tensor(x)
    if x.dim() == 1:
        x = x.unsqueeze(0)
    return x.to(device=device, dtype=torch.int64, non_blocking=True)


class Transformer:
    """Llama decoder with the reference's class name and methods."""

    def __init__(self, cfg: TransformerConfig, device: Union[str, torch.device] = "cuda",
                 seed: int = 1234):
        self.cfg = cfg
        self.device = torch.device(device)
        self.engine = LlamaModel(cfg, self.device, seed=seed)

    def forward(self, ids) -> torch.Tensor:
        """Logits [B, S, vocab] (bf16) for token ids [B, S]."""
        return self.engine.forward(_as_ids(ids, self.device))

    __call__ = forward

    def num_parameters(self) -> int:
        return self.cfg.num_parameters()

    @property
    def params(self):
        return self.engine.params

    def state_dict(self):
        return self.engine.params.to_reference_state_dict()

    def load_state_dict(self, sd) -> None:
        self.engine.params.load_reference_state_dict(sd)


class TrainingPipeline:
    def __init__(self, model: Transformer, lr: float = 3e-4, weight_decay: float = 0.1,
                 max_grad_norm: float = 1.0, train_cfg: Optional[TrainConfig] = None):
        tc = train_cfg or TrainConfig(lr=lr, weight_decay=weight_decay, max_grad_norm=max_grad_norm)
        tc.lr, tc.weight_decay, tc.max_grad_norm = lr, weight_decay, max_grad_norm
        self.tc = tc
        self.model = model
        eng = model.engine
        self.engine = eng
        eng.recompute = tc.recompute_activations
        if tc.offload_optimizer:
            from .offload import OffloadedAdamW
            if tc.ema_decay > 0:
                raise NotImplementedError("EMA with the offloaded optimizer")
            self.opt = OffloadedAdamW(eng.params.flat.float().cpu(), eng.params.segments(decay_norms=tc.decay_norms),
                                      eng.device, lr=lr, betas=(tc.beta1, tc.beta2), eps=tc.eps,
                                      weight_decay=weight_decay, max_grad_norm=max_grad_norm,
                                      dynamic_loss_scale=tc.dynamic_loss_scale,
                                      init_loss_scale=tc.init_loss_scale,
                                      growth_interval=tc.loss_scale_growth_interval)
        else:
            master = eng.params.flat.float()
            self.opt = FusedAdamW(master, eng.params.segments(decay_norms=tc.decay_norms), lr=lr,
                                  betas=(tc.beta1, tc.beta2), eps=tc.eps, weight_decay=weight_decay,
                                  max_grad_norm=max_grad_norm, dynamic_loss_scale=tc.dynamic_loss_scale,
                                  init_loss_scale=tc.init_loss_scale,
                                  growth_interval=tc.loss_scale_growth_interval,
                                  ema_decay=tc.ema_decay)
        self.accum_steps = max(1, tc.grad_accum_steps)
        self._micro = 0
        self._opt_steps = 0
        self.swa: Optional[SWA] = None
        self.loss_acc = torch.zeros(2, dtype=torch.float32, device=eng.device)
        self.last_loss = float("nan")
        self.pre_optimizer = None  # optional callable(flat fp32 grads), e.g. fault injection
        if tc.swa_start >= 0:
            self.init_swa(tc.swa_start)

    # ----------------------------------------------------- reference setters
    def set_learning_rate(self, lr: float) -> None:
        self.opt.set_lr(lr)

    def current_step(self) -> int:
        return self._opt_steps

    def set_gradient_accumulation_steps(self, n: int) -> None:
        self.accum_steps = max(1, int(n))

    def init_swa(self, start_step: int, every: int = 1) -> None:
        self.swa = SWA(self.opt.p32, start_step, every)

    def init_ema(self, decay: float) -> None:
        self.opt.ema_decay = float(decay)
        if self.opt.ema is None:
            self.opt.ema = self.opt.p32.clone()

    def get_loss_scaler(self):
        return self.opt.scaler

    # -------------------------------------------------------------- stepping
    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        """Forward + backward of one micro-batch; on the last micro-batch of an
        accumulation window also runs the optimizer.  No host synchronisation."""
        n_tok = ids.numel()
        self.engine.forward_backward(ids, targets, loss_scale=self.opt.scaler.scale_tensor(),
                                     grad_scale=1.0 / (n_tok * self.accum_steps),
                                     label_smoothing=self.tc.label_smoothing, z_loss=self.tc.z_loss,
                                     loss_acc=self.loss_acc,
                                     overwrite_grads=(self._micro % self.accum_steps == 0))
        self._micro += 1
        if self._micro % self.accum_steps == 0:
            if self.pre_optimizer is not None:
                self.pre_optimizer(self.engine.grads.flat)
            with ph("step.grad_norm+finalize"):
                self.opt.norm_partials(self.engine.grads.flat)
                self.opt.finalize()
            with ph("step.adamw"):
                self.opt.apply(self.engine.grads.flat, self.engine.params.flat, zero_grad=False)
            self._opt_steps += 1
            if self.swa is not None:
                self.swa.update(self.opt.p32, self._opt_steps)

    def train_step(self, ids, targets) -> float:
        """One micro-step; returns the mean token loss of this micro-batch."""
        ids = _as_ids(ids, self.engine.device)
        targets = _as_ids(targets, self.engine.device)
        self.loss_acc.zero_()
        self.micro_step_async(ids, targets)
        s, n = self.loss_acc.tolist()
        self.last_loss = s / max(n, 1.0)
        if self.opt.scaler.consecutive_skips() > self.tc.max_consecutive_skips:
            raise FloatingPointError(
                f"{self.opt.scaler.consecutive_skips()} consecutive overflow steps; aborting")
        return self.last_loss

    def ema_weights(self) -> Optional[torch.Tensor]:
        return self.opt.ema


class LoRATrainingPipeline(TrainingPipeline):
    """Fine-tune LoRA adapters on a frozen base model (same stepping API)."""

    def __init__(self, model: Transformer, lora_cfg=None, lr: float = 1e-4, weight_decay: float = 0.0,
                 max_grad_norm: float = 1.0, train_cfg: Optional[TrainConfig] = None):
        from ..models.lora import LoRAAdapters, LoRAConfig
        tc = train_cfg or TrainConfig(lr=lr, weight_decay=weight_decay, max_grad_norm=max_grad_norm)
        tc.lr, tc.weight_decay, tc.max_grad_norm = lr, weight_decay, max_grad_norm
        self.tc = tc
        self.model = model
        eng = self.engine = model.engine
        self.lora = LoRAAdapters(model.cfg, lora_cfg or LoRAConfig(), eng.device)
        eng.lora = self.lora
        eng.train_base = False
        self.opt = FusedAdamW(self.lora.flat.float(), self.lora.segments(), lr=lr,
                              betas=(tc.beta1, tc.beta2), eps=tc.eps, weight_decay=weight_decay,
                              max_grad_norm=max_grad_norm, dynamic_loss_scale=tc.dynamic_loss_scale,
                              init_loss_scale=tc.init_loss_scale,
                              growth_interval=tc.loss_scale_growth_interval, ema_decay=tc.ema_decay)
        self.accum_steps = max(1, tc.grad_accum_steps)
        self._micro = 0
        self._opt_steps = 0
        self.swa = None
        self.loss_acc = torch.zeros(2, dtype=torch.float32, device=eng.device)
        self.last_loss = float("nan")
        self.pre_optimizer = None

    def micro_step_async(self, ids: torch.Tensor, targets: torch.Tensor) -> None:
        first = self._micro % self.accum_steps == 0
        self.engine.forward_backward(ids, targets, loss_scale=self.opt.scaler.scale_tensor(),
                                     grad_scale=1.0 / (ids.numel() * self.accum_steps),
                                     loss_acc=self.loss_acc, overwrite_grads=first)
        self._micro += 1
        if self._micro % self.accum_steps == 0:
            if self.pre_optimizer is not None:
                self.pre_optimizer(self.lora.grads)
            self.opt.norm_partials(self.lora.grads)
            self.opt.finalize()
            self.opt.apply(self.lora.grads, self.lora.flat, zero_grad=False)
            self._opt_steps += 1

    def merge(self) -> None:
        """Fold the adapters into the base weights (W += s B A) and detach them."""
        self.lora.merge_into(self.engine.params)
        self.engine.lora = None
