"""Continuous-batching inference engine.

Scheduler (one `step()` = one decode batch plus prefill chunks):
  * running sequences each get one decode token per step (up to
    max_num_seqs); a sequence whose next token needs a new KV block takes one,
    and if none is free the most recently admitted running sequence is
    preempted (its blocks freed, it returns to the head of the queue and is
    recomputed later);
  * waiting requests are admitted in (priority, arrival) order while the
    step's token budget (max_num_batched_tokens) and free KV blocks allow;
    long prompts are split into chunks (chunked prefill) so one huge prompt
    does not stall the decode batch;
  * prompt blocks already in the prefix cache are not recomputed.

Reference: ContinuousBatching (include/nn/inference.hpp:89-170, FIFO admit to
max_batch), DynamicBatcher / PriorityScheduler
(include/api/serving_production.hpp:24-106) and SpeculativeDecoding's greedy
sampling (include/nn/inference.hpp:13-86).
"""
from __future__ import annotations

import itertools
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import torch

from ..config import ServeConfig, TransformerConfig
from ..models.params import FlatParams
from ..ops import serving as SV
from .kv_cache import BlockManager
from .model_runner import ModelRunner, PrefillItem


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    top_p: float = 1.0
    stop_token_ids: tuple = ()
    # token sequences that end generation when the output ends with one (the
    # server's OpenAI `stop` strings, tokenized); the server leaves them out of the text
    stop_sequences: tuple = ()
    seed: Optional[int] = None


def _mix64(a: int, b: int) -> int:
    """splitmix64 finaliser of a + golden-ratio * (b + 1): a 64-bit seed per (stream, index)."""
    z = (int(a) + 0x9E3779B97F4A7C15 * (int(b) + 1)) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def _ends_with_any(out: List[int], seqs) -> bool:
    for sq in seqs:
        n = len(sq)
        if n and len(out) >= n and tuple(out[-n:]) == tuple(sq):
            return True
    return False


@dataclass
class Request:
    req_id: int
    prompt: List[int]
    params: SamplingParams
    priority: int = 0
    arrival: float = 0.0
    output: List[int] = field(default_factory=list)
    table: List[int] = field(default_factory=list)
    computed: int = 0           # tokens whose K/V are in the cache
    prefill_len: int = 0        # tokens to prefill before decoding (all but a pending last token)
    cached_prefix: int = 0
    first_token_time: Optional[float] = None
    scheduled_time: Optional[float] = None  # first admission to the running set (queue time ends)
    token_times: List[float] = field(default_factory=list)
    finished: bool = False
    finish_reason: Optional[str] = None
    on_token: Optional[Callable[["Request", int], None]] = None

    @property
    def tokens(self) -> List[int]:
        return self.prompt + self.output

    # O(1) forms of len(tokens) and tokens[-1] for the per-step paths
    @property
    def n_tokens(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def last_token(self) -> int:
        return self.output[-1] if self.output else self.prompt[-1]

    @property
    def in_prefill(self) -> bool:
        return self.computed < self.prefill_len


class LLMEngine:
    def __init__(self, cfg: TransformerConfig, params: FlatParams, serve: Optional[ServeConfig] = None, *,
                 device="cuda", kv_dtype: str = "fp8", weights: str = "none", group_size: int = 128,
                 clock: Callable[[], float] = time.perf_counter, runner=None):
        """runner: an already built runner (e.g. the tensor-parallel
        serve.tp_runner.RunnerProxy on rank 0); params is then unused."""
        self.cfg = cfg
        self.sc = serve or ServeConfig()
        self.runner = runner if runner is not None else ModelRunner(
            cfg, params, device, kv_dtype=kv_dtype, weights=weights, group_size=group_size,
            num_blocks=self.sc.num_kv_blocks, block_size=self.sc.block_size,
            max_model_len=self.sc.max_model_len)
        if self.sc.cuda_graphs and hasattr(self.runner, "enable_graphs"):
            self.runner.enable_graphs(self.sc.max_num_seqs)
        self.blocks = BlockManager(self.runner.num_blocks, self.sc.block_size,
                                   self.sc.enable_prefix_caching)
        self.waiting: deque = deque()
        self.running: List[Request] = []
        self.ids = itertools.count()
        self.clock = clock
        self.finished: Dict[int, Request] = {}
        self.stats = {"prompt_tokens": 0, "generated_tokens": 0, "preemptions": 0, "steps": 0,
                      "prefill_tokens_computed": 0}
        self._seed = 1234
        # when a list: one (schedule_s, prefill_s, decode_s, prefill_tokens,
        # decode_seqs) record per step, host clock; the prefill and decode
        # phases each end with the device read of their sampled tokens
        self.step_log: Optional[list] = None

    # ---------------------------------------------------------- requests
    def add_request(self, prompt: List[int], params: Optional[SamplingParams] = None, priority: int = 0,
                    on_token=None, arrival: Optional[float] = None) -> int:
        if not prompt:
            raise ValueError("empty prompt")
        if len(prompt) + (params.max_tokens if params else 16) > self.sc.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        if params is not None and params.temperature > 0 and not getattr(self.runner, "supports_top_p", False):
            if params.top_p < 1.0:
                raise ValueError("top_p < 1 is not supported by this runner (tensor-parallel serving samples "
                                 "from vocabulary slices); use top_p = 1")
            if params.seed is not None:
                raise ValueError("per-request seeds are not supported by this runner (tensor-parallel serving)")
        r = Request(next(self.ids), list(prompt), params or SamplingParams(), priority,
                    self.clock() if arrival is None else arrival, on_token=on_token)
        self.stats["prompt_tokens"] += len(prompt)
        # priority first (lower value = sooner), FIFO within a priority: every
        # request, priority 0 included, goes in front of the first waiting
        # request with a larger priority value
        idx = next((k for k, w in enumerate(self.waiting) if w.priority > priority), len(self.waiting))
        self.waiting.insert(idx, r)
        return r.req_id

    def abort_request(self, req_id: int) -> bool:
        """Drop a request that has not finished (its client went away): its KV
        blocks are freed and it leaves the waiting / running queues.  Returns
        False when the request is unknown or already finished."""
        for r in list(self.running):
            if r.req_id == req_id:
                self.blocks.free_seq(r.table)
                self.running.remove(r)
                r.finished, r.finish_reason = True, "abort"
                self.finished[r.req_id] = r
                return True
        for r in list(self.waiting):
            if r.req_id == req_id:
                if r.table:
                    self.blocks.free_seq(r.table)
                self.waiting.remove(r)
                r.finished, r.finish_reason = True, "abort"
                self.finished[r.req_id] = r
                return True
        return False

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ---------------------------------------------------------- scheduling
    def _preempt(self, r: Request) -> None:
        """Free a running request's blocks; it is recomputed when readmitted
        (prompt and generated tokens, except the last one, which decode feeds)."""
        self.blocks.free_seq(r.table)
        r.computed = 0
        self.running.remove(r)
        self.waiting.appendleft(r)
        self.stats["preemptions"] += 1

    def _schedule(self):
        decode: List[Request] = []
        preempted = set()  # request ids preempted during this pass
        for r in list(self.running):
            if r.in_prefill or r.req_id in preempted:
                continue
            while True:
                try:
                    self.blocks.append_slot(r.table, r.n_tokens - 1)
                    break
                except MemoryError:
                    victims = [x for x in self.running if x is not r]
                    if not victims:
                        raise
                    preempted.add(victims[-1].req_id)
                    self._preempt(victims[-1])
            decode.append(r)
        if preempted:
            decode = [r for r in decode if r.req_id not in preempted]
        budget = max(self.sc.max_num_batched_tokens - len(decode), 1)
        prefill: List[Request] = [r for r in self.running if r.in_prefill]
        admitted_tokens = sum(r.prefill_len - r.computed for r in prefill)
        while (self.waiting and len(self.running) < self.sc.max_num_seqs
               and admitted_tokens < budget):
            r = self.waiting[0]
            seq = r.tokens if not r.output else r.tokens[:-1]
            try:
                r.table, cached = self.blocks.allocate(seq)
            except MemoryError:
                break
            self.waiting.popleft()
            if r.scheduled_time is None:
                r.scheduled_time = self.clock()
            r.prefill_len = len(seq)
            r.computed = cached
            r.cached_prefix = cached
            self.running.append(r)
            prefill.append(r)
            admitted_tokens += r.prefill_len - cached
        items = []
        for r in prefill:
            if budget <= 0:
                break
            n = min(r.prefill_len - r.computed, budget)
            chunk = r.tokens[r.computed:r.computed + n]
            slots = self.blocks.slots_for(r.table, 0, r.computed + n)
            last = r.computed + n == r.prefill_len
            items.append((r, PrefillItem(r.req_id, chunk, r.computed, slots, last and not r.output)))
            budget -= n
        return decode, items

    # ---------------------------------------------------------------- step
    def _emit(self, r: Request, tok: int, now: float) -> None:
        r.output.append(tok)
        r.token_times.append(now)
        if r.first_token_time is None:
            r.first_token_time = now
        self.stats["generated_tokens"] += 1
        if tok in r.params.stop_token_ids or _ends_with_any(r.output, r.params.stop_sequences):
            r.finished, r.finish_reason = True, "stop"
        elif len(r.output) >= r.params.max_tokens:
            r.finished, r.finish_reason = True, "length"
        if r.on_token:
            r.on_token(r, tok)
        if r.finished:
            self.blocks.free_seq(r.table)
            self.running.remove(r)
            self.finished[r.req_id] = r

    def _sample(self, reqs: List[Request], logits: torch.Tensor) -> List[int]:
        temps = [r.params.temperature for r in reqs]
        if all(t <= 0 for t in temps):
            tok = self.runner.sample(logits, None, 0)
        else:
            self._seed += 1
            kw = {}
            top_ps = [r.params.top_p for r in reqs]
            if any(p < 1.0 for p, t in zip(top_ps, temps) if t > 0):
                kw["top_ps"] = top_ps
            if any(r.params.seed is not None for r, t in zip(reqs, temps) if t > 0):
                # a seeded request's draw k uses (its seed, k), whatever its batch row
                kw["row_seeds"] = [_mix64(r.params.seed, len(r.output)) if r.params.seed is not None
                                   else _mix64(self._seed, i) for i, r in enumerate(reqs)]
            tok = self.runner.sample(logits, temps, self._seed, **kw)
        return tok.tolist()

    def step(self) -> List[Request]:
        """Run one scheduling step; returns requests that finished during it."""
        t0 = self.clock() if self.step_log is not None else 0.0
        decode, items = self._schedule()
        self.stats["steps"] += 1
        done_before = set(self.finished)
        t1 = self.clock() if self.step_log is not None else 0.0
        n_pre = sum(len(it.tokens) for _, it in items)
        if items:
            seq_ids, logits = self.runner.prefill([it for _, it in items])
            for r, it in items:
                r.computed += len(it.tokens)
                self.stats["prefill_tokens_computed"] += len(it.tokens)
                if not r.in_prefill:
                    self.blocks.register_full_blocks(r.tokens, r.table, r.prefill_len)
            if seq_ids:
                by_id = {r.req_id: r for r, _ in items}
                reqs = [by_id[i] for i in seq_ids]
                toks = self._sample(reqs, logits)
                now = self.clock()
                for r, t in zip(reqs, toks):
                    self._emit(r, t, now)
        t2 = self.clock() if self.step_log is not None else 0.0
        if decode:
            live = {x.req_id for x in self.running}
            decode = [r for r in decode if not r.finished and r.req_id in live]
        if decode:
            toks_in = [r.last_token for r in decode]
            pos = [r.n_tokens - 1 for r in decode]
            bs = self.blocks.block_size
            slots = [r.table[p // bs] * bs + p % bs for r, p in zip(decode, pos)]
            logits = self.runner.decode(toks_in, pos, slots, [r.table for r in decode])
            toks = self._sample(decode, logits)
            now = self.clock()
            for r, t in zip(decode, toks):
                self._emit(r, t, now)
        if self.step_log is not None:
            t3 = self.clock()
            self.step_log.append((t1 - t0, t2 - t1, t3 - t2, n_pre, len(decode)))
        return [self.finished[i] for i in self.finished if i not in done_before]

    def generate(self, prompts: List[List[int]], params: Optional[SamplingParams] = None) -> List[List[int]]:
        ids = [self.add_request(p, params) for p in prompts]
        while any(i not in self.finished for i in ids):
            self.step()
        return [self.finished[i].output for i in ids]
