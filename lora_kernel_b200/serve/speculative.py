"""Speculative decoding: a small draft model proposes k tokens, the target
model scores all of them in one chunked forward, and the longest acceptable
prefix is kept (plus one token from the target), so each target forward yields
between 1 and k+1 tokens.

Greedy (temperature 0): draft tokens are accepted while they equal the
target's argmax; the first mismatch is replaced by the target's argmax.  The
output is token-for-token the target's own greedy decode.

Sampling (temperature > 0), the speculative sampling rule of Leviathan et al.
2023 / Chen et al. 2023: draft token d_j ~ q_j is accepted with probability
min(1, p_j(d_j) / q_j(d_j)); on the first rejection the token is redrawn from
the residual distribution norm(max(0, p_j - q_j)) and the round ends; when all
k are accepted a bonus token is drawn from p_{k+1}.  Every emitted token is
distributed exactly as a sample from the target.

KV caches: each model keeps the KV of a prefix of the committed tokens.  A
round feeds the draft the committed tokens it has not seen plus its own
proposals, and feeds the target the unseen committed tokens plus the k
proposals with logits for every row.  Rejected positions are dropped by
truncating the cached length; their stale KV is overwritten later.

`Scorer` is the interface to a model: `RunnerScorer` drives a `ModelRunner`
(the paged-KV serving runner; one sequence, contiguous KV slots), and any
object with the same two methods works (the CPU tests use a table model).

Reference: SpeculativeDecoding (include/nn/inference.hpp:13-86: greedy draft,
accept/reject, residual resampling with a fixed seed).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch


class Scorer:
    """One sequence's view of a model with a KV cache."""

    def extend(self, tokens: List[int], all_logits: bool) -> torch.Tensor:
        """Append `tokens` after the cached prefix; return fp32 logits [n, V]
        for every appended row (all_logits) or [1, V] for the last one."""
        raise NotImplementedError

    def truncate(self, length: int) -> None:
        """Keep only the first `length` cached positions."""
        raise NotImplementedError

    @property
    def length(self) -> int:
        raise NotImplementedError


class RunnerScorer(Scorer):
    """A ModelRunner used for one sequence with KV slots [base, base + max_len)."""

    def __init__(self, runner, base_slot: int = 0, max_len: Optional[int] = None, seq_id: int = 0):
        self.runner = runner
        self.base = base_slot
        self.max_len = max_len or runner.max_model_len
        if base_slot + self.max_len > runner.num_blocks * runner.block_size:
            raise ValueError("RunnerScorer: slot range exceeds the runner's KV cache")
        self.seq_id = seq_id
        self._len = 0

    @property
    def length(self) -> int:
        return self._len

    def extend(self, tokens: List[int], all_logits: bool) -> torch.Tensor:
        from .model_runner import PrefillItem
        n = len(tokens)
        if self._len + n > self.max_len:
            raise ValueError("RunnerScorer: sequence longer than its slot range")
        slots = list(range(self.base, self.base + self._len + n))
        item = PrefillItem(self.seq_id, list(tokens), self._len, slots, True, all_logits)
        _, logits = self.runner.prefill([item])
        self._len += n
        return logits.float()

    def truncate(self, length: int) -> None:
        self._len = min(self._len, length)


@dataclass
class SpecStats:
    rounds: int = 0
    proposed: int = 0
    accepted: int = 0
    emitted: int = 0
    target_forwards: int = 0
    per_round: List[int] = field(default_factory=list)

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / max(1, self.proposed)

    @property
    def tokens_per_target_forward(self) -> float:
        return self.emitted / max(1, self.target_forwards)


class SpeculativeDecoder:
    def __init__(self, target: Scorer, draft: Scorer, k: int = 4, temperature: float = 0.0, seed: int = 0,
                 eos_id: Optional[int] = None):
        if k < 1:
            raise ValueError("k must be >= 1")
        self.target, self.draft, self.k = target, draft, k
        self.temperature = float(temperature)
        self.eos_id = eos_id
        self.gen = torch.Generator().manual_seed(seed)
        self.stats = SpecStats()

    # ------------------------------------------------------------ helpers
    def _probs(self, logits: torch.Tensor) -> torch.Tensor:
        return torch.softmax(logits.float().cpu() / self.temperature, dim=-1)

    def _draw(self, p: torch.Tensor) -> int:
        return int(torch.multinomial(p, 1, generator=self.gen))

    def _uniform(self) -> float:
        return float(torch.rand(1, generator=self.gen))

    # ---------------------------------------------------------------- run
    @torch.no_grad()
    def generate(self, prompt: List[int], max_new_tokens: int) -> List[int]:
        if not prompt:
            raise ValueError("empty prompt")
        greedy = self.temperature <= 0.0
        T, Dm = self.target, self.draft
        T.truncate(0)
        Dm.truncate(0)
        committed = list(prompt)
        out: List[int] = []
        # the prompt (all but its last token, which each round feeds)
        if len(committed) > 1:
            T.extend(committed[:-1], all_logits=False)
            Dm.extend(committed[:-1], all_logits=False)
        while len(out) < max_new_tokens:
            k = min(self.k, max_new_tokens - len(out))
            # ---- draft proposals
            drafts: List[int] = []
            qs: List[torch.Tensor] = []
            feed = committed[Dm.length:]
            for j in range(k):
                lg = Dm.extend(feed, all_logits=False)[-1]
                if greedy:
                    d = int(torch.argmax(lg))
                else:
                    q = self._probs(lg)
                    d = self._draw(q)
                    qs.append(q)
                drafts.append(d)
                feed = [d]
            # ---- one target forward over the unseen committed tokens + proposals
            t_feed = committed[T.length:] + drafts
            t0 = len(committed) - 1 - T.length  # row predicting drafts[0]
            lg_t = T.extend(t_feed, all_logits=True)[t0:]
            self.stats.target_forwards += 1
            accepted = 0
            if greedy:
                tgt = torch.argmax(lg_t, dim=-1).tolist()
                while accepted < k and drafts[accepted] == tgt[accepted]:
                    accepted += 1
                extra = tgt[accepted]
            else:
                ps = self._probs(lg_t)
                extra = None
                while accepted < k:
                    d = drafts[accepted]
                    p, q = ps[accepted], qs[accepted]
                    if self._uniform() * float(q[d]) <= float(p[d]):
                        accepted += 1
                        continue
                    resid = torch.clamp(p - q, min=0.0)
                    tot = float(resid.sum())
                    extra = self._draw(resid / tot) if tot > 0 else self._draw(p)
                    break
                if extra is None:
                    extra = self._draw(ps[k])
            new = drafts[:accepted] + [extra]
            self.stats.rounds += 1
            self.stats.proposed += k
            self.stats.accepted += accepted
            self.stats.per_round.append(accepted)
            # ---- keep the cached prefixes that match the committed tokens
            base = len(committed)
            committed += new
            T.truncate(base + accepted)  # the target saw drafts[:accepted] correctly; `extra` is unseen
            Dm.truncate(min(Dm.length, base + accepted))
            stop = False
            for t in new:
                if len(out) >= max_new_tokens:
                    break
                out.append(t)
                self.stats.emitted += 1
                if self.eos_id is not None and t == self.eos_id:
                    stop = True
                    break
            if stop:
                break
        return out


def greedy_reference(target: Scorer, prompt: List[int], max_new_tokens: int) -> List[int]:
    """Plain greedy decoding through the same scorer (one token per forward)."""
    target.truncate(0)
    out: List[int] = []
    feed = list(prompt)
    for _ in range(max_new_tokens):
        lg = target.extend(feed, all_logits=False)[-1]
        t = int(torch.argmax(lg))
        out.append(t)
        feed = [t]
    return out
