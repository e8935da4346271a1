"""Speculative decoding on CPU with table (bigram) models: greedy output is the
target's own greedy decode, and speculative sampling draws from the target
distribution."""
import pytest
import torch

from lora_kernel_b200.serve.speculative import Scorer, SpeculativeDecoder, greedy_reference


class Bigram(Scorer):
    """Next-token logits depend on the current token only: logits[t] = table[t]."""

    def __init__(self, table: torch.Tensor):
        self.table = table
        self._len = 0
        self.calls = 0

    @property
    def length(self):
        return self._len

    def extend(self, tokens, all_logits):
        self.calls += 1
        self._len += len(tokens)
        rows = self.table[torch.tensor(tokens)]
        return rows if all_logits else rows[-1:]

    def truncate(self, length):
        self._len = min(self._len, length)


def _table(V, seed, scale=3.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(V, V, generator=g) * scale


@pytest.mark.parametrize("k", [1, 3, 5])
def test_greedy_speculative_equals_target_greedy(k):
    V = 50
    target, draft = Bigram(_table(V, 1)), Bigram(_table(V, 2))
    prompt = [3, 17, 9]
    ref = greedy_reference(Bigram(target.table), prompt, 40)
    sd = SpeculativeDecoder(target, draft, k=k)
    assert sd.generate(prompt, 40) == ref
    assert sd.stats.emitted == 40
    # fewer target forwards than tokens unless every proposal is rejected
    assert sd.stats.target_forwards <= 40


def test_identical_draft_accepts_everything():
    V = 30
    t = _table(V, 4)
    sd = SpeculativeDecoder(Bigram(t), Bigram(t.clone()), k=4)
    out = sd.generate([1, 2], 20)
    assert out == greedy_reference(Bigram(t), [1, 2], 20)
    assert sd.stats.acceptance_rate == 1.0
    assert sd.stats.tokens_per_target_forward == pytest.approx(5.0)


def test_partially_matching_draft():
    # the draft agrees with the target on half of the vocabulary
    V = 40
    t = _table(V, 5)
    d = _table(V, 6)
    d[: V // 2] = t[: V // 2]
    sd = SpeculativeDecoder(Bigram(t), Bigram(d), k=4)
    assert sd.generate([7], 60) == greedy_reference(Bigram(t), [7], 60)
    assert 0.0 < sd.stats.acceptance_rate < 1.0


def test_eos_and_length_limits():
    V = 20
    t = _table(V, 7)
    ref = greedy_reference(Bigram(t), [0], 30)
    eos = ref[5]
    first = ref.index(eos)
    sd = SpeculativeDecoder(Bigram(t), Bigram(_table(V, 8)), k=3, eos_id=eos)
    assert sd.generate([0], 30) == ref[:first + 1]
    sd2 = SpeculativeDecoder(Bigram(t), Bigram(_table(V, 8)), k=4)
    assert len(sd2.generate([0], 7)) == 7


def test_speculative_sampling_matches_target_distribution():
    V, runs = 5, 6000
    t, d = _table(V, 11, 1.0), _table(V, 12, 1.0)
    temp = 0.8
    p = torch.softmax(t / temp, dim=-1)
    # distribution of the 2nd generated token after prompt [2]: sum_a p(a|2) p(b|a)
    want = p[2] @ p
    counts = torch.zeros(V)
    for s in range(runs):
        sd = SpeculativeDecoder(Bigram(t), Bigram(d), k=3, temperature=temp, seed=s)
        out = sd.generate([2], 2)
        counts[out[1]] += 1
    e = want * runs
    chi2 = float(((counts - e) ** 2 / e).sum())
    assert chi2 < 25.0, (counts / runs, want)  # 4 dof: p ~ 5e-5
