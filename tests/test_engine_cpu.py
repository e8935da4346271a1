"""Continuous-batching engine on CPU with a fake runner that keeps a token-level
KV store: every token the engine makes the runner write lands in a slot, and
next-token logits are computed from the context read back through the block
tables.  Any wrong slot, stale prefix-cache block or broken preemption
changes the output, which is checked against a direct simulation."""
import random

import pytest
import torch

from lora_kernel_b200.config import ServeConfig, TransformerConfig
from lora_kernel_b200.serve.engine import LLMEngine, SamplingParams

V = 97


def next_token(context):
    h = 0
    for t in context:
        h = (h * 131 + t + 7) % 1_000_003
    return (h + len(context)) % V


class KVRunner:
    def __init__(self, num_blocks, block_size, max_model_len=4096):
        self.num_blocks, self.block_size, self.max_model_len = num_blocks, block_size, max_model_len
        self.kv = {}
        self.prefill_rows = 0

    def _logits(self, ctx):
        z = torch.full((V,), -1e9)
        z[next_token(ctx)] = 0.0
        return z

    def prefill(self, items):
        ids, rows = [], []
        for it in items:
            n = len(it.tokens)
            self.prefill_rows += n
            for k, t in enumerate(it.tokens):
                self.kv[it.slots[it.start + k]] = t
            if it.want_logits:
                ctx = [self.kv[s] for s in it.slots[: it.start + n]]
                ids.append(it.seq_id)
                rows.append(self._logits(ctx))
        return ids, (torch.stack(rows) if rows else torch.empty(0, V))

    def decode(self, tokens, positions, slots, tables):
        out = []
        bs = self.block_size
        for t, p, s, table in zip(tokens, positions, slots, tables):
            self.kv[s] = t
            ctx = [self.kv[table[i // bs] * bs + i % bs] for i in range(p + 1)]
            out.append(self._logits(ctx))
        return torch.stack(out)

    def sample(self, logits, temps, seed):
        return torch.argmax(logits, dim=-1)


def reference(prompt, n):
    out = []
    for _ in range(n):
        out.append(next_token(prompt + out))
    return out


def _engine(num_blocks, block_size=4, **kw):
    sc = ServeConfig(num_kv_blocks=num_blocks, block_size=block_size, cuda_graphs=False, max_model_len=512, **kw)
    cfg = TransformerConfig(vocab_size=V)
    runner = KVRunner(num_blocks, block_size)
    return LLMEngine(cfg, None, sc, runner=runner), runner


@pytest.mark.parametrize("num_blocks,max_seqs,budget,gen", [(400, 64, 4096, 15), (40, 8, 64, 15), (20, 8, 16, 40)])
def test_engine_outputs_match_simulation(num_blocks, max_seqs, budget, gen):
    rng = random.Random(num_blocks)
    shared = [rng.randrange(V) for _ in range(13)]
    prompts = []
    for k in range(20):
        tail = [rng.randrange(V) for _ in range(rng.randrange(1, 12))]
        prompts.append((shared if k % 3 == 0 else []) + tail)
    eng, runner = _engine(num_blocks, max_num_seqs=max_seqs, max_num_batched_tokens=budget)
    params = [SamplingParams(max_tokens=rng.randrange(gen // 2, gen)) for _ in prompts]
    ids = [eng.add_request(p, sp) for p, sp in zip(prompts, params)]
    steps = 0
    while eng.has_work():
        eng.step()
        steps += 1
        assert steps < 5000
    for i, p, sp in zip(ids, prompts, params):
        assert eng.finished[i].output == reference(p, sp.max_tokens), i
    assert eng.blocks.num_free() == num_blocks  # every block came back
    if num_blocks == 20:
        assert eng.stats["preemptions"] > 0  # the small cache forced recomputation


def test_prefix_cache_skips_shared_blocks():
    eng, runner = _engine(200, block_size=4)
    prefix = list(range(40))
    eng.generate([prefix + [50]], SamplingParams(max_tokens=2))
    before = runner.prefill_rows
    out = eng.generate([prefix + [60, 61]], SamplingParams(max_tokens=3))
    assert out[0] == reference(prefix + [60, 61], 3)
    assert runner.prefill_rows - before <= 4 + 2  # only the tail block was prefilled
    assert eng.blocks.stats.hits >= 10


def test_stop_tokens_and_priority():
    eng, _ = _engine(100)
    p = [5, 6, 7]
    want = reference(p, 10)
    out = eng.generate([p], SamplingParams(max_tokens=10, stop_token_ids=(want[3],)))
    assert out[0] == want[: want.index(want[3]) + 1]
    eng2, _ = _engine(100, max_num_seqs=1)
    a = eng2.add_request([1, 2], SamplingParams(max_tokens=1))
    b = eng2.add_request([3, 4], SamplingParams(max_tokens=1), priority=-1)
    eng2.step()
    assert b in eng2.finished and a not in eng2.finished


def test_top_p_reaches_a_runner_that_supports_it_and_is_refused_otherwise():
    """Rows with temperature > 0 and top_p < 1 go to the runner's nucleus
    sampler; a runner without one (tensor-parallel serving) refuses the
    request instead of ignoring top_p; top_p = 1 keeps the plain call."""
    eng, runner = _engine(100)
    with pytest.raises(ValueError, match="top_p"):
        eng.add_request([1, 2], SamplingParams(max_tokens=2, temperature=0.8, top_p=0.9))
    eng.add_request([1, 2], SamplingParams(max_tokens=2, temperature=0.0, top_p=0.9))   # greedy: no nucleus
    calls = []

    class TopP(KVRunner):
        supports_top_p = True

        def sample(self, logits, temps, seed, top_ps=None):
            calls.append((temps, top_ps))
            return torch.argmax(logits, dim=-1)

    sc = ServeConfig(num_kv_blocks=100, block_size=4, cuda_graphs=False, max_model_len=512)
    eng = LLMEngine(TransformerConfig(vocab_size=V), None, sc, runner=TopP(100, 4))
    p = [9, 8, 7]
    out = eng.generate([p, p], SamplingParams(max_tokens=3, temperature=0.7, top_p=0.5))
    assert out == [reference(p, 3)] * 2
    assert calls and all(tp == [0.5] * len(t) for t, tp in calls)
    calls.clear()
    eng.generate([p], SamplingParams(max_tokens=2, temperature=0.7, top_p=1.0))
    assert calls and all(tp is None for _, tp in calls)


def test_stop_sequences_end_generation():
    """A request stops as soon as its output ends with one of its stop
    sequences (finish reason "stop"); the engine keeps the tokens (the server
    trims them)."""
    eng, _ = _engine(100)
    p = [11, 12, 13]
    want = reference(p, 12)
    seq = tuple(want[4:6])
    rid = eng.add_request(p, SamplingParams(max_tokens=12, stop_sequences=((99, 98, 97), seq)))
    while eng.has_work():
        eng.step()
    r = eng.finished[rid]
    first = next(i for i in range(1, 12) if tuple(want[i - 1:i + 1]) == seq)
    assert r.output == want[:first + 1] and r.finish_reason == "stop"


def test_request_seeds_give_row_independent_noise():
    """Seeded requests send one seed per row derived from (request seed, draw
    index), so equal seeds give equal seeds per draw whatever the batch row;
    a runner without per-row seeds refuses seeded sampling."""
    eng, _ = _engine(100)
    with pytest.raises(ValueError, match="seed"):
        eng.add_request([1, 2], SamplingParams(max_tokens=2, temperature=0.5, seed=3))
    calls = []

    class Seeded(KVRunner):
        supports_top_p = True

        def sample(self, logits, temps, seed, top_ps=None, row_seeds=None):
            calls.append(row_seeds)
            return torch.argmax(logits, dim=-1)

    sc = ServeConfig(num_kv_blocks=100, block_size=4, cuda_graphs=False, max_model_len=512)
    eng = LLMEngine(TransformerConfig(vocab_size=V), None, sc, runner=Seeded(100, 4))
    a = eng.add_request([5, 6], SamplingParams(max_tokens=3, temperature=0.9, seed=42))
    b = eng.add_request([7, 8, 9], SamplingParams(max_tokens=3, temperature=0.9))
    c = eng.add_request([5, 6], SamplingParams(max_tokens=3, temperature=0.9, seed=42))
    while eng.has_work():
        eng.step()
    assert calls and all(rs is not None and len(rs) == 3 for rs in calls)
    for rs in calls:   # rows a and c (same seed, same draw index) share a seed; b differs
        assert rs[0] == rs[2] != rs[1]
    assert len({rs[0] for rs in calls}) == len(calls)     # a new seed per draw
    assert eng.finished[a].output == eng.finished[c].output


def test_priority_zero_goes_before_waiting_lower_priorities():
    """Lower value = sooner for every request, the default priority 0 included."""
    eng, _ = _engine(100, max_num_seqs=1)
    a = eng.add_request([1, 2], SamplingParams(max_tokens=1), priority=5)
    b = eng.add_request([3, 4], SamplingParams(max_tokens=1))
    c = eng.add_request([5, 6], SamplingParams(max_tokens=1))
    assert [r.req_id for r in eng.waiting] == [b, c, a]  # FIFO within priority 0
    eng.step()
    assert b in eng.finished and a not in eng.finished


def test_abort_request_frees_blocks_and_work():
    eng, _ = _engine(64, block_size=4)
    free0 = eng.blocks.num_free()
    a = eng.add_request(list(range(1, 30)), SamplingParams(max_tokens=50))
    b = eng.add_request([7, 8, 9], SamplingParams(max_tokens=50))
    eng.step()
    eng.step()
    assert any(r.req_id == a for r in eng.running)
    assert eng.abort_request(a) and eng.abort_request(b)
    assert not eng.has_work()
    assert eng.finished[a].finish_reason == "abort"
    assert eng.blocks.num_free() == free0
    assert not eng.abort_request(a)  # already gone


def test_tp_runner_messages_round_trip():
    """The tensor-parallel serving control messages (decode inputs with ragged
    block tables, sampling temperatures and 64-bit seeds) survive packing."""
    import numpy as np
    from lora_kernel_b200.serve.tp_runner import pack_decode, pack_sample, unpack_decode, unpack_sample
    t, p, s, bt = unpack_decode(pack_decode([5, 6, 7], [10, 20, 30], [100, 200, 300], [[1], [3, 4, 5], [9, 8]]))
    assert t.tolist() == [5, 6, 7] and p.tolist() == [10, 20, 30] and s.tolist() == [100, 200, 300]
    assert bt.tolist() == [[1, 0, 0], [3, 4, 5], [9, 8, 0]] and bt.dtype == np.int32
    for temps, seed in [(None, 0), ([0.7, 1.0], (1 << 64) - 1), ([0.5], 7)]:
        got_t, got_s = unpack_sample(pack_sample(temps, seed))
        assert got_s == seed
        assert got_t is None if temps is None else np.allclose(got_t, temps)
