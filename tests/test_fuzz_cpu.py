"""Property-based (hypothesis) tests of host-side components: random inputs,
invariants checked on every example.  Covers what the reference's in-header
FuzzTester / StabilityTest only printed as passed."""
import zlib

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

FAST = settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@FAST
@given(st.text(max_size=200))
def test_byte_tokenizer_round_trip(text):
    from lora_kernel_b200.serve.tokenizer import ByteTokenizer
    tok = ByteTokenizer(256)
    ids = tok.encode(text)
    assert all(0 <= i < 256 for i in ids)
    assert tok.decode(ids) == text


@FAST
@given(stream=st.lists(st.integers(0, 5), min_size=1, max_size=40),
       stops=st.lists(st.lists(st.integers(0, 5), min_size=1, max_size=4).map(tuple), max_size=3))
def test_stop_trimmer_releases_exactly_the_text_before_the_stop(stream, stops):
    """Feed tokens as the engine would (finishing at the first point where the
    output ends with a stop sequence); the released tokens are the output
    without that sequence, and nothing is released early that is later cut."""
    from lora_kernel_b200.serve.server import StopTrimmer
    end, hit = len(stream), None
    for i in range(1, len(stream) + 1):
        m = [s for s in stops if tuple(stream[max(0, i - len(s)):i]) == s and i >= len(s)]
        if m:
            end, hit = i, m
            break
    tr = StopTrimmer(stops)
    out = []
    for k in range(end):
        done = k == end - 1
        out += tr.push(stream[k], done, ("stop" if hit else "length") if done else None)
        assert out == stream[:len(out)]                 # releases are always a prefix of the output
    if hit:
        first = next(s for s in tr.stops if tuple(stream[end - len(s):end]) == s)
        assert out == stream[:end - len(first)]
    else:
        assert out == stream[:end]


@FAST
@given(ops=st.lists(st.tuples(st.sampled_from(["alloc", "free", "grow"]), st.integers(0, 7),
                              st.integers(1, 60)), max_size=60),
       prefix=st.booleans())
def test_block_manager_conserves_blocks(ops, prefix):
    """Random allocate / grow / free with shared prompt prefixes: every block
    is free, evictable or referenced; reference counts equal the number of
    tables holding the block; freeing everything returns all blocks."""
    from lora_kernel_b200.serve.kv_cache import BlockManager
    bm = BlockManager(24, 4, enable_prefix_caching=prefix)
    base = list(range(100))
    live = {}
    for op, key, n in ops:
        if op == "alloc" and key not in live:
            toks = base[:n] if key % 2 else [key] * n                # half the prompts share a prefix
            try:
                table, cached = bm.allocate(toks)
            except MemoryError:
                continue
            assert cached % 4 == 0 and cached < len(toks) and len(table) == bm.blocks_needed(toks)
            bm.register_full_blocks(toks, table, len(toks))
            live[key] = [table, len(toks)]
        elif op == "grow" and key in live:
            table, length = live[key]
            try:
                bm.append_slot(table, length)
            except MemoryError:
                continue
            live[key][1] = length + 1
        elif op == "free" and key in live:
            bm.free_seq(live.pop(key)[0])
        held = {}
        for table, _ in live.values():
            for b in table:
                held[b] = held.get(b, 0) + 1
        assert all(bm.ref[b] == c for b, c in held.items())
        assert all(bm.ref[b] == 0 for b in range(24) if b not in held)
        assert len(set(bm.free)) == len(bm.free) and not (set(bm.free) & set(held))
        assert len(bm.free) + len(bm.evictable) + len(held) == 24
    for table, _ in list(live.values()):
        bm.free_seq(table)
    assert bm.num_free() == 24 and all(r == 0 for r in bm.ref)


@FAST
@given(a=st.binary(max_size=3000), b=st.binary(max_size=3000))
def test_native_crc32_matches_zlib_and_combines(a, b):
    from lora_kernel_b200 import _rt
    assert _rt.crc32(a, 0) == zlib.crc32(a)
    assert _rt.crc32(b, _rt.crc32(a, 0)) == zlib.crc32(a + b)
    assert _rt.crc32_combine(zlib.crc32(a), zlib.crc32(b), len(b)) == zlib.crc32(a + b)


@FAST
@given(world=st.integers(1, 8), layers=st.integers(1, 3), kv=st.sampled_from([1, 2, 4]))
def test_zero_shards_cover_the_layout_once(world, layers, kv):
    """Every flat element of every layer group is owned by exactly one rank and
    extract_shard / owned ranges agree."""
    from lora_kernel_b200.config import TransformerConfig
    from lora_kernel_b200.parallel.zero import ShardLayout
    cfg = TransformerConfig(hidden_dim=64, num_heads=4, num_kv_heads=kv, head_dim=16, ff_dim=96,
                            vocab_size=50, num_layers=layers)
    L0 = ShardLayout(cfg, world, 0)
    cover = torch.zeros(L0.total, dtype=torch.int32)
    for r in range(world):
        L = ShardLayout(cfg, world, r)
        for gname in L.names:
            lo, hi = L.owned(gname)[0], L.owned(gname)[0] + L.chunk[gname]
            cover[lo:hi] += 1
    assert bool((cover == 1).all())
    full = torch.arange(L0.total, dtype=torch.float32)
    shards = [ShardLayout(cfg, world, r).extract_shard(full) for r in range(world)]
    assert sum(s.numel() for s in shards) == L0.total


@pytest.mark.parametrize("world", [2, 3, 4])
def test_zigzag_positions_are_a_permutation(world):
    from lora_kernel_b200.parallel.cp import shard_zigzag
    S = 2 * world * 5
    x = torch.arange(S)[None]
    got = torch.cat([shard_zigzag(x, r, world) for r in range(world)], 1)[0]
    assert sorted(got.tolist()) == list(range(S))


_json = st.recursive(st.none() | st.booleans() | st.integers(-10 ** 6, 10 ** 6) | st.floats(allow_nan=True) |
                     st.text(max_size=8), lambda c: st.lists(c, max_size=4) | st.dictionaries(st.text(max_size=6), c,
                                                                                           max_size=4), max_leaves=8)


@FAST
@given(body=st.dictionaries(st.sampled_from(["max_tokens", "temperature", "top_p", "stop", "seed", "n", "priority",
                                             "logprobs", "presence_penalty", "frequency_penalty",
                                             "stop_token_ids"]), _json,
                            max_size=6),
       ids=st.lists(st.integers(-5, 300), min_size=0, max_size=6))
def test_request_validator_never_crashes(body, ids):
    """Arbitrary JSON values in the sampling fields are either accepted or
    rejected with ValidationError (a 400), never another exception (a 500)."""
    from lora_kernel_b200.serve.security import InputValidator, ValidationError
    try:
        InputValidator(256).check(ids, body)
    except ValidationError:
        return
    # what the validator accepts, the server turns into sampling parameters without error
    from lora_kernel_b200.serve.engine import SamplingParams
    stop = body.get("stop") or ()
    SamplingParams(max_tokens=int(body.get("max_tokens", 16)), temperature=float(body.get("temperature", 0.0) or 0.0),
                   top_p=float(body.get("top_p", 1.0) or 1.0),
                   stop_token_ids=tuple(body.get("stop_token_ids") or ()),
                   stop_sequences=tuple(tuple(x.encode()) for x in ((stop,) if isinstance(stop, str) else stop)),
                   seed=body.get("seed"))
    int(body.get("priority", 0) or 0)
