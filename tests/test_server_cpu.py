"""HTTP contract of the OpenAI-compatible server (CPU, fake engine)."""
import asyncio
import json
import time

import pytest
from aiohttp.test_utils import TestClient, TestServer

from lora_kernel_b200.serve.kv_cache import CacheStats
from lora_kernel_b200.serve.server import TokenBucket, create_app, jwt_decode, jwt_encode


class _Cfg:
    vocab_size = 256


class _Blocks:
    stats = CacheStats()

    def usage(self):
        return 0.0


class FakeEngine:
    """Echoes the prompt's bytes back one token per step."""

    def __init__(self):
        self.cfg = _Cfg()
        self.blocks = _Blocks()
        self.running, self.waiting = [], []
        self.n = 0

    def add_request(self, prompt, params, on_token=None, priority=0):
        class R:
            pass
        r = R()
        self.priorities = getattr(self, "priorities", []) + [priority]
        r.prompt, r.params, r.on_token = list(prompt), params, on_token
        r.output, r.finished, r.finish_reason = [], False, None
        r.arrival, r.first_token_time, r.token_times = time.perf_counter(), None, []
        self.waiting.append(r)
        self.n += 1
        return self.n

    def has_work(self):
        return bool(self.running or self.waiting)

    def step(self):
        for r in self.waiting:
            r.scheduled_time = time.perf_counter()
        self.running += self.waiting
        self.waiting = []
        done = []
        for r in list(self.running):
            t = r.prompt[len(r.output) % len(r.prompt)]
            r.output.append(t)
            now = time.perf_counter()
            r.token_times.append(now)
            r.first_token_time = r.first_token_time or now
            if len(r.output) >= r.params.max_tokens:
                r.finished, r.finish_reason = True, "length"
            for sq in getattr(r.params, "stop_sequences", ()):
                if sq and tuple(r.output[-len(sq):]) == tuple(sq):
                    r.finished, r.finish_reason = True, "stop"
            r.on_token(r, t)
            if r.finished:
                self.running.remove(r)
                done.append(r)
        return done


def _run(coro_fn, **kw):
    async def main():
        app = create_app(FakeEngine(), **kw)
        async with TestClient(TestServer(app)) as client:
            return await coro_fn(client)
    return asyncio.run(main())


def test_completion_json_schema():
    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": "hi!", "max_tokens": 5})
        assert r.status == 200
        d = await r.json()
        assert d["object"] == "text_completion" and d["choices"][0]["text"] == "hi!hi"
        assert d["choices"][0]["finish_reason"] == "length"
        assert d["usage"] == {"prompt_tokens": 3, "completion_tokens": 5, "total_tokens": 8}
        r = await c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "yo"}],
                                                      "max_tokens": 3})
        d = await r.json()
        assert d["object"] == "chat.completion" and d["choices"][0]["message"]["role"] == "assistant"
        r = await c.get("/v1/models")
        assert (await r.json())["data"][0]["id"]
        r = await c.get("/health")
        assert (await r.json())["status"] == "healthy"
        r = await c.post("/v1/completions", data="not json")
        assert r.status == 400
        r = await c.get("/metrics")
        text = await r.text()
        count = [ln for ln in text.splitlines() if ln.startswith("lora_kernel_request_queue_time_seconds_count")]
        assert count and float(count[0].split()[-1]) >= 2, text
        assert "lora_kernel_preemptions_total" in text
        r = await c.get("/alerts")
        assert r.status == 200 and (await r.json())["firing"] == []
    _run(go)


def test_sse_stream_framing():
    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": [65, 66], "max_tokens": 4, "stream": True})
        assert r.headers["Content-Type"].startswith("text/event-stream")
        body = (await r.read()).decode()
        events = [e for e in body.split("\n\n") if e]
        assert all(e.startswith("data: ") for e in events)
        assert events[-1] == "data: [DONE]"
        chunks = [json.loads(e[6:]) for e in events[:-1]]
        assert [ch["token"] for ch in chunks] == [65, 66, 65, 66]
        assert [ch["index"] for ch in chunks] == [0, 1, 2, 3]
        assert chunks[-1]["choices"][0]["finish_reason"] == "length"
        assert "".join(ch["choices"][0]["text"] for ch in chunks) == "ABAB"
        m = await (await c.get("/metrics")).text()
        assert "lora_kernel_generation_tokens_total" in m and '_bucket{le="+Inf"}' in m
    _run(go)


def test_auth_and_rate_limit():
    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": "x", "max_tokens": 1})
        assert r.status == 401
        r = await c.post("/v1/completions", json={"prompt": "x", "max_tokens": 1},
                         headers={"Authorization": "Bearer k1"})
        assert r.status == 200
        tok = jwt_encode({"sub": "u", "exp": time.time() + 60}, "s3cret")
        r = await c.post("/v1/completions", json={"prompt": "x", "max_tokens": 1},
                         headers={"Authorization": f"Bearer {tok}"})
        assert r.status == 200
        codes = []
        for _ in range(6):
            r = await c.post("/v1/completions", json={"prompt": "x", "max_tokens": 1},
                             headers={"Authorization": "Bearer k1"})
            codes.append(r.status)
        assert 429 in codes
    _run(go, api_keys=("k1",), jwt_secret="s3cret", rate_limit_rps=1.0)


def test_jwt_and_bucket_units():
    t = jwt_encode({"sub": "a", "exp": 100.0}, "k")
    assert jwt_decode(t, "k", now=50.0)["sub"] == "a"
    assert jwt_decode(t, "k", now=150.0) is None
    assert jwt_decode(t, "wrong", now=50.0) is None
    b = TokenBucket(rate=1.0, burst=2.0)
    assert b.allow("c", 0.0) and b.allow("c", 0.0) and not b.allow("c", 0.0)
    assert b.allow("c", 1.5)


# ------------------------------------------------------- policies and WebSocket
from lora_kernel_b200.serve.security import (AuditLog, InputValidator, PIIMasker,  # noqa: E402
                                             RequestSigner, RoleAccess, ValidationError)


def test_websocket_streaming():
    async def go(c):
        ws = await c.ws_connect("/v1/ws")
        await ws.send_json({"prompt": [72, 73], "max_tokens": 3})
        msgs = []
        while True:
            m = await ws.receive_json()
            msgs.append(m)
            if m.get("done"):
                break
        assert [m["token"] for m in msgs[:-1]] == [72, 73, 72]
        assert [m["index"] for m in msgs[:-1]] == [0, 1, 2]
        assert "".join(m["text"] for m in msgs[:-1]) == "HIH"
        assert msgs[-1]["finish_reason"] == "length" and msgs[-1]["usage"]["completion_tokens"] == 3
        # a bad request on the same socket gets an error message, the socket stays usable
        await ws.send_json({"prompt": [999], "max_tokens": 1})
        assert "error" in await ws.receive_json()
        await ws.send_json({"prompt": "ok", "max_tokens": 1})
        assert (await ws.receive_json())["token"] == ord("o")
        await ws.close()
    _run(go)


def test_input_validation_rejects_bad_requests():
    async def go(c):
        for body in ({"prompt": [1, 2, 300], "max_tokens": 2}, {"prompt": "x", "max_tokens": 0},
                     {"prompt": "x", "temperature": -1}, {"prompt": "x", "top_p": 1.5},
                     {"prompt": ""}, {"prompt": "x" * 50}):
            r = await c.post("/v1/completions", json=body)
            assert r.status == 400, body
    _run(go, validator=InputValidator(256, max_prompt_tokens=40))


def test_pii_masking_in_responses():
    m = PIIMasker()
    assert m.mask("mail bob.smith@example.com now") == "mail [EMAIL] now"
    assert m.mask("ssn 123-45-6789.") == "ssn [SSN]."
    assert m.mask("card 4111 1111 1111 1111 ok") == "card [CARD] ok"
    assert m.mask("num 4111 1111 1111 1112 ok") != "num [CARD] ok"  # fails the Luhn check
    assert m.mask("call (555) 123-4567") == "call [PHONE]"
    secret = "reach me at a@b.io please"

    async def go(c):
        ids = [ord(ch) for ch in secret]
        r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": len(ids)})
        assert (await r.json())["choices"][0]["text"] == "reach me at [EMAIL] please"
        r = await c.post("/v1/completions", json={"prompt": ids, "max_tokens": len(ids), "stream": True})
        events = [e for e in (await r.read()).decode().split("\n\n") if e and e != "data: [DONE]"]
        text = "".join(json.loads(e[6:])["choices"][0]["text"] for e in events)
        assert text == "reach me at [EMAIL] please"
    _run(go, pii_filter=True)


def test_roles_signatures_and_audit(tmp_path):
    roles = RoleAccess({"admin": ["*"], "user": ["/v1/completions", "/v1/chat", "/v1/ws"]},
                       key_roles={"k-admin": "admin", "k-user": "user"})
    signer = RequestSigner("sig")
    audit = AuditLog(str(tmp_path / "audit.jsonl"))

    async def go(c):
        body = json.dumps({"prompt": "x", "max_tokens": 1}).encode()
        h = {"Authorization": "Bearer k-user", "Content-Type": "application/json", **signer.sign(body)}
        assert (await c.post("/v1/completions", data=body, headers=h)).status == 200
        bad = dict(h, **{"X-Signature": "0" * 64})
        assert (await c.post("/v1/completions", data=body, headers=bad)).status == 401
        stale = dict(h, **signer.sign(body, ts=time.time() - 3600))
        assert (await c.post("/v1/completions", data=body, headers=stale)).status == 401
        assert (await c.get("/v1/models", headers={"Authorization": "Bearer k-user"})).status == 403
        assert (await c.get("/v1/models", headers={"Authorization": "Bearer k-admin"})).status == 200
        tok = jwt_encode({"sub": "u", "role": "admin", "exp": time.time() + 60}, "j")
        assert (await c.get("/v1/models", headers={"Authorization": f"Bearer {tok}"})).status == 200
    _run(go, api_keys=("k-admin", "k-user"), jwt_secret="j", roles=roles, signing_secret="sig", audit=audit)
    lines = [json.loads(x) for x in open(tmp_path / "audit.jsonl")]
    assert [x["status"] for x in lines] == [200, 401, 401, 403, 200, 200]
    assert [x["role"] for x in lines] == ["user"] * 4 + ["admin"] * 2
    with pytest.raises(ValidationError):
        InputValidator(10).check([11], {})


def test_replica_pool_policies():
    from lora_kernel_b200.serve.engine import SamplingParams
    from lora_kernel_b200.serve.replicas import ReplicaPool
    done = []
    rr = ReplicaPool([FakeEngine() for _ in range(3)], policy="round_robin")
    for k in range(9):
        rr.submit([65 + k], SamplingParams(max_tokens=2), lambda r, t: done.append(r) if r.finished else None)
    assert rr.routed == [3, 3, 3]
    aff = ReplicaPool([FakeEngine() for _ in range(4)], policy="prefix_affinity", affinity_tokens=4, slack=100)
    picks = {aff.pick([1, 2, 3, 4, k]) for k in range(10)}
    assert len(picks) == 1  # shared 4-token prefix -> one replica
    ll = ReplicaPool([FakeEngine() for _ in range(2)], policy="least_loaded")
    ll.outstanding = [5, 1]
    assert ll.pick([1]) == 1
    deadline = time.time() + 10
    while len(done) < 9 and time.time() < deadline:
        time.sleep(0.01)
    assert len(done) == 9 and rr.outstanding == [0, 0, 0]
    for p in (rr, aff, ll):
        p.shutdown()


def test_server_over_replicas():
    engines = [FakeEngine(), FakeEngine()]

    async def go(c):
        for k in range(4):
            r = await c.post("/v1/completions", json={"prompt": [70 + k], "max_tokens": 2})
            assert r.status == 200
        assert (await (await c.get("/health")).json())["status"] == "healthy"

    async def main():
        app = create_app(engines, replica_policy="round_robin")
        async with TestClient(TestServer(app)) as client:
            await go(client)
    asyncio.run(main())
    assert engines[0].n == 2 and engines[1].n == 2


def test_training_flops_mfu_and_metrics_file(tmp_path):
    """Model FLOPs per token against a hand count for the 1.1B shape, MFU
    arithmetic, and the JSONL file / gauges of TrainMetrics."""
    import json as _json
    from lora_kernel_b200.config import get_preset
    from lora_kernel_b200.utils.metrics import Registry, TrainMetrics, mfu, train_flops_per_token
    cfg = get_preset("llama-1.1b-zero3").model
    D, F, L, V = 2048, 5632, 22, 32000
    gemm_params = L * (D * 2560 + 2048 * D + 3 * D * F) + D * V
    want = 6 * gemm_params + L * 6 * 2048 * 32 * 64
    assert train_flops_per_token(cfg, 2048) == want
    assert abs(mfu(100_000.0, 1e10, 2, peak_tflops=1000.0) - 0.5) < 1e-12
    reg = Registry("t_")
    path = str(tmp_path / "m.jsonl")
    m = TrainMetrics(path, reg)
    m.record({"step": 1, "loss": 2.5, "tokens_per_s": 10.0, "mfu": 0.4})
    m.record({"step": 2, "loss": 2.0, "tokens_per_s": 12.0, "mfu": 0.5, "grad_norm": 1.5})
    m.close()
    lines = [_json.loads(x) for x in open(path)]
    assert [r["step"] for r in lines] == [1, 2] and lines[1]["grad_norm"] == 1.5
    text = reg.exposition()
    assert "t_train_loss 2.0" in text and "t_train_mfu 0.5" in text and "t_train_step 2.0" in text


def test_stop_trimmer_holds_back_and_drops_the_stop_sequence():
    from lora_kernel_b200.serve.server import StopTrimmer
    tr = StopTrimmer([(7, 8, 9), (5,)])
    got = []
    for t in [1, 2, 7, 8]:
        got += tr.push(t, False, None)
    assert got == [1, 2]                      # 7, 8 might start the stop sequence
    got += tr.push(9, True, "stop")
    assert got == [1, 2]                      # ... and did
    tr = StopTrimmer([(7, 8, 9)])
    assert tr.push(7, False, None) + tr.push(8, False, None) + tr.push(3, True, "length") == [7, 8, 3]
    assert StopTrimmer().push(4, False, None) == [4]


def test_stop_strings_over_http():
    """`stop` ends generation at the first occurrence and is left out of the
    text, in plain and streamed responses; bad `stop` values are rejected."""
    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": "abcXYdef", "max_tokens": 30, "stop": ["XY", "zz"]})
        d = await r.json()
        assert d["choices"][0]["text"] == "abc" and d["choices"][0]["finish_reason"] == "stop", d
        assert d["usage"]["completion_tokens"] == 5
        r = await c.post("/v1/completions", json={"prompt": "abcXYdef", "max_tokens": 30, "stop": "XY",
                                                  "stream": True})
        body = (await r.read()).decode()
        chunks = [json.loads(x[6:]) for x in body.split("\n\n") if x.startswith("data: {")]
        assert "".join(ch["choices"][0]["text"] for ch in chunks) == "abc"
        assert chunks[-1]["choices"][0]["finish_reason"] == "stop"
        r = await c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 3, "stop": ["a", "b", "c", "d", "e"]})
        assert r.status == 400
    _run(go)


def test_seed_validation():
    from lora_kernel_b200.serve.security import InputValidator, ValidationError
    v = InputValidator(256)
    v.check([1], {"seed": 5})
    for bad in (-1, 2 ** 63, "7", True, 1.5):
        with pytest.raises(ValidationError, match="seed"):
            v.check([1], {"seed": bad})


def test_unimplemented_openai_options_are_refused():
    from lora_kernel_b200.serve.security import InputValidator, ValidationError
    v = InputValidator(256)
    v.check([1], {"n": 1, "presence_penalty": 0, "logprobs": None})
    for body, msg in [({"n": 2}, "n must be 1"), ({"frequency_penalty": 0.5}, "frequency_penalty"),
                      ({"logprobs": 5}, "logprobs")]:
        with pytest.raises(ValidationError, match=msg):
            v.check([1], body)


def test_device_metrics_from_a_fake_nvml():
    """DeviceMetrics reads NVML (read-only queries) into gpu-labelled gauges;
    without CUDA or NVML the gauges stay at 0 and nothing raises."""
    from types import SimpleNamespace
    from lora_kernel_b200.utils.metrics import DeviceMetrics, Registry

    class FakeNVML:
        NVML_CLOCK_SM, NVML_TEMPERATURE_GPU = 1, 0

        def nvmlInit(self):
            pass

        def nvmlDeviceGetHandleByIndex(self, i):
            return ("h", i)

        def nvmlDeviceGetUtilizationRates(self, h):
            return SimpleNamespace(gpu=87, memory=40)

        def nvmlDeviceGetMemoryInfo(self, h):
            return SimpleNamespace(used=123 * 2 ** 20, total=180 * 2 ** 30)

        def nvmlDeviceGetClockInfo(self, h, kind):
            return 1845

        def nvmlDeviceGetPowerUsage(self, h):
            return 987654   # milliwatts

        def nvmlDeviceGetTemperature(self, h, kind):
            return 61

    reg = Registry("t_")
    got = DeviceMetrics(3, reg, nvml=FakeNVML()).update()
    assert got["gpu_utilization_percent"] == 87 and got["gpu_sm_clock_mhz"] == 1845
    text = reg.exposition()
    assert 't_gpu_power_watts{gpu="3"} 987.654' in text and 't_gpu_temperature_celsius{gpu="3"} 61.0' in text
    assert text.count("# TYPE t_gpu_power_watts gauge") == 1
    DeviceMetrics(1, reg).update()      # second GPU's series under the same names, one header each
    text = reg.exposition()
    assert text.count("# TYPE t_gpu_power_watts gauge") == 1 and 't_gpu_power_watts{gpu="1"}' in text

    class Broken(FakeNVML):
        def nvmlInit(self):
            raise RuntimeError("no driver")
    assert DeviceMetrics(0, Registry("u_"), nvml=Broken()).update() == {}


def test_text_sanitizer_and_inflight_limit():
    from lora_kernel_b200.serve.security import ConnectionLimiter, sanitize_text
    assert sanitize_text("a\x00b\x1bc\td\ne\x7f") == "a b c\td\ne "
    assert len(sanitize_text("x" * 10, max_chars=4)) == 4
    lim = ConnectionLimiter(2)
    assert lim.acquire("a") and lim.acquire("a") and not lim.acquire("a") and lim.acquire("b")
    lim.release("a")
    assert lim.acquire("a")
    assert all(ConnectionLimiter(0).acquire("z") for _ in range(100))

    async def go(c):
        # control characters become spaces before tokenization (the echo engine returns the prompt)
        r = await c.post("/v1/completions", json={"prompt": "a\x01b", "max_tokens": 3})
        assert (await r.json())["choices"][0]["text"] == "a b"
        for _ in range(3):   # the limit is released after every request
            r = await c.post("/v1/completions", json={"prompt": "ok", "max_tokens": 2})
            assert r.status == 200
    _run(go, max_inflight_per_client=1)


def test_alert_rules():
    from lora_kernel_b200.utils.metrics import AlertManager, AlertRule, Registry
    reg = Registry("a_")
    g = reg.gauge("kv_cache_usage")
    h = reg.histogram("time_to_first_token_seconds")
    am = AlertManager([AlertRule("kv_full", "kv_cache_usage", ">=", 0.95, for_s=5.0),
                       AlertRule("slow_ttft", "time_to_first_token_seconds", ">", 0.5, quantile=0.9),
                       AlertRule("nothing", "missing_metric", ">", 0)], reg)
    g.set(0.97)
    assert am.check(now=0.0) == []                      # must hold for 5 s
    assert [a["name"] for a in am.check(now=6.0)] == ["kv_full"]
    for v in [0.1] * 5 + [0.9] * 5:
        h.observe(v)
    assert {a["name"] for a in am.check(now=7.0)} == {"kv_full", "slow_ttft"}
    g.set(0.5)
    assert [a["name"] for a in am.check(now=8.0)] == ["slow_ttft"] and "kv_full" not in am.firing
    with pytest.raises(ValueError):
        AlertRule("x", "m", "!=", 1)


def _word_tokenizer(tmp_path, template=True):
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import Whitespace
    words = ["<unk>", "</s>", "hello", "world", "user", "assistant", ":", "hi", "there"]
    t = Tokenizer(WordLevel({w: i for i, w in enumerate(words)}, unk_token="<unk>"))
    t.pre_tokenizer = Whitespace()
    path = tmp_path / "tokenizer.json"
    t.save(str(path))
    if template:
        (tmp_path / "tokenizer_config.json").write_text(json.dumps({
            "eos_token": "</s>",
            "chat_template": "{% for m in messages %}{{ m['role'] }} : {{ m['content'] }} {% endfor %}"
                             "{% if add_generation_prompt %}assistant :{% endif %}"}))
    return str(path)


def test_hf_tokenizer_file(tmp_path):
    from lora_kernel_b200.serve.tokenizer import HFTokenizer
    tok = HFTokenizer(_word_tokenizer(tmp_path))
    assert tok.encode("hello world") == [2, 3] and tok.decode([2, 3]) == "hello world"
    assert tok.eos_token_id == 1 and tok.stop_ids == (1,)
    assert tok.apply_chat_template([{"role": "user", "content": "hi there"}]) == [4, 6, 7, 8, 5, 6]
    plain = HFTokenizer(_word_tokenizer(tmp_path / "x" if (tmp_path / "x").mkdir() is None else tmp_path,
                                        template=False))
    assert plain.stop_ids == () and plain.apply_chat_template([{"role": "user", "content": "hi"}])[:3] == [4, 6, 7]

    async def go(c):
        r = await c.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 3})
        d = await r.json()
        assert d["choices"][0]["text"] == "hello world hello" and d["usage"]["prompt_tokens"] == 2
    _run(go, tokenizer=tok)


def test_dashboard_renders_the_exposition():
    from lora_kernel_b200.utils.dashboard import histogram_quantile, parse_prometheus, render
    from lora_kernel_b200.utils.metrics import Registry
    reg = Registry("lora_kernel_")
    reg.counter("requests_total").inc(3)
    reg.counter("generation_tokens_total").inc(120)
    reg.gauge("kv_cache_usage").set(0.25)
    h = reg.histogram("time_to_first_token_seconds")
    for v in (0.004, 0.02, 0.02, 0.3):
        h.observe(v)
    reg.gauge("gpu_utilization_percent", labels={"gpu": "0"}).set(91)
    m = parse_prometheus(reg.exposition())
    assert m[("lora_kernel_requests_total", ())] == 3.0
    assert m[("lora_kernel_gpu_utilization_percent", (("gpu", "0"),))] == 91.0
    assert histogram_quantile(m, "lora_kernel_time_to_first_token_seconds", 0.5) == 0.025
    text = render(m, [{"name": "kv", "metric": "kv_cache_usage", "op": ">", "threshold": 0.2, "value": 0.25}])
    assert "requests 3" in text and "KV cache 25.0%" in text and "TTFT" in text and "GPU 0: util 91%" in text
    assert "ALERT kv" in text


def test_priority_reaches_the_engine():
    from lora_kernel_b200.serve.security import InputValidator, ValidationError
    eng = FakeEngine()

    async def main():
        app = create_app(eng)
        async with TestClient(TestServer(app)) as c:
            r = await c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 2, "priority": -5})
            assert r.status == 200
            r = await c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 2})
            assert r.status == 200
            r = await c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 2, "priority": 5000})
            assert r.status == 400
    asyncio.run(main())
    assert eng.priorities == [-5, 0]
    with pytest.raises(ValidationError, match="priority"):
        InputValidator(256).check([1], {"priority": "high"})


class SlowEngine(FakeEngine):
    """FakeEngine that takes 10 ms a step, refuses prompt + max_tokens over 64
    (the engine's max_model_len check) and can abort requests."""

    def add_request(self, prompt, params, on_token=None, priority=0):
        if len(prompt) + params.max_tokens > 64:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        rid = super().add_request(prompt, params, on_token, priority)
        self.waiting[-1].req_id = rid
        return rid

    def step(self):
        time.sleep(0.01)
        return super().step()

    def abort_request(self, rid):
        for lst in (self.running, self.waiting):
            for r in list(lst):
                if r.req_id == rid:
                    lst.remove(r)
                    self.aborted = getattr(self, "aborted", []) + [rid]
                    return True
        return False


def test_client_disconnect_aborts_the_request():
    """A streaming client that goes away mid-stream stops its request: the
    engine has no work left and the request was aborted, not decoded on."""
    eng = SlowEngine()

    async def main():
        app = create_app(eng)
        async with TestClient(TestServer(app)) as c:
            r = await c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 60, "stream": True})
            assert r.status == 200
            await r.content.readline()  # first chunk arrived
            r.close()  # drop the connection
            for _ in range(200):
                await asyncio.sleep(0.02)
                if not eng.has_work():
                    break
            assert not eng.has_work()
            assert getattr(eng, "aborted", []) == [1]
    asyncio.run(main())


def test_websocket_disconnect_aborts_and_engine_errors_are_messages():
    eng = SlowEngine()

    async def main():
        app = create_app(eng)
        async with TestClient(TestServer(app)) as c:
            ws = await c.ws_connect("/v1/ws")
            # the engine refuses prompt + max_tokens over its limit: an error message, not a closed socket
            await ws.send_json({"prompt": "ab", "max_tokens": 63})
            assert "max_model_len" in (await ws.receive_json())["error"]["message"]
            await ws.send_json({"prompt": "ab", "max_tokens": 2})
            msgs = [await ws.receive_json() for _ in range(3)]
            assert msgs[-1]["done"]
            await ws.send_json({"prompt": "ab", "max_tokens": 60})
            await ws.receive_json()
            await ws.close()
            for _ in range(200):
                await asyncio.sleep(0.02)
                if not eng.has_work():
                    break
            assert not eng.has_work() and len(getattr(eng, "aborted", [])) == 1
    asyncio.run(main())


def test_boolean_max_tokens_and_token_ids_are_rejected():
    from lora_kernel_b200.serve.security import InputValidator, ValidationError
    v = InputValidator(256)
    with pytest.raises(ValidationError, match="max_tokens"):
        v.check([1], {"max_tokens": True})
    with pytest.raises(ValidationError, match="token id"):
        v.check([True], {})
