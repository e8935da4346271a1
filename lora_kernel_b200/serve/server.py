"""OpenAI-compatible HTTP server with SSE streaming.

Routes
  POST /v1/completions        {prompt (str | [ids]), max_tokens, temperature, top_p, stream, stop}
  POST /v1/chat/completions   {messages: [{role, content}], ...}
  GET  /v1/models, /health, /metrics (Prometheus text)
Streaming responses are server-sent events: one `data: {json}\\n\\n` per token
(OpenAI `choices[0].text` / `choices[0].delta.content`, plus the reference
README's `token` and `index` fields) and a final `data: [DONE]\\n\\n`.

Middleware (optional): Bearer API keys or HS256 JWTs (stdlib hmac), a
token-bucket rate limit per client, and a JSON audit log line per request.

The engine runs in one background thread; HTTP handlers only enqueue requests
and await tokens pushed back through asyncio queues.

Reference: RestApiServer (include/api/rest_api.hpp:24-212, canned responses),
SSEStreamer (include/api/serving_production.hpp:111-131), JWTAuth /
TokenBucketLimiter (include/monitoring/production_monitoring.hpp:272-406).
"""
from __future__ import annotations

import asyncio
import base64
import hashlib
import hmac
import json
import threading
import time
import uuid
from typing import Dict, Optional

from aiohttp import web

from ..utils.logging import get_logger, log_fields
from ..utils.metrics import REGISTRY
from .engine import LLMEngine, SamplingParams
from .tokenizer import ByteTokenizer

log = get_logger("lora_kernel.serve")


# ------------------------------------------------------------------ security
def _b64url(b: bytes) -> str:
    return base64.urlsafe_b64encode(b).rstrip(b"=").decode()


def _b64url_dec(s: str) -> bytes:
    return base64.urlsafe_b64decode(s + "=" * (-len(s) % 4))


def jwt_encode(payload: dict, secret: str) -> str:
    head = _b64url(json.dumps({"alg": "HS256", "typ": "JWT"}).encode())
    body = _b64url(json.dumps(payload).encode())
    sig = hmac.new(secret.encode(), f"{head}.{body}".encode(), hashlib.sha256).digest()
    return f"{head}.{body}.{_b64url(sig)}"


def jwt_decode(token: str, secret: str, now: Optional[float] = None) -> Optional[dict]:
    try:
        head, body, sig = token.split(".")
        want = hmac.new(secret.encode(), f"{head}.{body}".encode(), hashlib.sha256).digest()
        if not hmac.compare_digest(want, _b64url_dec(sig)):
            return None
        payload = json.loads(_b64url_dec(body))
        if "exp" in payload and (now or time.time()) > payload["exp"]:
            return None
        return payload
    except Exception:
        return None


class TokenBucket:
    def __init__(self, rate: float, burst: float):
        self.rate, self.burst = rate, burst
        self.state: Dict[str, tuple] = {}

    def allow(self, key: str, now: Optional[float] = None) -> bool:
        now = time.monotonic() if now is None else now
        tokens, last = self.state.get(key, (self.burst, now))
        tokens = min(self.burst, tokens + (now - last) * self.rate)
        ok = tokens >= 1.0
        self.state[key] = (tokens - 1.0 if ok else tokens, now)
        return ok


# -------------------------------------------------------------- engine thread
class EngineWorker:
    """Runs engine.step() in a thread while there is work."""

    def __init__(self, engine: LLMEngine):
        self.engine = engine
        self.lock = threading.Lock()
        self.wake = threading.Event()
        self.stop = False
        self.m_ttft = REGISTRY.histogram("time_to_first_token_seconds", "TTFT")
        self.m_itl = REGISTRY.histogram("inter_token_latency_seconds", "inter-token latency")
        self.m_e2e = REGISTRY.histogram("e2e_request_latency_seconds", "request latency")
        self.m_out = REGISTRY.counter("generation_tokens_total", "generated tokens")
        self.m_in = REGISTRY.counter("prompt_tokens_total", "prompt tokens")
        self.m_req = REGISTRY.counter("requests_total", "finished requests")
        self.g_run = REGISTRY.gauge("num_requests_running", "running sequences")
        self.g_wait = REGISTRY.gauge("num_requests_waiting", "waiting requests")
        self.g_kv = REGISTRY.gauge("kv_cache_usage", "fraction of KV blocks in use")
        self.g_hit = REGISTRY.gauge("prefix_cache_hit_rate", "prefix cache block hit rate")
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def submit(self, prompt, params, on_token) -> int:
        with self.lock:
            rid = self.engine.add_request(prompt, params, on_token=on_token)
        self.m_in.inc(len(prompt))
        self.wake.set()
        return rid

    def _loop(self):
        while not self.stop:
            if not self.engine.has_work():
                self.wake.wait(0.05)
                self.wake.clear()
                continue
            with self.lock:
                finished = self.engine.step()
            e = self.engine
            self.g_run.set(len(e.running))
            self.g_wait.set(len(e.waiting))
            self.g_kv.set(e.blocks.usage())
            self.g_hit.set(e.blocks.stats.hit_rate)
            for r in finished:
                self.m_req.inc()
                self.m_out.inc(len(r.output))
                if r.first_token_time is not None:
                    self.m_ttft.observe(r.first_token_time - r.arrival)
                    self.m_e2e.observe(r.token_times[-1] - r.arrival)
                for a, b in zip(r.token_times, r.token_times[1:]):
                    self.m_itl.observe(b - a)


# ------------------------------------------------------------------- the app
def create_app(engine: LLMEngine, model_name: str = "lora-kernel-b200", api_keys=(),
               jwt_secret: str = "", rate_limit_rps: float = 0.0,
               tokenizer: Optional[ByteTokenizer] = None) -> web.Application:
    tok = tokenizer or ByteTokenizer(engine.cfg.vocab_size)
    worker = EngineWorker(engine)
    bucket = TokenBucket(rate_limit_rps, max(1.0, rate_limit_rps * 2)) if rate_limit_rps > 0 else None
    keys = set(api_keys)

    @web.middleware
    async def guard(request: web.Request, handler):
        client = request.remote or "?"
        if request.path.startswith("/v1/") and (keys or jwt_secret):
            auth = request.headers.get("Authorization", "")
            cred = auth[7:] if auth.startswith("Bearer ") else ""
            ok = cred in keys or (jwt_secret and jwt_decode(cred, jwt_secret) is not None)
            if not ok:
                return web.json_response({"error": {"message": "unauthorized", "type": "auth"}}, status=401)
            client = cred[:16]
        if bucket is not None and request.path.startswith("/v1/") and not bucket.allow(client):
            return web.json_response({"error": {"message": "rate limit exceeded", "type": "rate_limit"}},
                                     status=429)
        t0 = time.perf_counter()
        resp = await handler(request)
        log_fields(log, "request", path=request.path, status=resp.status, client=client,
                   ms=round((time.perf_counter() - t0) * 1e3, 2))
        return resp

    app = web.Application(middlewares=[guard])
    loop_holder = {}

    def _params(body) -> SamplingParams:
        stop = body.get("stop_token_ids") or ()
        return SamplingParams(max_tokens=int(body.get("max_tokens", 16)),
                              temperature=float(body.get("temperature", 0.0) or 0.0),
                              top_p=float(body.get("top_p", 1.0) or 1.0), stop_token_ids=tuple(stop))

    async def _run(prompt, params, stream: bool, request: web.Request, chat: bool):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        def on_token(r, t):
            loop.call_soon_threadsafe(q.put_nowait, (t, r.finished, r.finish_reason))
        rid = worker.submit(prompt, params, on_token)
        cid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:16]}"
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        if stream:
            resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
            await resp.prepare(request)
            idx = 0
            while True:
                t, done, reason = await q.get()
                text = tok.decode([t])
                choice = {"index": 0, "finish_reason": reason if done else None}
                if chat:
                    choice["delta"] = {"content": text}
                else:
                    choice["text"] = text
                chunk = {"id": cid, "object": obj + ".chunk" if chat else obj, "created": created,
                         "model": model_name, "choices": [choice], "token": t, "index": idx}
                await resp.write(f"data: {json.dumps(chunk)}\n\n".encode())
                idx += 1
                if done:
                    break
            await resp.write(b"data: [DONE]\n\n")
            await resp.write_eof()
            return resp
        out, reason = [], None
        while True:
            t, done, reason = await q.get()
            out.append(t)
            if done:
                break
        text = tok.decode(out)
        choice = {"index": 0, "finish_reason": reason}
        if chat:
            choice["message"] = {"role": "assistant", "content": text}
        else:
            choice["text"] = text
        return web.json_response({
            "id": cid, "object": obj, "created": created, "model": model_name, "choices": [choice],
            "usage": {"prompt_tokens": len(prompt), "completion_tokens": len(out),
                      "total_tokens": len(prompt) + len(out)},
            "token_ids": out})

    async def completions(request: web.Request):
        try:
            body = await request.json()
        except Exception:
            return web.json_response({"error": {"message": "invalid JSON", "type": "invalid_request"}}, status=400)
        prompt = body.get("prompt", "")
        ids = prompt if isinstance(prompt, list) else tok.encode(str(prompt))
        if not ids:
            return web.json_response({"error": {"message": "empty prompt", "type": "invalid_request"}}, status=400)
        try:
            return await _run(ids, _params(body), bool(body.get("stream")), request, chat=False)
        except ValueError as e:
            return web.json_response({"error": {"message": str(e), "type": "invalid_request"}}, status=400)

    async def chat(request: web.Request):
        try:
            body = await request.json()
        except Exception:
            return web.json_response({"error": {"message": "invalid JSON", "type": "invalid_request"}}, status=400)
        ids = tok.apply_chat_template(body.get("messages", []))
        try:
            return await _run(ids, _params(body), bool(body.get("stream")), request, chat=True)
        except ValueError as e:
            return web.json_response({"error": {"message": str(e), "type": "invalid_request"}}, status=400)

    async def models(_):
        return web.json_response({"object": "list", "data": [{"id": model_name, "object": "model",
                                                               "owned_by": "lora_kernel_b200"}]})

    async def health(_):
        return web.json_response({"status": "healthy", "running": len(engine.running),
                                  "waiting": len(engine.waiting)})

    async def metrics(_):
        return web.Response(text=REGISTRY.exposition(), content_type="text/plain")

    app.router.add_post("/v1/completions", completions)
    app.router.add_post("/v1/chat/completions", chat)
    app.router.add_get("/v1/models", models)
    app.router.add_get("/health", health)
    app.router.add_get("/metrics", metrics)

    async def on_shutdown(_):
        worker.stop = True
        worker.wake.set()
    app.on_shutdown.append(on_shutdown)
    app["worker"] = worker
    return app


def serve(engine: LLMEngine, host: str = "127.0.0.1", port: int = 8080, **kw) -> None:
    web.run_app(create_app(engine, **kw), host=host, port=port, print=None)
