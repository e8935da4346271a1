"""OpenAI-compatible HTTP server with SSE streaming.

Routes
  POST /v1/completions        {prompt (str | [ids]), max_tokens, temperature, top_p, stream, stop}
  POST /v1/chat/completions   {messages: [{role, content}], ...}
  GET  /v1/models, /health, /metrics (Prometheus text), /alerts (firing alert rules)
  GET  /v1/ws                 WebSocket: JSON requests in, one JSON message per token out
Streaming responses are server-sent events: one `data: {json}\\n\\n` per token
(OpenAI `choices[0].text` / `choices[0].delta.content`, plus the reference
README's `token` and `index` fields) and a final `data: [DONE]\\n\\n`.

Middleware (optional): Bearer API keys or HS256 JWTs (stdlib hmac), role-based
path access, HMAC request signatures, a token-bucket rate limit per client, PII
masking of generated text and an audit log (serve/security.py); requests are
validated before they reach the engine.

The engine runs in one background thread; HTTP handlers only enqueue requests
and await tokens pushed back through asyncio queues.

Reference: RestApiServer (include/api/rest_api.hpp:24-212, canned responses),
SSEStreamer (include/api/serving_production.hpp:111-131), WebSocketStreamer
(include/api/websocket_streaming.hpp:9-33, a local queue with no socket), JWTAuth /
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
from collections import deque
from typing import Dict, List, Optional

import torch
from aiohttp import WSMsgType, web

from ..utils.logging import get_logger, log_fields
from ..utils.metrics import REGISTRY, AlertManager, AlertRule, DeviceMetrics
from .engine import LLMEngine, SamplingParams
from .security import (AuditLog, ConnectionLimiter, InputValidator, PIIMasker, RequestSigner, RoleAccess,
                       sanitize_text)
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
        self.m_queue = REGISTRY.histogram("request_queue_time_seconds", "arrival to first scheduling")
        self.m_pre = REGISTRY.counter("preemptions_total", "sequences preempted for KV blocks")
        self._pre_seen = 0
        self.m_out = REGISTRY.counter("generation_tokens_total", "generated tokens")
        self.m_in = REGISTRY.counter("prompt_tokens_total", "prompt tokens")
        self.m_req = REGISTRY.counter("requests_total", "finished requests")
        self.g_run = REGISTRY.gauge("num_requests_running", "running sequences")
        self.g_wait = REGISTRY.gauge("num_requests_waiting", "waiting requests")
        self.g_kv = REGISTRY.gauge("kv_cache_usage", "fraction of KV blocks in use")
        self.g_hit = REGISTRY.gauge("prefix_cache_hit_rate", "prefix cache block hit rate")
        self._aborts: deque = deque()
        self._gate = threading.Lock()
        self._callers = 0
        self.thread = threading.Thread(target=self._loop, daemon=True)
        self.thread.start()

    def running(self) -> int:
        return len(self.engine.running)

    def waiting(self) -> int:
        return len(self.engine.waiting)

    def shutdown(self) -> None:
        self.stop = True
        self.wake.set()

    def submit(self, prompt, params, on_token, priority: int = 0) -> int:
        # announce the caller so the worker lets go of the lock between steps
        # (a plain lock is not fair: the worker would take it straight back)
        with self._gate:
            self._callers += 1
        try:
            with self.lock:
                rid = (self.engine.add_request(prompt, params, on_token=on_token, priority=priority) if priority
                       else self.engine.add_request(prompt, params, on_token=on_token))
        finally:
            with self._gate:
                self._callers -= 1
        self.m_in.inc(len(prompt))
        self.wake.set()
        return rid

    def abort(self, rid: int, on_done=None) -> None:
        """Stop a request whose client is gone (frees its KV blocks).  Does not
        block: the worker applies it before its next step and then calls
        on_done(aborted) with whether the request was still unfinished."""
        self._aborts.append((rid, on_done))
        self.wake.set()

    def _apply_aborts(self) -> None:
        while self._aborts:
            rid, cb = self._aborts.popleft()
            ok = self.engine.abort_request(rid)
            if cb is not None:
                cb(ok)

    def _loop(self):
        # kernels launch on the current device's stream: make it the engine's
        dev = getattr(getattr(self.engine, "runner", None), "device", None)
        if isinstance(dev, torch.device) and dev.type == "cuda":
            torch.cuda.set_device(dev)
        while not self.stop:
            if self._aborts:
                with self.lock:
                    self._apply_aborts()
            if not self.engine.has_work():
                self.wake.wait(0.05)
                self.wake.clear()
                continue
            while self._callers:  # a submit() is waiting for the lock
                time.sleep(0.0002)
            with self.lock:
                finished = self.engine.step()
            e = self.engine
            self.g_run.set(len(e.running))
            self.g_wait.set(len(e.waiting))
            self.g_kv.set(e.blocks.usage())
            self.g_hit.set(e.blocks.stats.hit_rate)
            pre = getattr(e, "stats", {}).get("preemptions", 0)
            if pre > self._pre_seen:
                self.m_pre.inc(pre - self._pre_seen)
                self._pre_seen = pre
            for r in finished:
                self.m_req.inc()
                self.m_out.inc(len(r.output))
                if getattr(r, "scheduled_time", None) is not None:
                    self.m_queue.observe(r.scheduled_time - r.arrival)
                if r.first_token_time is not None:
                    self.m_ttft.observe(r.first_token_time - r.arrival)
                    self.m_e2e.observe(r.token_times[-1] - r.arrival)
                for a, b in zip(r.token_times, r.token_times[1:]):
                    self.m_itl.observe(b - a)


class StopTrimmer:
    """Releases generated tokens so that a matched stop sequence never reaches
    the client: while a request runs, the last (longest stop length - 1)
    tokens are held back (they could be the start of a stop sequence); when it
    finishes with reason "stop" and its output ends with a stop sequence, that
    sequence is dropped and the rest released (OpenAI `stop` semantics)."""

    def __init__(self, stop_sequences=()):
        self.stops = [tuple(sq) for sq in stop_sequences if sq]
        self.hold = max((len(sq) for sq in self.stops), default=1) - 1
        self.pending: List[int] = []

    def push(self, tok_id: int, done: bool, reason: Optional[str]) -> List[int]:
        self.pending.append(tok_id)
        if done:
            if reason == "stop":
                for sq in self.stops:
                    n = len(sq)
                    if len(self.pending) >= n and tuple(self.pending[-n:]) == sq:
                        del self.pending[-n:]
                        break
            out, self.pending = self.pending, []
            return out
        n = max(0, len(self.pending) - self.hold)
        out, self.pending = self.pending[:n], self.pending[n:]
        return out


# alert rules the server evaluates at GET /alerts unless create_app is given its own
DEFAULT_ALERTS = (
    AlertRule("kv_cache_nearly_full", "kv_cache_usage", ">=", 0.95, for_s=30.0),
    AlertRule("ttft_p90_over_2s", "time_to_first_token_seconds", ">", 2.0, quantile=0.9),
    AlertRule("requests_queued", "num_requests_waiting", ">", 64, for_s=30.0),
)


# ------------------------------------------------------------------- the app
WORKER_KEY = web.AppKey("worker", object)


def create_app(engine: LLMEngine, model_name: str = "lora-kernel-b200", api_keys=(),
               jwt_secret: str = "", rate_limit_rps: float = 0.0,
               tokenizer=None, *,
               validator: Optional[InputValidator] = None, pii_filter: bool = False,
               roles: Optional[RoleAccess] = None, signing_secret: str = "",
               audit: Optional[AuditLog] = None, replica_policy: str = "least_loaded",
               sanitize_input: bool = True, max_inflight_per_client: int = 0,
               alert_rules=None) -> web.Application:
    """OpenAI-compatible app.  Optional policies: API keys / HS256 JWT bearer
    auth, token-bucket rate limit per client, role-based path access (JWT
    `role` claim or the key's role), HMAC request signatures, PII masking of
    generated text, an audit log, a per-client limit on requests in flight
    (429 beyond it); prompt text has its control characters replaced
    (sanitize_input) and every request is validated (prompt length, token
    ids, sampling parameters) before it reaches the engine.  `engine`
    may be a list of engines: requests are then routed over the replicas by
    `replica_policy`."""
    engines = list(engine) if isinstance(engine, (list, tuple)) else [engine]
    if isinstance(engine, (list, tuple)):
        # several replicas behind one server (serve/replicas.py)
        from .replicas import ReplicaPool
        worker = ReplicaPool(engine, policy=replica_policy)
        engine = engine[0]
    else:
        worker = EngineWorker(engine)
    # per-GPU memory / utilisation gauges, refreshed at each /metrics scrape
    gpus = sorted({d.index for d in (getattr(getattr(e, "runner", None), "device", None) for e in engines)
                   if isinstance(d, torch.device) and d.type == "cuda" and d.index is not None})
    dev_metrics = [DeviceMetrics(i) for i in gpus]
    tok = tokenizer or ByteTokenizer(engine.cfg.vocab_size)
    bucket = TokenBucket(rate_limit_rps, max(1.0, rate_limit_rps * 2)) if rate_limit_rps > 0 else None
    keys = set(api_keys)
    validator = validator or InputValidator(engine.cfg.vocab_size)
    masker = PIIMasker() if pii_filter else None
    signer = RequestSigner(signing_secret) if signing_secret else None

    def _err(msg, typ, status):
        return web.json_response({"error": {"message": msg, "type": typ}}, status=status)

    async def _admit(request: web.Request, who: dict):
        """None when the request may proceed, else the rejection response."""
        api = request.path.startswith("/v1/")
        if api and (keys or jwt_secret):
            auth = request.headers.get("Authorization", "")
            cred = auth[7:] if auth.startswith("Bearer ") else ""
            claims = jwt_decode(cred, jwt_secret) if (jwt_secret and cred not in keys) else None
            if not (cred in keys or claims is not None):
                return _err("unauthorized", "auth", 401)
            who["client"] = cred[:16]
            if roles is not None:
                who["role"] = roles.role_for(cred if cred in keys else None, claims)
        elif roles is not None:
            who["role"] = roles.default_role
        if roles is not None and not roles.allowed(who["role"], request.path):
            return _err(f"role {who['role']!r} may not access {request.path}", "forbidden", 403)
        if signer is not None and api and request.method == "POST":
            body = await request.read()  # cached: handlers read it again
            if not signer.verify(body, request.headers.get("X-Timestamp", ""),
                                 request.headers.get("X-Signature", "")):
                return _err("bad or stale request signature", "auth", 401)
        if bucket is not None and api and not bucket.allow(who["client"]):
            return _err("rate limit exceeded", "rate_limit", 429)
        return None

    @web.middleware
    async def guard(request: web.Request, handler):
        who = {"client": request.remote or "?", "role": None}
        t0 = time.perf_counter()
        resp = await _admit(request, who)
        if resp is None:
            if not limiter.acquire(who["client"]):
                resp = _err("too many requests in flight for this client", "rate_limited", 429)
            else:
                try:
                    resp = await handler(request)
                finally:
                    limiter.release(who["client"])
        client, role = who["client"], who["role"]
        ms = round((time.perf_counter() - t0) * 1e3, 2)
        log_fields(log, "request", path=request.path, status=resp.status, client=client, ms=ms)
        if audit is not None:
            audit.record(client=client, role=role, path=request.path, method=request.method,
                         status=resp.status, ms=ms)
        return resp

    limiter = ConnectionLimiter(max_inflight_per_client)
    clean = sanitize_text if sanitize_input else (lambda t: t)
    app = web.Application(middlewares=[guard])
    loop_holder = {}

    def _params(body) -> SamplingParams:
        stop = tuple(body.get("stop_token_ids") or ()) + tuple(getattr(tok, "stop_ids", ()))
        strs = body.get("stop") or ()
        if isinstance(strs, str):
            strs = (strs,)
        seqs = tuple(tuple(tok.encode(x)) for x in strs if x)
        return SamplingParams(max_tokens=int(body.get("max_tokens", 16)),
                              temperature=float(body.get("temperature", 0.0) or 0.0),
                              top_p=float(body.get("top_p", 1.0) or 1.0), stop_token_ids=tuple(stop),
                              stop_sequences=seqs, seed=body.get("seed"))

    async def _run(prompt, params, stream: bool, request: web.Request, chat: bool, priority: int = 0):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()

        def on_token(r, t):
            loop.call_soon_threadsafe(q.put_nowait, (t, r.finished, r.finish_reason))
        rid = worker.submit(prompt, params, on_token, priority)
        finished = False
        try:
            resp = await _respond(rid, q, prompt, params, stream, request, chat)
            finished = True
            return resp
        finally:
            # a client that disconnected (or a failed write) leaves the request
            # unfinished: stop it so it neither decodes on nor holds KV blocks
            if not finished:
                worker.abort(rid)

    async def _respond(rid, q, prompt, params, stream: bool, request: web.Request, chat: bool):
        cid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:16]}"
        created = int(time.time())
        obj = "chat.completion" if chat else "text_completion"
        if stream:
            resp = web.StreamResponse(headers={"Content-Type": "text/event-stream", "Cache-Control": "no-cache"})
            await resp.prepare(request)
            idx = 0
            toks: List[int] = []
            sent = 0
            trim = StopTrimmer(params.stop_sequences)

            async def send(t, last, reason):
                nonlocal idx, sent
                if masker is None:
                    text = tok.decode([t]) if t is not None else ""
                else:
                    # mask the whole text so far; release all but the last 64
                    # characters (a pattern shorter than that is final once it
                    # is out of the window)
                    if t is not None:
                        toks.append(t)
                    full = masker.mask(tok.decode(toks))
                    upto = len(full) if last else max(sent, len(full) - 64)
                    text, sent = full[sent:upto], upto
                choice = {"index": 0, "finish_reason": reason if last else None}
                if chat:
                    choice["delta"] = {"content": text}
                else:
                    choice["text"] = text
                chunk = {"id": cid, "object": obj + ".chunk" if chat else obj, "created": created,
                         "model": model_name, "choices": [choice], "token": t, "index": idx}
                await resp.write(f"data: {json.dumps(chunk)}\n\n".encode())
                idx += 1

            while True:
                t, done, reason = await q.get()
                ready = trim.push(t, done, reason)
                for k, rt in enumerate(ready):
                    await send(rt, done and k == len(ready) - 1, reason)
                if done:
                    if not ready:  # the stop sequence was all that was left
                        await send(None, True, reason)
                    break
            await resp.write(b"data: [DONE]\n\n")
            await resp.write_eof()
            return resp
        out, kept, reason = [], [], None
        trim = StopTrimmer(params.stop_sequences)
        while True:
            t, done, reason = await q.get()
            out.append(t)
            kept += trim.push(t, done, reason)
            if done:
                break
        text = tok.decode(kept)
        if masker is not None:
            text = masker.mask(text)
        choice = {"index": 0, "finish_reason": reason}
        if chat:
            choice["message"] = {"role": "assistant", "content": text}
        else:
            choice["text"] = text
        return web.json_response({
            "id": cid, "object": obj, "created": created, "model": model_name, "choices": [choice],
            "usage": {"prompt_tokens": len(prompt), "completion_tokens": len(out),
                      "total_tokens": len(prompt) + len(out)},
            "token_ids": kept})

    async def completions(request: web.Request):
        try:
            body = await request.json()
        except Exception:
            return web.json_response({"error": {"message": "invalid JSON", "type": "invalid_request"}}, status=400)
        prompt = body.get("prompt", "")
        ids = prompt if isinstance(prompt, list) else tok.encode(clean(str(prompt)))
        try:
            validator.check(ids, body)
            return await _run(ids, _params(body), bool(body.get("stream")), request, chat=False,
                              priority=int(body.get("priority", 0) or 0))
        except ValueError as e:
            return _err(str(e), "invalid_request", 400)

    async def chat(request: web.Request):
        try:
            body = await request.json()
        except Exception:
            return web.json_response({"error": {"message": "invalid JSON", "type": "invalid_request"}}, status=400)
        msgs = body.get("messages", [])
        if isinstance(msgs, list):
            msgs = [dict(m, content=clean(str(m.get("content", "")))) if isinstance(m, dict) else m for m in msgs]
        ids = tok.apply_chat_template(msgs)
        try:
            validator.check(ids, body)
            return await _run(ids, _params(body), bool(body.get("stream")), request, chat=True,
                              priority=int(body.get("priority", 0) or 0))
        except ValueError as e:
            return _err(str(e), "invalid_request", 400)

    async def models(_):
        return web.json_response({"object": "list", "data": [{"id": model_name, "object": "model",
                                                               "owned_by": "lora_kernel_b200"}]})

    async def health(_):
        return web.json_response({"status": "healthy", "running": worker.running(),
                                  "waiting": worker.waiting()})

    alerts = AlertManager(alert_rules if alert_rules is not None else DEFAULT_ALERTS, log=log)

    async def alerts_view(_):
        for dm in dev_metrics:
            dm.update()
        return web.json_response({"firing": alerts.check()})

    async def metrics(_):
        for dm in dev_metrics:
            dm.update()
        return web.Response(text=REGISTRY.exposition(), content_type="text/plain")

    async def websocket(request: web.Request):
        """Token streaming over one WebSocket: each text message is a request
        ({"prompt": str | [ids], "max_tokens", "temperature", "top_p"}); the
        server answers {"id", "token", "index", "text"} per token, then
        {"id", "done": true, "finish_reason", "usage"}.  Requests on one
        socket run one after another; a reader task keeps reading the socket
        while a request streams, so a client that closes it mid-request stops
        that request."""
        ws = web.WebSocketResponse(heartbeat=30.0)
        await ws.prepare(request)
        loop = asyncio.get_running_loop()
        inbox: asyncio.Queue = asyncio.Queue()
        closed = asyncio.Event()

        async def reader():
            try:
                async for msg in ws:
                    if msg.type == WSMsgType.TEXT:
                        inbox.put_nowait(msg.data)
            finally:
                closed.set()
                inbox.put_nowait(None)

        rtask = asyncio.create_task(reader())
        try:
            while True:
                data = await inbox.get()
                if data is None or closed.is_set():
                    break
                if not await _ws_request(ws, data, loop, closed):
                    break
        finally:
            rtask.cancel()
        return ws

    async def _ws_request(ws, data, loop, closed: asyncio.Event) -> bool:
        """Serve one WebSocket request; False when the socket closed meanwhile."""
        try:
            body = json.loads(data)
            prompt = body.get("prompt", "")
            ids = prompt if isinstance(prompt, list) else tok.encode(clean(str(prompt)))
            validator.check(ids, body)
            params = _params(body)
        except (ValueError, AttributeError) as e:
            await ws.send_json({"error": {"message": str(e), "type": "invalid_request"}})
            return True
        q: asyncio.Queue = asyncio.Queue()
        try:
            rid = worker.submit(ids, params, lambda r, t: loop.call_soon_threadsafe(
                q.put_nowait, (t, r.finished, r.finish_reason)), int(body.get("priority", 0) or 0))
        except ValueError as e:  # e.g. prompt + max_tokens over max_model_len
            await ws.send_json({"error": {"message": str(e), "type": "invalid_request"}})
            return True
        cid = f"ws-{uuid.uuid4().hex[:16]}"
        out: List[int] = []
        kept: List[int] = []
        trim = StopTrimmer(params.stop_sequences)
        done, reason = False, None
        closing = asyncio.ensure_future(closed.wait())
        try:
            while True:
                get = asyncio.ensure_future(q.get())
                await asyncio.wait({get, closing}, return_when=asyncio.FIRST_COMPLETED)
                if not get.done():
                    get.cancel()
                    return False  # the socket went away mid-request
                t, done, reason = get.result()
                out.append(t)
                for rt in trim.push(t, done, reason):
                    kept.append(rt)
                    text = tok.decode([rt]) if masker is None else ""
                    await ws.send_json({"id": cid, "token": rt, "index": len(kept) - 1, "text": text})
                if done:
                    break
        finally:
            closing.cancel()
            if not done:
                worker.abort(rid)
        final = {"id": cid, "done": True, "finish_reason": reason,
                 "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                           "total_tokens": len(ids) + len(out)}}
        if masker is not None:
            final["text"] = masker.mask(tok.decode(kept))
        await ws.send_json(final)
        return True

    app.router.add_post("/v1/completions", completions)
    app.router.add_get("/v1/ws", websocket)
    app.router.add_post("/v1/chat/completions", chat)
    app.router.add_get("/v1/models", models)
    app.router.add_get("/health", health)
    app.router.add_get("/metrics", metrics)
    app.router.add_get("/alerts", alerts_view)

    async def on_shutdown(_):
        worker.shutdown()
    app.on_shutdown.append(on_shutdown)
    app[WORKER_KEY] = worker
    return app


def serve(engine: LLMEngine, host: str = "127.0.0.1", port: int = 8080, **kw) -> None:
    web.run_app(create_app(engine, **kw), host=host, port=port, print=None)
