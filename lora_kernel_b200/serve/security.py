"""Request and response policies for the HTTP server.

InputValidator   prompt length, token-id range, max_tokens / temperature /
                 top_p bounds, stop strings, seed; refuses the OpenAI
                 options it does not implement (n > 1, penalties,
                 logprobs) with a message instead of letting a bad request
                 reach the engine or silently ignoring it.
PIIMasker        masks e-mail addresses, phone numbers, US social-security
                 and payment-card numbers (Luhn-checked) in generated text.
RoleAccess       role -> allowed path prefixes; the role comes from the JWT
                 `role` claim (API keys map to a configured role).
RequestSigner    HMAC-SHA256 over "<timestamp>.<body>" in X-Signature with
                 X-Timestamp inside a freshness window (replay guard).
AuditLog         one JSON line per request (time, client, role, path,
                 status, tokens) to a file or the logger.

Reference: InputValidator, OutputFilter/PIIMaskingFilter, AuditLogger, RBAC,
RequestSigner, DDoSProtection (include/monitoring/production_monitoring.hpp:
409-509), TextSanitizer / PII regexes (include/data/text_sanitizer.hpp:10-60),
Authentication (include/api/security.hpp:9-20).
"""
from __future__ import annotations

import hashlib
import hmac
import json
import re
import threading
import time
from typing import Dict, Iterable, List, Optional, Sequence


class ValidationError(ValueError):
    pass


class InputValidator:
    def __init__(self, vocab_size: int, max_prompt_tokens: int = 32768, max_new_tokens: int = 8192):
        self.vocab_size = vocab_size
        self.max_prompt_tokens = max_prompt_tokens
        self.max_new_tokens = max_new_tokens

    def check(self, ids: Sequence[int], body: dict) -> None:
        if not ids:
            raise ValidationError("empty prompt")
        if len(ids) > self.max_prompt_tokens:
            raise ValidationError(f"prompt has {len(ids)} tokens; the limit is {self.max_prompt_tokens}")
        for t in ids:
            if not isinstance(t, int) or isinstance(t, bool) or t < 0 or t >= self.vocab_size:
                raise ValidationError(f"token id {t!r} outside [0, {self.vocab_size})")
        mt = body.get("max_tokens", 16)
        if not isinstance(mt, int) or isinstance(mt, bool) or mt < 1 or mt > self.max_new_tokens:
            raise ValidationError(f"max_tokens must be an integer in [1, {self.max_new_tokens}]")
        temp = body.get("temperature", 0.0) or 0.0
        if not isinstance(temp, (int, float)) or not 0.0 <= float(temp) <= 10.0:
            raise ValidationError("temperature must be in [0, 10]")
        top_p = body.get("top_p", 1.0) or 1.0
        if not isinstance(top_p, (int, float)) or not 0.0 < float(top_p) <= 1.0:
            raise ValidationError("top_p must be in (0, 1]")
        n = body.get("n", 1)
        if n != 1:
            raise ValidationError("n must be 1 (one choice per request)")
        for k in ("presence_penalty", "frequency_penalty"):
            if body.get(k, 0) not in (0, 0.0, None):
                raise ValidationError(f"{k} is not supported (use 0)")
        if body.get("logprobs") not in (None, False, 0):
            raise ValidationError("logprobs are not returned by this server")
        pr = body.get("priority", 0)
        if pr is not None and (not isinstance(pr, int) or isinstance(pr, bool) or not -1000 <= pr <= 1000):
            raise ValidationError("priority must be an integer in [-1000, 1000] (lower runs sooner)")
        seed = body.get("seed")
        if seed is not None and (not isinstance(seed, int) or isinstance(seed, bool) or not 0 <= seed < 2 ** 63):
            raise ValidationError("seed must be an integer in [0, 2^63)")
        sti = body.get("stop_token_ids")
        if sti is not None and (not isinstance(sti, list) or len(sti) > 64 or not all(
                isinstance(t, int) and not isinstance(t, bool) and 0 <= t < self.vocab_size for t in sti)):
            raise ValidationError(f"stop_token_ids must be a list of at most 64 token ids in [0, {self.vocab_size})")
        stop = body.get("stop")
        if stop is not None:
            seqs = [stop] if isinstance(stop, str) else stop
            if not isinstance(seqs, list) or len(seqs) > 4 or \
                    not all(isinstance(x, str) and 0 < len(x) <= 256 for x in seqs):
                raise ValidationError("stop must be a string or a list of at most 4 non-empty strings")


def _luhn_ok(digits: str) -> bool:
    s, alt = 0, False
    for ch in reversed(digits):
        d = ord(ch) - 48
        if alt:
            d *= 2
            if d > 9:
                d -= 9
        s += d
        alt = not alt
    return s % 10 == 0


def sanitize_text(text: str, max_chars: int = 100_000) -> str:
    """Prompt text with C0 control characters other than tab / newline /
    carriage return replaced by spaces, cut to max_chars (reference:
    TextSanitizer::sanitize, include/data/text_sanitizer.hpp:10-24)."""
    out = "".join(c if (c >= " " or c in "\t\n\r") and c != "\x7f" else " " for c in text)
    return out[:max_chars]


class ConnectionLimiter:
    """At most `limit` requests in flight per client (0 = unlimited): a
    client that opens more gets 429 until one finishes (reference:
    DDoSProtection, include/monitoring/production_monitoring.hpp:500-509, which
    counts connections but never releases them)."""

    def __init__(self, limit: int = 0):
        self.limit = int(limit)
        self.inflight: Dict[str, int] = {}
        self._lock = threading.Lock()

    def acquire(self, client: str) -> bool:
        if self.limit <= 0:
            return True
        with self._lock:
            n = self.inflight.get(client, 0)
            if n >= self.limit:
                return False
            self.inflight[client] = n + 1
            return True

    def release(self, client: str) -> None:
        if self.limit <= 0:
            return
        with self._lock:
            n = self.inflight.get(client, 0) - 1
            if n > 0:
                self.inflight[client] = n
            else:
                self.inflight.pop(client, None)


class PIIMasker:
    EMAIL = re.compile(r"[A-Za-z0-9._%+-]+@[A-Za-z0-9.-]+\.[A-Za-z]{2,}")
    SSN = re.compile(r"\b\d{3}-\d{2}-\d{4}\b")
    CARD = re.compile(r"\b(?:\d[ -]?){12,18}\d\b")
    PHONE = re.compile(r"(?:\+?\d{1,2}[ .-]?)?(?:\(\d{3}\)|\b\d{3})[ .-]?\d{3}[ .-]?\d{4}\b")

    def mask(self, text: str) -> str:
        text = self.EMAIL.sub("[EMAIL]", text)
        text = self.SSN.sub("[SSN]", text)

        def card(m):
            digits = re.sub(r"\D", "", m.group(0))
            return "[CARD]" if 13 <= len(digits) <= 19 and _luhn_ok(digits) else m.group(0)
        text = self.CARD.sub(card, text)
        return self.PHONE.sub("[PHONE]", text)


class RoleAccess:
    """roles: {role: [path prefixes]}; "*" allows every path."""

    def __init__(self, roles: Dict[str, Iterable[str]], key_roles: Optional[Dict[str, str]] = None,
                 default_role: str = "user"):
        self.roles = {r: list(p) for r, p in roles.items()}
        self.key_roles = dict(key_roles or {})
        self.default_role = default_role

    def role_for(self, api_key: Optional[str], claims: Optional[dict]) -> str:
        if claims and isinstance(claims.get("role"), str):
            return claims["role"]
        if api_key and api_key in self.key_roles:
            return self.key_roles[api_key]
        return self.default_role

    def allowed(self, role: str, path: str) -> bool:
        prefixes = self.roles.get(role, [])
        return any(p == "*" or path.startswith(p) for p in prefixes)


class RequestSigner:
    def __init__(self, secret: str, window_s: float = 300.0):
        self.key = secret.encode()
        self.window_s = window_s

    def sign(self, body: bytes, ts: Optional[float] = None) -> Dict[str, str]:
        ts = int(time.time() if ts is None else ts)
        mac = hmac.new(self.key, f"{ts}.".encode() + body, hashlib.sha256).hexdigest()
        return {"X-Timestamp": str(ts), "X-Signature": mac}

    def verify(self, body: bytes, ts_header: str, sig_header: str, now: Optional[float] = None) -> bool:
        try:
            ts = int(ts_header)
        except (TypeError, ValueError):
            return False
        now = time.time() if now is None else now
        if abs(now - ts) > self.window_s:
            return False
        mac = hmac.new(self.key, f"{ts}.".encode() + body, hashlib.sha256).hexdigest()
        return hmac.compare_digest(mac, sig_header or "")


class AuditLog:
    def __init__(self, path: Optional[str] = None, logger=None):
        self.path = path
        self.logger = logger
        self._lock = threading.Lock()
        self.records: List[dict] = []  # the last few, for inspection
        self.keep = 1000

    def record(self, **fields) -> None:
        rec = {"ts": round(time.time(), 3), **fields}
        with self._lock:
            self.records.append(rec)
            if len(self.records) > self.keep:
                del self.records[: len(self.records) - self.keep]
            if self.path:
                with open(self.path, "a") as f:
                    f.write(json.dumps(rec) + "\n")
        if self.logger is not None:
            self.logger.info(json.dumps(rec))
