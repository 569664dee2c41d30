"""HTTP request guards, as one ASGI middleware around the app:

  auth           an API key, given as ``Authorization: Bearer <key>`` (scheme
                 case-insensitive) or ``x-api-key: <key>``, compared in
                 constant time; /health and /health/ready never need it and
                 /metrics not from the loopback address.  No key configured:
                 everything is open (a local server).
  CORS           browsers may call from localhost origins on the server's port
                 (and configured extra origins); preflights are answered here.
  rate limits    a token bucket per client address: `rpm` requests a minute on
                 the generation routes (/v1/*, /mcp), refilled continuously;
                 over it -> 429 with Retry-After.  0 = unlimited.
  body limit     requests declaring more than `max_body` bytes -> 413.
  headers        nosniff, frame denial and no-referrer on every response.

Reference behaviour: src/api/middleware.rs (constant_time_eq:17,
cors_layer:32, security_headers:71, RateLimiter:175-300, is_exempt_request:429,
auth_middleware:477).
"""
from __future__ import annotations

import hmac
import json
import os
import threading
import time
from dataclasses import dataclass, field

_EXEMPT = ("/health", "/health/ready")
_LOOPBACK = ("127.0.0.1", "::1", "localhost")


def bearer_or_key(headers: dict) -> str:
    """The credential of a request: the bearer token, else x-api-key."""
    auth = headers.get("authorization", "")
    scheme, sep, tok = auth.partition(" ")
    if sep and scheme.lower() == "bearer" and tok.strip():
        return tok.strip()
    return headers.get("x-api-key", "").strip()


def key_matches(given: str, expected: str) -> bool:
    return hmac.compare_digest(given.encode(), expected.encode())


class RateLimiter:
    """Token buckets keyed by (client, class); `rpm` tokens a minute, at most
    `rpm` banked.  At most `max_clients` buckets (new clients are refused when
    full, so a flood of addresses cannot grow the table without bound)."""

    def __init__(self, rpm: int, max_clients: int = 100_000, clock=time.monotonic):
        self.rpm, self.max_clients, self.clock = rpm, max_clients, clock
        self.buckets: dict = {}
        self.lock = threading.Lock()

    def acquire(self, client: str, cls: str = "api") -> float:
        """0.0 if admitted, else seconds until a token is available."""
        if self.rpm <= 0:
            return 0.0
        now = self.clock()
        with self.lock:
            key = (client, cls)
            b = self.buckets.get(key)
            if b is None:
                if len(self.buckets) >= self.max_clients:
                    self.cleanup(120.0, now)
                    if len(self.buckets) >= self.max_clients:
                        return 60.0
                b = self.buckets[key] = [float(self.rpm), now]
            rate = self.rpm / 60.0
            b[0] = min(float(self.rpm), b[0] + (now - b[1]) * rate)
            b[1] = now
            if b[0] >= 1.0:
                b[0] -= 1.0
                return 0.0
            return (1.0 - b[0]) / rate

    def cleanup(self, max_idle: float, now: float | None = None):
        now = self.clock() if now is None else now
        for k in [k for k, b in self.buckets.items() if now - b[1] > max_idle]:
            del self.buckets[k]


@dataclass
class ServerSettings:
    """Guard settings the admin API may change at run time (read per request)."""
    api_key: str | None = None
    port: int = 8800
    cors_origins: tuple = ()
    rpm: int = 0
    max_body: int = 32 << 20
    key_file: str | None = None          # where a rotated key is written (0600)
    ws_tickets: dict = field(default_factory=dict)   # one-time websocket tickets -> expiry

    TICKET_S = 30.0

    def issue_ticket(self, now: float | None = None) -> str:
        """A one-time ticket for the status websocket (`?t=<ticket>`): a
        browser cannot set an Authorization header on a websocket, and the
        key itself should not sit in a URL."""
        import secrets
        now = time.monotonic() if now is None else now
        for t, exp in list(self.ws_tickets.items()):
            if exp < now:
                del self.ws_tickets[t]
        t = secrets.token_hex(16)
        self.ws_tickets[t] = now + self.TICKET_S
        return t

    def take_ticket(self, t: str, now: float | None = None) -> bool:
        exp = self.ws_tickets.pop(t, None)
        return exp is not None and exp >= (time.monotonic() if now is None else now)

    def rotate_key(self) -> str:
        """A new random key, in force from the next request; the old one stops
        working at once (and is overwritten in `key_file` when one is set)."""
        import secrets
        key = secrets.token_hex(32)
        if self.key_file:
            fd = os.open(self.key_file, os.O_WRONLY | os.O_CREAT | os.O_TRUNC, 0o600)
            with os.fdopen(fd, "w") as f:
                f.write(key + "\n")
        self.api_key = key
        self.ws_tickets.clear()
        return key

    def public(self) -> dict:
        return {"auth_required": bool(self.api_key), "port": self.port,
                "cors_origins": list(self.cors_origins), "rpm": self.rpm, "max_body": self.max_body}


class SecurityMiddleware:
    def __init__(self, app, settings: ServerSettings | None = None, api_key: str | None = None,
                 port: int = 8800, cors_origins=(), rpm: int = 0, max_body: int = 32 << 20):
        self.app = app
        self.settings = settings or ServerSettings(api_key or None, port, tuple(cors_origins), rpm,
                                                   max_body)
        self.limiter = RateLimiter(self.settings.rpm)

    @property
    def api_key(self):
        return self.settings.api_key or None

    @property
    def max_body(self):
        return self.settings.max_body

    @property
    def origins(self):
        p = self.settings.port
        return {f"http://localhost:{p}", f"http://127.0.0.1:{p}", f"http://[::1]:{p}",
                *self.settings.cors_origins}

    async def __call__(self, scope, receive, send):
        if scope["type"] not in ("http", "websocket"):
            return await self.app(scope, receive, send)
        self.limiter.rpm = self.settings.rpm
        path = scope.get("path", "")
        headers = {k.decode("latin-1").lower(): v.decode("latin-1") for k, v in scope.get("headers", [])}
        client = (scope.get("client") or ("?", 0))[0]
        origin = headers.get("origin")
        cors = origin if origin in self.origins else None

        if scope["type"] == "websocket":
            if self.api_key and not self._ok(headers, scope):
                return await send({"type": "websocket.close", "code": 4401})
            return await self.app(scope, receive, send)

        method = scope.get("method", "GET")
        if method == "OPTIONS" and origin is not None:
            if cors is None:
                return await self._reply(send, 403, {"error": {"message": "origin not allowed",
                                                               "type": "cors_error"}})
            return await self._reply(send, 204, None, [
                ("access-control-allow-origin", cors), ("vary", "Origin"),
                ("access-control-allow-methods", "GET, POST, PUT, DELETE, OPTIONS"),
                ("access-control-allow-headers",
                 "content-type, authorization, accept, x-api-key, anthropic-version, anthropic-beta"),
                ("access-control-max-age", "600")])
        # limit before auth, so rejected keys are throttled too
        if path.startswith("/v1/") or path == "/mcp":
            wait = self.limiter.acquire(client)
            if wait > 0:
                return await self._reply(send, 429, {"error": {
                    "message": "rate limit exceeded", "type": "rate_limit_error"}},
                    [("retry-after", str(max(1, int(wait + 0.999))))], cors=cors)
        exempt = path in _EXEMPT or (path == "/metrics" and client in _LOOPBACK)
        if self.api_key and not exempt and not self._ok(headers, scope):
            return await self._reply(send, 401, {"error": {
                "message": "missing or invalid API key", "type": "authentication_error"}}, cors=cors)
        too_big = {"error": {"message": f"request body over {self.max_body} bytes",
                             "type": "invalid_request_error"}}
        cl = headers.get("content-length")
        if cl is not None:
            try:
                if int(cl) > self.max_body:
                    return await self._reply(send, 413, too_big, cors=cors)
            except ValueError:
                return await self._reply(send, 400, {"error": {"message": "bad content-length",
                                                               "type": "invalid_request_error"}})
        elif method in ("POST", "PUT", "PATCH"):
            # no declared length (chunked): read it here, bounded, then replay it to the app
            chunks, n = [], 0
            while True:
                msg = await receive()
                if msg["type"] != "http.request":
                    break
                chunks.append(msg.get("body", b""))
                n += len(chunks[-1])
                if n > self.max_body:
                    return await self._reply(send, 413, too_big, cors=cors)
                if not msg.get("more_body"):
                    break
            pending = [{"type": "http.request", "body": b"".join(chunks), "more_body": False}]

            async def receive_replay():
                return pending.pop() if pending else await receive()
            receive = receive_replay

        async def send_wrapped(msg):
            if msg["type"] == "http.response.start":
                hs = list(msg.get("headers", []))
                hs += _SECURITY
                if cors:
                    hs += [(b"access-control-allow-origin", cors.encode()), (b"vary", b"Origin")]
                msg = dict(msg, headers=hs)
            await send(msg)
        return await self.app(scope, receive, send_wrapped)

    def _ok(self, headers, scope) -> bool:
        tok = bearer_or_key(headers)
        if not tok and scope["type"] == "websocket":   # browsers cannot set headers on a websocket
            from urllib.parse import parse_qs
            q = parse_qs(scope.get("query_string", b"").decode())
            ticket = (q.get("t") or [""])[0]
            if ticket:
                return self.settings.take_ticket(ticket)
            tok = (q.get("token") or [""])[0]
        return bool(tok) and key_matches(tok, self.api_key)

    @staticmethod
    async def _reply(send, status, body, extra=(), cors=None):
        data = b"" if body is None else json.dumps(body).encode()
        hs = [(b"content-type", b"application/json"), (b"content-length", str(len(data)).encode())]
        hs += [(k.encode(), v.encode()) for k, v in extra] + _SECURITY
        if cors:
            hs += [(b"access-control-allow-origin", cors.encode()), (b"vary", b"Origin")]
        await send({"type": "http.response.start", "status": status, "headers": hs})
        await send({"type": "http.response.body", "body": data})


_SECURITY = [(b"x-content-type-options", b"nosniff"), (b"x-frame-options", b"DENY"),
             (b"referrer-policy", b"no-referrer")]
