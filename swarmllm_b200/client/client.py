"""Synchronous client for a swarmllm_b200 server (OpenAI / Anthropic
compatible routes plus the admin routes).

Covers what the reference's Python client offers over HTTP
(python/swarmllm_client/client.py:48 `SwarmLLM`): models, chat completions
with and without streaming, single-turn chat, embeddings, status / health /
metrics, and an admin sub-client.  Built on `requests`; every error answer is
raised as SwarmLLMError with the message taken from the server's OpenAI-style
error envelope.
"""
from __future__ import annotations

import json
from typing import Any, Iterator, Optional, Union

import requests

from .types import ChatMessage, ChatResponse, CompletionResponse, EmbeddingResponse, Model, Usage


class SwarmLLMError(Exception):
    def __init__(self, status_code: int, message: str):
        self.status_code, self.message = status_code, message
        super().__init__(f"SwarmLLM API error ({status_code}): {message}")


def error_message(body: Any, fallback: str) -> str:
    """The message of an error answer: {"error": {"message": ...}} (OpenAI),
    {"error": "..."} or {"type": "error", "error": {"message": ...}} (Anthropic)."""
    err = body.get("error") if isinstance(body, dict) else None
    if isinstance(err, dict) and isinstance(err.get("message"), str) and err["message"]:
        return err["message"]
    if isinstance(err, str) and err:
        return err
    if isinstance(body, dict) and isinstance(body.get("detail"), str):
        return body["detail"]
    return fallback


def iter_sse(lines) -> Iterator[dict]:
    """JSON payloads of a server-sent-event stream, up to `data: [DONE]`."""
    for line in lines:
        if isinstance(line, bytes):
            line = line.decode("utf-8", "replace")
        if not line or line.startswith(":") or not line.startswith("data:"):
            continue
        data = line[5:].strip()
        if data == "[DONE]":
            return
        try:
            yield json.loads(data)
        except json.JSONDecodeError:
            continue


def _messages(messages) -> list[dict]:
    return [m.to_dict() if isinstance(m, ChatMessage) else dict(m) for m in messages]


def chat_response(data: dict, model: str) -> ChatResponse:
    choice = (data.get("choices") or [{}])[0]
    msg = choice.get("message") or {}
    return ChatResponse(id=data.get("id", ""), content=msg.get("content") or "",
                        finish_reason=choice.get("finish_reason"),
                        model=data.get("model", model), usage=Usage.of(data.get("usage")),
                        tool_calls=list(msg.get("tool_calls") or []), raw=data)


def completion_response(data: dict, model: str) -> CompletionResponse:
    choice = (data.get("choices") or [{}])[0]
    return CompletionResponse(id=data.get("id", ""), text=choice.get("text") or "",
                              finish_reason=choice.get("finish_reason"),
                              model=data.get("model", model), usage=Usage.of(data.get("usage")),
                              raw=data)


class AdminClient:
    """The server's /api/admin routes."""

    def __init__(self, parent: "SwarmLLM"):
        self._p = parent

    def stats(self) -> dict:
        return self._p._get("/api/admin/stats")

    def performance(self) -> dict:
        return self._p._get("/api/admin/performance")

    def config(self) -> dict:
        return self._p._get("/api/admin/config")

    def update_config(self, **kwargs) -> dict:
        return self._p._request("PUT", "/api/admin/config", kwargs)

    def reload_config(self) -> dict:
        return self._p._post("/api/admin/config/reload", {})

    def models(self) -> Any:
        return self._p._get("/api/admin/models")

    def model_status(self, model_id: str) -> dict:
        return self._p._get(f"/api/admin/models/{model_id}/status")

    def adapters(self) -> Any:
        return self._p._get("/api/admin/adapters")

    def add_adapter(self, name: str, path: str, scale: float = 1.0) -> dict:
        return self._p._post("/api/admin/adapters", {"name": name, "path": path, "scale": scale})

    def delete_adapter(self, name: str) -> dict:
        return self._p._request("DELETE", f"/api/admin/adapters/{name}")

    def schedule(self) -> dict:
        return self._p._get("/api/admin/schedule")

    def capacity(self) -> dict:
        return self._p._get("/api/admin/swarm/capacity")

    def storage(self) -> dict:
        return self._p._get("/api/admin/storage/breakdown")

    def diagnostics(self) -> dict:
        return self._p._get("/api/admin/diagnostics")

    def version(self) -> dict:
        return self._p._get("/api/admin/version")

    def shutdown(self) -> dict:
        return self._p._post("/api/admin/shutdown", {})


class SwarmLLM:
    """Client of one server.

    >>> c = SwarmLLM("http://127.0.0.1:8800")
    >>> c.chat("hello", max_tokens=16).content
    """

    def __init__(self, base_url: str = "http://127.0.0.1:8800", api_key: Optional[str] = None,
                 timeout: float = 300.0, session: Optional[requests.Session] = None):
        self.base_url = base_url.rstrip("/")
        self.timeout = timeout
        self._session = session or requests.Session()
        if api_key:
            self._session.headers["Authorization"] = f"Bearer {api_key}"
        self.admin = AdminClient(self)

    # ------------------------------------------------------------------ plumbing
    def _url(self, path: str) -> str:
        return self.base_url + path

    def _check(self, resp) -> Any:
        if resp.status_code >= 400:
            try:
                msg = error_message(resp.json(), resp.text)
            except ValueError:
                msg = resp.text
            raise SwarmLLMError(resp.status_code, msg)
        ctype = resp.headers.get("content-type", "")
        return resp.json() if "json" in ctype else resp.text

    def _request(self, method: str, path: str, body: Optional[dict] = None, **kw) -> Any:
        resp = self._session.request(method, self._url(path), json=body, timeout=self.timeout,
                                     **kw)
        return self._check(resp)

    def _get(self, path: str, params: Optional[dict] = None) -> Any:
        return self._request("GET", path, params=params)

    def _post(self, path: str, body: dict) -> Any:
        return self._request("POST", path, body)

    def _stream(self, path: str, body: dict) -> Iterator[dict]:
        resp = self._session.post(self._url(path), json=body, stream=True, timeout=self.timeout)
        if resp.status_code >= 400:
            self._check(resp)
        try:
            yield from iter_sse(resp.iter_lines())
        finally:
            resp.close()

    def _default_model(self, model: Optional[str]) -> str:
        if model:
            return model
        ms = self.models()
        if not ms:
            raise SwarmLLMError(404, "no models available on the server")
        return ms[0].id

    # ------------------------------------------------------------------ OpenAI routes
    def models(self) -> list[Model]:
        data = self._get("/v1/models")
        return [Model(m["id"], m.get("object", "model"), m.get("owned_by", "swarmllm"))
                for m in data.get("data", [])]

    def chat_completion(self, messages, model: Optional[str] = None, *, stream: bool = False,
                        max_tokens: Optional[int] = None, temperature: float = 0.7,
                        top_p: float = 0.9, stop: Union[str, list, None] = None,
                        tools: Optional[list] = None, seed: Optional[int] = None,
                        **kwargs) -> Union[ChatResponse, Iterator[str]]:
        """POST /v1/chat/completions.  stream=True yields the content deltas."""
        model = self._default_model(model)
        body: dict[str, Any] = {"model": model, "messages": _messages(messages),
                                "temperature": temperature, "top_p": top_p, "stream": stream,
                                **kwargs}
        for k, v in (("max_tokens", max_tokens), ("stop", stop), ("tools", tools),
                     ("seed", seed)):
            if v is not None:
                body[k] = v
        if stream:
            return self._stream_deltas(body)
        return chat_response(self._post("/v1/chat/completions", body), model)

    def _stream_deltas(self, body: dict) -> Iterator[str]:
        for chunk in self._stream("/v1/chat/completions", body):
            delta = ((chunk.get("choices") or [{}])[0].get("delta") or {}).get("content")
            if delta:
                yield delta

    def chat(self, prompt: str, *, model: Optional[str] = None, system: Optional[str] = None,
             stream: bool = False, **kwargs) -> Union[ChatResponse, Iterator[str]]:
        """Single-turn chat."""
        msgs = ([{"role": "system", "content": system}] if system else []) + \
            [{"role": "user", "content": prompt}]
        return self.chat_completion(msgs, model, stream=stream, **kwargs)

    def completion(self, prompt: Union[str, list], model: Optional[str] = None, *,
                   max_tokens: int = 16, temperature: float = 0.0, stream: bool = False,
                   **kwargs) -> Union[CompletionResponse, Iterator[str]]:
        """POST /v1/completions (legacy text completion)."""
        model = self._default_model(model)
        body = {"model": model, "prompt": prompt, "max_tokens": max_tokens,
                "temperature": temperature, "stream": stream, **kwargs}
        if stream:
            return (((c.get("choices") or [{}])[0].get("text") or "")
                    for c in self._stream("/v1/completions", body))
        return completion_response(self._post("/v1/completions", body), model)

    def embeddings(self, inputs: Union[str, list], model: Optional[str] = None
                   ) -> EmbeddingResponse:
        model = self._default_model(model)
        data = self._post("/v1/embeddings", {"model": model, "input": inputs})
        return EmbeddingResponse([d["embedding"] for d in data.get("data", [])],
                                 data.get("model", model), Usage.of(data.get("usage")))

    # ------------------------------------------------------------------ Anthropic / Responses
    def messages(self, messages, model: Optional[str] = None, *, max_tokens: int = 256,
                 system: Optional[str] = None, **kwargs) -> dict:
        """POST /v1/messages (Anthropic Messages); the raw answer."""
        body = {"model": self._default_model(model), "messages": _messages(messages),
                "max_tokens": max_tokens, **kwargs}
        if system:
            body["system"] = system
        return self._post("/v1/messages", body)

    def responses(self, input: Union[str, list], model: Optional[str] = None, **kwargs) -> dict:
        """POST /v1/responses (OpenAI Responses); the raw answer."""
        return self._post("/v1/responses",
                          {"model": self._default_model(model), "input": input, **kwargs})

    # ------------------------------------------------------------------ node
    def status(self) -> dict:
        return self._get("/api/status")

    def health(self) -> Any:
        return self._get("/health")

    def health_ready(self) -> Any:
        return self._get("/health/ready")

    def metrics(self) -> str:
        return self._get("/metrics")

    def close(self):
        self._session.close()

    def __enter__(self) -> "SwarmLLM":
        return self

    def __exit__(self, *exc):
        self.close()
