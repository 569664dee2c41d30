"""asyncio client (aiohttp) with the same methods as the synchronous one
(reference: python/swarmllm_client/async_client.py:313 `AsyncSwarmLLM`)."""
from __future__ import annotations

from typing import Any, AsyncIterator, Optional, Union

import aiohttp

from .client import (SwarmLLMError, _messages, chat_response, completion_response,
                     error_message)
from .types import ChatResponse, CompletionResponse, EmbeddingResponse, Model, Usage


class AsyncSwarmLLM:
    def __init__(self, base_url: str = "http://127.0.0.1:8800", api_key: Optional[str] = None,
                 timeout: float = 300.0):
        self.base_url = base_url.rstrip("/")
        self._headers = {"Authorization": f"Bearer {api_key}"} if api_key else {}
        self._timeout = aiohttp.ClientTimeout(total=timeout)
        self._session: Optional[aiohttp.ClientSession] = None

    async def _sess(self) -> aiohttp.ClientSession:
        if self._session is None or self._session.closed:
            self._session = aiohttp.ClientSession(headers=self._headers, timeout=self._timeout)
        return self._session

    async def _check(self, resp: aiohttp.ClientResponse) -> Any:
        if resp.status >= 400:
            text = await resp.text()
            try:
                import json
                msg = error_message(json.loads(text), text)
            except ValueError:
                msg = text
            raise SwarmLLMError(resp.status, msg)
        if "json" in resp.headers.get("content-type", ""):
            return await resp.json()
        return await resp.text()

    async def _request(self, method: str, path: str, body: Optional[dict] = None,
                       params: Optional[dict] = None) -> Any:
        s = await self._sess()
        async with s.request(method, self.base_url + path, json=body, params=params) as resp:
            return await self._check(resp)

    async def _stream(self, path: str, body: dict) -> AsyncIterator[dict]:
        import json
        s = await self._sess()
        async with s.post(self.base_url + path, json=body) as resp:
            if resp.status >= 400:
                await self._check(resp)
            async for raw in resp.content:
                line = raw.decode("utf-8", "replace").strip()
                if not line.startswith("data:"):
                    continue
                data = line[5:].strip()
                if data == "[DONE]":
                    return
                try:
                    yield json.loads(data)
                except json.JSONDecodeError:
                    continue

    async def _default_model(self, model: Optional[str]) -> str:
        if model:
            return model
        ms = await self.models()
        if not ms:
            raise SwarmLLMError(404, "no models available on the server")
        return ms[0].id

    async def models(self) -> list[Model]:
        data = await self._request("GET", "/v1/models")
        return [Model(m["id"], m.get("object", "model"), m.get("owned_by", "swarmllm"))
                for m in data.get("data", [])]

    async def chat_completion(self, messages, model: Optional[str] = None, *,
                              max_tokens: Optional[int] = None, temperature: float = 0.7,
                              top_p: float = 0.9, **kwargs) -> ChatResponse:
        model = await self._default_model(model)
        body = {"model": model, "messages": _messages(messages), "temperature": temperature,
                "top_p": top_p, **kwargs}
        if max_tokens is not None:
            body["max_tokens"] = max_tokens
        return chat_response(await self._request("POST", "/v1/chat/completions", body), model)

    async def chat_stream(self, messages, model: Optional[str] = None, **kwargs
                          ) -> AsyncIterator[str]:
        """Content deltas of a streamed chat completion."""
        body = {"model": await self._default_model(model), "messages": _messages(messages),
                "stream": True, **kwargs}
        async for chunk in self._stream("/v1/chat/completions", body):
            delta = ((chunk.get("choices") or [{}])[0].get("delta") or {}).get("content")
            if delta:
                yield delta

    async def chat(self, prompt: str, *, system: Optional[str] = None, **kwargs) -> ChatResponse:
        msgs = ([{"role": "system", "content": system}] if system else []) + \
            [{"role": "user", "content": prompt}]
        return await self.chat_completion(msgs, **kwargs)

    async def completion(self, prompt: Union[str, list], model: Optional[str] = None,
                         **kwargs) -> CompletionResponse:
        model = await self._default_model(model)
        body = {"model": model, "prompt": prompt, **kwargs}
        return completion_response(await self._request("POST", "/v1/completions", body), model)

    async def embeddings(self, inputs, model: Optional[str] = None) -> EmbeddingResponse:
        model = await self._default_model(model)
        data = await self._request("POST", "/v1/embeddings", {"model": model, "input": inputs})
        return EmbeddingResponse([d["embedding"] for d in data.get("data", [])],
                                 data.get("model", model), Usage.of(data.get("usage")))

    async def status(self) -> dict:
        return await self._request("GET", "/api/status")

    async def health(self) -> Any:
        return await self._request("GET", "/health")

    async def close(self):
        if self._session is not None and not self._session.closed:
            await self._session.close()

    async def __aenter__(self) -> "AsyncSwarmLLM":
        return self

    async def __aexit__(self, *exc):
        await self.close()
