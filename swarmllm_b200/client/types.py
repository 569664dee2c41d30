"""Plain data types returned by the client (no HTTP library types leak out)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional


@dataclass
class ChatMessage:
    role: str
    content: str
    name: Optional[str] = None

    def to_dict(self) -> dict[str, Any]:
        d: dict[str, Any] = {"role": self.role, "content": self.content}
        if self.name:
            d["name"] = self.name
        return d


@dataclass
class Usage:
    prompt_tokens: int = 0
    completion_tokens: int = 0
    total_tokens: int = 0

    @classmethod
    def of(cls, d: Optional[dict]) -> "Usage":
        d = d or {}
        return cls(int(d.get("prompt_tokens", d.get("input_tokens", 0)) or 0),
                   int(d.get("completion_tokens", d.get("output_tokens", 0)) or 0),
                   int(d.get("total_tokens", 0) or 0))


@dataclass
class ChatResponse:
    id: str
    content: str
    finish_reason: Optional[str]
    model: str
    usage: Usage
    tool_calls: list = field(default_factory=list)
    raw: dict = field(default_factory=dict)


@dataclass
class CompletionResponse:
    id: str
    text: str
    finish_reason: Optional[str]
    model: str
    usage: Usage
    raw: dict = field(default_factory=dict)


@dataclass
class Model:
    id: str
    object: str = "model"
    owned_by: str = "swarmllm"


@dataclass
class EmbeddingResponse:
    embeddings: list
    model: str
    usage: Usage
