"""Python client of a swarmllm_b200 server: `SwarmLLM` (requests) and
`AsyncSwarmLLM` (aiohttp) over the OpenAI / Anthropic-compatible routes and
the admin routes."""
from .async_client import AsyncSwarmLLM
from .client import AdminClient, SwarmLLM, SwarmLLMError
from .types import (ChatMessage, ChatResponse, CompletionResponse, EmbeddingResponse, Model,
                    Usage)

__all__ = ["SwarmLLM", "AsyncSwarmLLM", "AdminClient", "SwarmLLMError", "ChatMessage",
           "ChatResponse", "CompletionResponse", "EmbeddingResponse", "Model", "Usage"]
