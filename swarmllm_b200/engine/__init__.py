from .engine import EngineConfig, LLMEngine, RequestOutput  # noqa: F401
from .sampling import SamplingParams  # noqa: F401
