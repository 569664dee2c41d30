"""swarmllm_b200: a B200-native (sm_100a) LLM inference engine.

Public entry points:
  * ``swarmllm_b200.engine.LLMEngine``        single-process engine (GPU or CPU)
  * ``swarmllm_b200.parallel.pipeline``       multi-GPU pipeline (NCCL p2p)
  * ``swarmllm_b200.serve.api``               OpenAI-compatible HTTP server (:8800)
  * ``swarmllm_b200.models.config.preset``    the benchmark model presets
"""
__version__ = "0.1.0"
