"""torchpp.llmops on B200: KV cache, LLM inference driver, decode engine."""
from .kvcache import KVCache  # noqa: F401
from .llm import LLMInference  # noqa: F401
