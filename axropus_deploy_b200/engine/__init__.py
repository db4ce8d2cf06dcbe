from .block_manager import BlockManager, block_hashes
from .engine import EngineConfig, LLMEngine, Request, SamplingParams

__all__ = ["BlockManager", "block_hashes", "EngineConfig", "LLMEngine", "Request", "SamplingParams"]
