"""nanovllm_self_b200: a nano-vLLM-style inference engine written for NVIDIA B200 (sm_100a)."""
from .config import Config, EngineConfig
from .llm import HFLLM, LLM, LLM_self
from .sampling_params import SamplingParams

__all__ = ["LLM", "LLM_self", "HFLLM", "SamplingParams", "EngineConfig", "Config"]
__version__ = "0.1.0"
