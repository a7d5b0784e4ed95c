"""B200-native serving engine for gated-delta-net hybrid LLMs with MXFP4 W4A8 weights."""
__version__ = "0.1.0"

from .config import EngineConfig, ModelConfig, get_model_config  # noqa: F401
from .engine.request import RequestOutput, SamplingParams  # noqa: F401


def __getattr__(name):
    if name == "LLM":
        from .engine.llm import LLM
        return LLM
    if name == "LLMEngine":
        from .engine.llm_engine import LLMEngine
        return LLMEngine
    raise AttributeError(name)
