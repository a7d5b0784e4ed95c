"""Offline API: ``LLM(model=...).generate(prompts, SamplingParams(...))`` (vLLM-compatible)."""
from __future__ import annotations

from typing import Optional, Union

from ..config import EngineConfig
from .llm_engine import LLMEngine
from .request import RequestOutput, SamplingParams


class LLM:
    def __init__(self, model: str = "tiny_hybrid", tokenizer: Optional[str] = None, **kwargs):
        self.engine = LLMEngine(EngineConfig(model=model, **kwargs), tokenizer_path=tokenizer)

    def generate(self, prompts: Union[str, list], sampling_params=None) -> list[RequestOutput]:
        if isinstance(prompts, str) or (prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        return self.engine.generate(prompts, sampling_params)

    def chat(self, messages: list[dict], sampling_params=None, **template_kw) -> RequestOutput:
        text = self.engine.tokenizer.apply_chat_template(messages, add_generation_prompt=True,
                                                         **template_kw)
        return self.generate([text], sampling_params)[0]
