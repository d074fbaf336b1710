"""``LLM`` is the engine itself (``braidinfer/llm.py:4-5``)."""
from .engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    pass
