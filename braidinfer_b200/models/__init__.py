"""Model families, selected by ``config.json``'s ``model_type``
(dispatch as in ``braidinfer/engine/model_loader.py:41-50``)."""
from .decoder import DecoderLM
from .gpt2 import GPT2LM


def build_model(spec, tp, dtype, device, max_pos):
    if spec.family == "gpt2":
        return GPT2LM(spec, tp, dtype, device, max_pos)
    return DecoderLM(spec, tp, dtype, device, max_pos)


# Names kept for parity with the reference's model classes.
LlamaForCausalLM = Qwen3ForCausalLM = ERNIE45ForCausalLM = DecoderLM
GPT2ForCausalLM = GPT2LM

__all__ = ["DecoderLM", "GPT2LM", "build_model", "LlamaForCausalLM", "Qwen3ForCausalLM",
           "ERNIE45ForCausalLM", "GPT2ForCausalLM"]
