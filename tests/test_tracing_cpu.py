"""NVTX ranges around engine steps: off by default, balanced when on, and
named for the step's phase and batch."""
from braidinfer_b200 import LLM, SamplingParams
from braidinfer_b200.utils import tracing


def test_nvtx_ranges_bracket_every_step(tiny_llama_dir):
    events = []
    llm = LLM(tiny_llama_dir, num_kvcache_blocks=32, kvcache_block_size=16, device="cpu", dtype="float32")
    sp = SamplingParams(temperature=0, max_tokens=3, ignore_eos=True)
    assert not tracing.enabled()
    llm.generate([list(range(3, 20))], sp)  # off: nothing is pushed
    tracing.enable(True, push=lambda n: events.append(("push", n)), pop=lambda: events.append(("pop", None)))
    try:
        llm.generate([list(range(3, 20)), list(range(5, 9))], sp)
    finally:
        tracing.enable(False)
    depth = 0
    for kind, _ in events:
        depth += 1 if kind == "push" else -1
        assert depth >= 0
    assert depth == 0
    names = [n for k, n in events if k == "push"]
    assert any(n.startswith("prefill b=") for n in names)
    assert any(n.startswith("decode b=2") for n in names)
    assert "sample" in names and any(n.startswith("forward t=") for n in names)


def test_ranges_label_torch_profiler_events(tiny_llama_dir):
    import torch

    llm = LLM(tiny_llama_dir, num_kvcache_blocks=32, kvcache_block_size=16, device="cpu", dtype="float32")
    sp = SamplingParams(temperature=0, max_tokens=2, ignore_eos=True)
    tracing.enable(True, push=lambda n: None, pop=lambda: None)
    try:
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
            llm.generate([list(range(3, 20))], sp)
    finally:
        tracing.enable(False)
    names = {e.name for e in prof.events()}
    assert any(n.startswith("prefill b=1") for n in names)
    assert any(n.startswith("decode b=1") for n in names) and "sample" in names
