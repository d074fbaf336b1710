"""The decode plan prebuilt while the previous step runs (ModelRunner._speculate)
equals, once its token ids are filled in, the plan built from scratch for the
next step, whenever the batch state key matches; a step that needs a new KV
page is not prebuilt."""
import types

import numpy as np
import pytest

from braidinfer_b200 import LLM, SamplingParams
from braidinfer_b200.engine.batch import build_plan, pack


@pytest.mark.parametrize("max_tokens", [(30, 30, 30), (9, 30, 17)], ids=["same", "batch-shrinks"])
def test_speculated_plan_equals_next_step_plan(tiny_llama_dir, max_tokens):
    llm = LLM(tiny_llama_dir, num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32")
    runner = llm.model_runner
    B = 4
    g = types.SimpleNamespace()
    g.seg_cap, g.page_cap = runner._graph_caps(B)
    g.sizes = None
    state = {"spec": None, "hits": 0, "decode_steps": 0, "refused": 0}
    orig = runner.run

    def run(seqs, is_prefill):
        if not is_prefill:
            state["decode_steps"] += 1
            actual = build_plan(runner._items_for(seqs), runner.page_size, pad_seqs=B - len(seqs),
                                scratch_page=runner.page_manager.scratch_page, seg_cap=g.seg_cap, page_cap=g.page_cap)
            g.sizes = actual.sizes
            spec = state["spec"]
            if spec is not None and spec[1] == runner._decode_key(seqs, 0):
                packed = spec[2].copy()
                packed[:len(seqs)] = [s.token_ids[-1] for s in seqs]
                assert np.array_equal(packed, pack(actual))
                state["hits"] += 1
            state["spec"] = runner._speculate(g, seqs, B)
            state["refused"] += state["spec"] is None
        return orig(seqs, is_prefill)

    runner.run = run
    sps = [SamplingParams(temperature=0, max_tokens=m, ignore_eos=True) for m in max_tokens]
    llm.generate([list(range(3, 3 + n)) for n in (5, 20, 31)], sps)
    assert state["decode_steps"] >= 29
    assert state["refused"] >= 3          # page boundaries (16-token pages) are not prebuilt
    # a step after the batch changed (a sequence finished) is rebuilt, not reused
    shrinks = len(set(max_tokens)) - 1
    assert state["hits"] >= state["decode_steps"] - state["refused"] - 2 - shrinks
