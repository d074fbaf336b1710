"""Host-side plan validation (``validate_plans`` / ``BRAID_VALIDATE_PLAN=1``):
the engine's own plans pass, including chunk compositions; a plan whose
metadata points outside the KV pool, the cache, the RoPE table or its own
index arrays is rejected with the offending field named."""
import copy

import pytest

from braidinfer_b200 import ChunkedLLM, ChunkType, SamplingParams
from braidinfer_b200.engine.batch import FwdItem, build_plan, validate_plan
from braidinfer_b200.errors import PlanValidationError

PS, P, ROPE = 16, 32, 512


def _plan():
    items = [FwdItem(tokens=[5, 6, 7], pos0=40, priv_index0=0, priv_pages=[3, 4], priv_pos0=40, segments=[]),
             FwdItem(tokens=[9], pos0=20, priv_index0=20, priv_pages=[7, 8], priv_pos0=0, segments=[])]
    return build_plan(items, PS, pad_seqs=2, scratch_page=0, seg_cap=8, page_cap=16)


def test_engine_plans_pass_validation(tiny_llama_dir):
    cl = ChunkedLLM(tiny_llama_dir, num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32",
                    validate_plans=True)
    assert cl.llm.model_runner.validate
    s = cl.register_chunk("s", ChunkType.SYSTEM_PROMPT, token_ids=list(range(3, 40)))
    c = cl.register_chunk("c", ChunkType.CONTEXT, token_ids=list(range(50, 90)))
    q = cl.register_chunk("q", ChunkType.QUERY, token_ids=list(range(100, 110)))
    out = cl.generate_from_chunks(s, q, [c], SamplingParams(temperature=0, max_tokens=20, ignore_eos=True))
    assert len(out["token_ids"]) == 20


@pytest.mark.parametrize("field,value,where", [
    ("page_ids", P, (0,)), ("slots", P * PS, (1,)), ("positions", ROPE, (2,)), ("positions", -1, (0,)),
    ("qo_indptr", 99, (1,)), ("seg_len", -3, (0,)), ("logits_idx", 1000, (0,))])
def test_out_of_range_metadata_is_rejected(field, value, where):
    plan = _plan()
    validate_plan(plan, PS, P, ROPE)
    bad = copy.deepcopy(plan)
    bad.arrays[field][where] = value
    with pytest.raises(PlanValidationError, match=field.split("_")[0]):
        validate_plan(bad, PS, P, ROPE)


def test_segment_without_enough_pages_is_rejected():
    plan = _plan()
    bad = copy.deepcopy(plan)
    bad.arrays["seg_len"][0] = 3 * PS  # the first segment now spans three pages but owns one
    with pytest.raises(PlanValidationError, match="fewer pages"):
        validate_plan(bad, PS, P, ROPE)
