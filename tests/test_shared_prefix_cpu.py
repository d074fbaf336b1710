"""Shared-prefix decode batching on CPU: sequences composing the same cached
chunk at the same position form a group whose shared segments are listed
once (the GPU attends to them in one pass for the whole group).  The plan
and the fp32 restatement must give the same tokens and logits as the
ungrouped plan."""
import torch

from braidinfer_b200 import ChunkedLLM, ChunkType, SamplingParams
from braidinfer_b200.engine.batch import FwdItem, build_plan, find_shared_group
from braidinfer_b200.engine.sequence import SegmentRef
from braidinfer_b200.utils.synthetic import make_checkpoint

KW = dict(num_kvcache_blocks=96, kvcache_block_size=16, device="cpu", dtype="float32")


def test_find_shared_group_picks_the_widest_shared_segment():
    shared = SegmentRef(pages=[5, 6, 7], offset=0, length=40, pos0=10, delta=0)
    other = SegmentRef(pages=[9], offset=0, length=10, pos0=0, delta=0)
    moved = SegmentRef(pages=[5, 6, 7], offset=0, length=40, pos0=12, delta=2)  # same pages, other position
    items = [FwdItem([1], 60, 5, [20], 50, [other, shared]), FwdItem([2], 61, 6, [21], 50, [shared]),
             FwdItem([3], 62, 3, [22], 52, [moved]), FwdItem([4], 63, 7, [23], 50, [other, shared])]
    members, keys = find_shared_group(items, 16, min_keys=32)
    assert members == [0, 1, 3] and len(keys) == 1
    order = members + [2]
    plan = build_plan([items[i] for i in order], 16, group=(3, keys))
    a = plan.arrays
    assert list(a["seq_nsh"]) == [1, 1, 1, 0]
    g0, g1 = a["grp_seg_indptr"]
    assert g1 - g0 == 1 and a["seg_len"][g0] == 40 and list(a["grp_qo_indptr"]) == [0, 3]
    # members list only their own segments; the moved copy of the pages is not shared
    lens = [list(a["seg_len"][a["seg_indptr"][b]:a["seg_indptr"][b + 1]]) for b in range(4)]
    assert lens == [[10, 6], [7], [10, 8], [40, 4]]


def test_grouped_decode_equals_ungrouped(tmp_path):
    d = make_checkpoint(str(tmp_path / "m"), "tiny-llama", seed=0, dtype=torch.float32)
    g = torch.Generator().manual_seed(7)
    rnd = lambda n: torch.randint(3, 1024, (n,), generator=g).tolist()  # noqa: E731
    sys_t, ctx_t, qs = rnd(16), rnd(300), [rnd(n) for n in (5, 9, 13, 7)]
    outs = []
    for share in (True, False):
        cl = ChunkedLLM(d, shared_prefix_batching=share, **KW)
        s = cl.registry.get(cl.register_chunk("s", ChunkType.SYSTEM_PROMPT, token_ids=sys_t))
        c = cl.registry.get(cl.register_chunk("c", ChunkType.CONTEXT, token_ids=ctx_t))
        llm = cl.llm
        llm.model_runner.capture_logits = []
        sp = SamplingParams(temperature=0, max_tokens=6, ignore_eos=True)
        seqs = []
        for i, qt in enumerate(qs):
            q = cl.registry.get(cl.register_chunk(f"q{i}", ChunkType.QUERY, token_ids=qt))
            cl._ensure_kv(cl._place(s, [c], q))
            seqs.append(llm.add_composition({"system_chunk": s, "context_chunks": [c], "query_chunk": q}, sp))
        while any(not x.is_finished for x in seqs):
            llm.step()
        outs.append(([x.completion_token_ids for x in seqs], llm.model_runner.capture_logits))
    (ta, la), (tb, lb) = outs
    assert ta == tb
    assert len(la) == len(lb)
    assert max((x - y).abs().max().item() for x, y in zip(la, lb)) < 1e-4
