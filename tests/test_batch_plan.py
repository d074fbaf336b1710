"""Per-step plan packing on CPU: the padding used by the short-prefill CUDA
graphs keeps every array size fixed, confines padding tokens to the scratch
page and gives them no logits row."""
import numpy as np

from braidinfer_b200.engine.batch import FwdItem, build_plan, pack, unpack
from braidinfer_b200.engine.sequence import SegmentRef

PS, SCRATCH = 16, 99


def _seq_item(n_priv: int, segs):
    pages = list(range(40, 40 + (n_priv + PS - 1) // PS))
    return FwdItem(tokens=list(range(3, 3 + n_priv)), pos0=sum(s.length for s in segs), priv_index0=0,
                   priv_pages=pages, priv_pos0=sum(s.length for s in segs), segments=segs)


def _segs():
    return [SegmentRef(pages=[1, 2, 3], offset=0, length=40, pos0=0, delta=0, chunk=None),
            SegmentRef(pages=[7, 8], offset=5, length=20, pos0=40, delta=12, chunk=None)]


def test_prefill_graph_padding_keeps_sizes_fixed():
    seg_cap, page_cap, Tb = 17, 49, 64
    dummy = FwdItem(tokens=[0], pos0=0, priv_index0=0, priv_pages=[SCRATCH], priv_pos0=0)
    cap = build_plan([dummy], PS, scratch_page=SCRATCH, seg_cap=seg_cap, page_cap=page_cap, pad_tokens=Tb - 1)
    for n in (1, 5, 33, 64):
        run = build_plan([_seq_item(n, _segs())], PS, scratch_page=SCRATCH, seg_cap=seg_cap, page_cap=page_cap,
                         pad_tokens=Tb - n)
        assert run.sizes == cap.sizes, n
        a = run.arrays
        assert len(a["input_ids"]) == Tb and len(a["qo_indptr"]) == 3
        assert list(a["qo_indptr"]) == [0, n, Tb]
        # padding tokens write only into the scratch page
        assert all(s // PS == SCRATCH for s in a["slots"][n:])
        # one logits row: the real sequence's last token
        assert list(a["logits_idx"]) == [n - 1]
        # the real sequence keeps its cascade segments + its private segment
        assert a["seg_indptr"][1] == 3
        assert list(a["seg_delta"][:2]) == [0, 12]
        # the packed buffer round-trips
        views = unpack(np.asarray(pack(run)), run.sizes)
        assert list(views["positions"][:n]) == list(range(60, 60 + n))


def test_pad_sequences_for_decode_graphs():
    item = _seq_item(1, _segs())
    p = build_plan([item], PS, pad_seqs=3, scratch_page=SCRATCH, seg_cap=64, page_cap=200)
    assert p.num_seqs == 4 and p.decode
    assert list(p.arrays["logits_idx"]) == [0, 1, 2, 3]
    assert all(s // PS == SCRATCH for s in p.arrays["slots"][1:])
