"""Tensor parallelism on CPU ranks (gloo): TP2 must reproduce TP1 exactly
(greedy tokens) and to fp32 tolerance (logits), including cascade chunks and
KV-head replication (tp > num_kv_heads)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, ckpt, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    torch.set_num_threads(1)
    from braidinfer_b200 import ChunkedLLM, ChunkType, SamplingParams
    from braidinfer_b200.parallel.state import get_tp
    try:
        cl = ChunkedLLM(ckpt, num_kvcache_blocks=64, kvcache_block_size=16, device="cpu", dtype="float32",
                        tensor_parallel_size=world)
        llm = cl.llm
        llm.model_runner.capture_logits = []
        out = llm.generate([list(range(5, 60)), list(range(9, 30))],
                           SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
        g = torch.Generator().manual_seed(0)
        toks = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (32, 48, 16)]
        ids = [cl.register_chunk(f"c{i}", t, token_ids=toks[i])
               for i, t in enumerate([ChunkType.SYSTEM_PROMPT, ChunkType.CONTEXT, ChunkType.QUERY])]
        o2 = cl.generate_from_chunks(ids[0], ids[2], [ids[1]], dict(temperature=0, max_tokens=6, ignore_eos=True))
        # sampled (non-greedy) decoding must agree across ranks: same logits, same counter-based RNG
        o3 = llm.generate(list(range(5, 40)), SamplingParams(temperature=0.8, top_p=0.9, max_tokens=8,
                                                             ignore_eos=True, seed=7))
        if get_tp().rank == 0 or world == 1:
            q.put((rank, [o["token_ids"] for o in out], o2["token_ids"], o3[0]["token_ids"],
                   [l.numpy().copy() for l in llm.model_runner.capture_logits[:3]]))
        else:
            q.put((rank, [o["token_ids"] for o in out], o2["token_ids"], o3[0]["token_ids"], None))
    except Exception as e:  # pragma: no cover - surfaced by the parent
        import traceback
        q.put((rank, "error", traceback.format_exc(), None, None))
    finally:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(world, ckpt):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    if world == 1:
        ps = [ctx.Process(target=_worker, args=(0, 1, port, ckpt, q))]
    else:
        ps = [ctx.Process(target=_worker, args=(r, world, port, ckpt, q)) for r in range(world)]
    [p.start() for p in ps]
    res = [q.get(timeout=300) for _ in ps]
    [p.join(timeout=60) for p in ps]
    for r in res:
        assert r[1] != "error", r[2]
    return sorted(res, key=lambda r: r[0])


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    from braidinfer_b200.utils.synthetic import make_checkpoint
    return make_checkpoint(str(tmp_path_factory.mktemp("tp")), "tiny-llama", seed=1, dtype=torch.float32)


@pytest.mark.timeout(600)
@pytest.mark.parametrize("world", [2, 4])
def test_tp_matches_tp1(ckpt, world):
    ref = _run(1, ckpt)[0]
    res = _run(world, ckpt)
    for r in res:
        assert r[1] == ref[1] and r[2] == ref[2] and r[3] == ref[3]
    for a, b in zip(res[0][4], ref[4]):
        torch.testing.assert_close(torch.from_numpy(a), torch.from_numpy(b), atol=2e-4, rtol=1e-4)


def test_layout_kv_replication():
    from braidinfer_b200.parallel.layout import TPLayout
    # TinyLlama at TP8: 4 KV heads -> each on 2 consecutive ranks
    ls = [TPLayout(8, r, 32, 4, 64, 5632, 32000) for r in range(8)]
    assert [l.kv_head_start for l in ls] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert all(l.kv_heads == 1 and l.q_heads == 4 for l in ls)
    # q heads of rank r belong to its kv head
    for l in ls:
        assert l.q_head_start // (32 // 4) == l.kv_head_start
    # Llama-3-70B at TP8: 1 KV head per rank, intermediate 28672 / 8 = 3584 = 56 * 64
    l = TPLayout(8, 3, 64, 8, 128, 28672, 128256)
    assert l.kv_heads == 1 and l.inter == 3584 and l.inter_pad == 3584 and l.vocab_local == 16032
    with pytest.raises(Exception):
        TPLayout(3, 0, 32, 8, 128, 1024, 1000)
