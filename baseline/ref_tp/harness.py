"""Reference arm of ``bench.py``: the UNMODIFIED reference (installed under
``baseline/_ref``) driven through its public ``LLM.generate`` API.

This file imports nothing from ``braidinfer_b200``; it only prepares inputs
the reference needs and, for tensor parallelism, assembles the NCCL
all-reduce build that the reference's own dead code describes.

TP1 (``run_tp1``)
    ``LLM(checkpoint_dir)`` on one GPU.  One process-local shim is applied
    before the reference is imported: transformers 5.5 returns
    ``rope_scaling = {'rope_type': 'default', 'rope_theta': θ}`` for a
    ``config.json`` that has no ``rope_scaling`` at all, and the reference's
    ``lru_cache``'d ``get_rope`` (``braidinfer/layers/rotary_embedding.py:69-78``)
    can neither hash that dict nor accept a non-None value.  The shim turns
    such a dict (type ``default``, no scaling fields) back into ``None`` and
    keeps θ as the ``rope_theta`` attribute — what transformers 4.x returned
    for the same file.  Nothing under ``baseline/_ref`` is edited.

TP>1 (``run_tp``)
    The reference is single-GPU; its only collective is the dead
    ``RowParallelLinear.forward`` (``dist.all_reduce`` after the row-parallel
    GEMM, ``braidinfer/layers/linear_distributed.py:170-174``).  This harness
    builds the tensor-parallel baseline from that code:

    * one process per GPU (torchrun); each process sees only its own GPU
      (``CUDA_VISIBLE_DEVICES``), because the reference hard-wires ``cuda:0``
      (``braidinfer/engine/model_runner.py:30``);
    * the checkpoint is a per-rank SHARD of the architecture: head counts and
      the intermediate size divided by the TP degree, so the reference's own
      model, KV pool, fused Triton RMSNorm+QKV kernel and attention all run
      on the local heads (Megatron layout: QKV and gate/up column-split,
      o_proj and down row-split, embedding and LM head replicated);
    * the reference's single-GPU ``RowParallelLinear`` in the Llama model is
      replaced by its ``linear_distributed.RowParallelLinear`` (F.linear, bias
      on rank 0, ``dist.all_reduce`` over NCCL), sized for the local input
      shard that the checkpoint already holds.

    Weights are random N(0, 0.02) in both arms, so every rank may load the
    same shard file; values do not change the work.

The reference raises ``NotImplementedError`` for batch > 1
(``braidinfer/layers/attention.py:146-147``), so the batch's requests are
decoded one after another; the number is a lower bound and labelled so.
"""
from __future__ import annotations

import contextlib
import datetime
import io
import json
import os
import struct
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "_ref")

ARCH = {
    "llama3-8b": dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, intermediate_size=14336, vocab_size=128256, rms_norm_eps=1e-5,
                      rope_theta=500000.0, max_position_embeddings=8192),
    "llama3-70b": dict(hidden_size=8192, num_hidden_layers=80, num_attention_heads=64, num_key_value_heads=8,
                       head_dim=128, intermediate_size=28672, vocab_size=128256, rms_norm_eps=1e-5,
                       rope_theta=500000.0, max_position_embeddings=16384),
    "tinyllama-1.1b": dict(hidden_size=2048, num_hidden_layers=22, num_attention_heads=32, num_key_value_heads=4,
                           head_dim=64, intermediate_size=5632, vocab_size=32000, rms_norm_eps=1e-5,
                           rope_theta=10000.0, max_position_embeddings=4096),
    # Qwen3: per-head q_norm / k_norm (k_norm weights drawn with |w| up to 100,
    # the benchmark configuration's extreme-weight case)
    "qwen3-0.6b": dict(hidden_size=1024, num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                       head_dim=128, intermediate_size=3072, vocab_size=151936, rms_norm_eps=1e-6,
                       rope_theta=1000000.0, max_position_embeddings=40960, model_type="qwen3",
                       tie_word_embeddings=True, k_norm_range=100.0),
}


# ------------------------------------------------------------ checkpoint
def _write_tokenizer(path: str, vocab: int) -> None:
    """Word-level tokenizer with exactly ``vocab`` entries (token i = word wi)."""
    from tokenizers import AddedToken, Tokenizer, decoders, models, pre_tokenizers

    words = {f"w{i}": i for i in range(3, vocab)}
    words.update({"<unk>": 0, "<s>": 1, "</s>": 2})
    tok = Tokenizer(models.WordLevel(vocab=words, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.decoder = decoders.WordPiece(prefix="##")
    tok.add_special_tokens([AddedToken(s, special=True) for s in ("<unk>", "<s>", "</s>")])
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "unk_token": "<unk>", "bos_token": "<s>",
                   "eos_token": "</s>", "model_max_length": 1 << 20, "add_bos_token": False}, f)


def _stream_safetensors(path: str, tensors) -> None:
    """Write ``[(name, shape, fill)]`` as one safetensors file without holding
    the model in memory; ``fill(n)`` returns ``n`` bf16 values as bytes."""
    header, off = {}, 0
    for name, shape, _ in tensors:
        n = 1
        for s in shape:
            n *= s
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + 2 * n]}
        off += 2 * n
    header["__metadata__"] = {"format": "pt"}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)
    with open(path + ".tmp", "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name, shape, fill in tensors:
            n = 1
            for s in shape:
                n *= s
            done = 0
            while done < n:
                k = min(n - done, 1 << 26)
                f.write(fill(k))
                done += k
    os.replace(path + ".tmp", path)


def write_checkpoint(path: str, model: str, tp: int = 1, seed: int = 0) -> str:
    """HF-layout Llama checkpoint of ``model`` (or of one TP shard of it):
    ``config.json``, tokenizer files and ``model.safetensors`` with N(0, 0.02)
    weights and unit norm weights.  Written once per path."""
    import torch

    if os.path.exists(os.path.join(path, "model.safetensors")):
        return path
    os.makedirs(path, exist_ok=True)
    a = dict(ARCH[model])
    model_type = a.pop("model_type", "llama")
    tie = a.pop("tie_word_embeddings", False)
    k_norm_range = a.pop("k_norm_range", None)
    H, D, L, V = a["hidden_size"], a["head_dim"], a["num_hidden_layers"], a["vocab_size"]
    nh, nkv, inter = a["num_attention_heads"] // tp, a["num_key_value_heads"] // tp, a["intermediate_size"] // tp
    assert nh * tp == a["num_attention_heads"] and nkv * tp == a["num_key_value_heads"], "heads must divide by tp"
    arch = {"llama": "LlamaForCausalLM", "qwen3": "Qwen3ForCausalLM"}[model_type]
    cfg = dict(a, num_attention_heads=nh, num_key_value_heads=nkv, intermediate_size=inter, model_type=model_type,
               architectures=[arch], torch_dtype="bfloat16", bos_token_id=1, eos_token_id=2,
               hidden_act="silu", attention_bias=False, tie_word_embeddings=tie)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    _write_tokenizer(path, V)
    # A pool of N(0, 0.02) bf16 values; each tensor reads it from a random offset.
    g = torch.Generator().manual_seed(seed)
    # host tensors: the reference makes CUDA the default device once its engine exists
    pool = (torch.randn(1 << 27, generator=g, device="cpu") * 0.02).to(torch.bfloat16).view(torch.int16).numpy().tobytes()
    ones = torch.ones(1 << 16, dtype=torch.bfloat16, device="cpu").view(torch.int16).numpy().tobytes()
    state = {"pos": 0}

    def rnd(n):
        p = (state["pos"] * 2654435761) % ((1 << 27) - n) if n < (1 << 27) else 0
        state["pos"] += 1
        return pool[2 * p:2 * (p + n)]

    def one(n):
        return ones[:2 * n]

    def k_norm(n):
        w = (torch.rand(n, generator=g, device="cpu") * 2 - 1) * (k_norm_range or 1.0)
        return w.to(torch.bfloat16).view(torch.int16).numpy().tobytes()

    ts = [("model.embed_tokens.weight", (V, H), rnd)]
    for i in range(L):
        p = f"model.layers.{i}."
        ts += [(p + "input_layernorm.weight", (H,), one), (p + "post_attention_layernorm.weight", (H,), one),
               (p + "self_attn.q_proj.weight", (nh * D, H), rnd), (p + "self_attn.k_proj.weight", (nkv * D, H), rnd),
               (p + "self_attn.v_proj.weight", (nkv * D, H), rnd), (p + "self_attn.o_proj.weight", (H, nh * D), rnd),
               (p + "mlp.gate_proj.weight", (inter, H), rnd), (p + "mlp.up_proj.weight", (inter, H), rnd),
               (p + "mlp.down_proj.weight", (H, inter), rnd)]
        if model_type == "qwen3":
            ts += [(p + "self_attn.q_norm.weight", (D,), one),
                   (p + "self_attn.k_norm.weight", (D,), k_norm if k_norm_range else one)]
    # the reference's Qwen3 has its own lm_head parameter (no tying), so the head is always written
    ts += [("model.norm.weight", (H,), one), ("lm_head.weight", (V, H), rnd)]
    _stream_safetensors(os.path.join(path, "model.safetensors"), ts)
    return path


# ----------------------------------------------------------------- shims
def apply_rope_config_shim() -> None:
    """transformers 5.5 → 4.x view of a config without ``rope_scaling`` (this process only)."""
    from transformers import AutoConfig

    if getattr(AutoConfig.from_pretrained, "_braid_shim", False):
        return
    orig = AutoConfig.from_pretrained

    def from_pretrained(*a, **kw):
        cfg = orig(*a, **kw)
        rs = getattr(cfg, "rope_scaling", None)
        if isinstance(rs, dict) and rs.get("rope_type", rs.get("type")) == "default" and \
                set(rs) <= {"rope_type", "type", "rope_theta"}:
            theta = rs.get("rope_theta", None)
            cfg.rope_scaling = None
            if theta is not None:
                cfg.rope_theta = theta
        return cfg

    from_pretrained._braid_shim = True
    AutoConfig.from_pretrained = from_pretrained


def install_tp_row_parallel() -> None:
    """Swap the Llama model's single-GPU RowParallelLinear for the reference's
    NCCL all-reduce RowParallelLinear (``linear_distributed.py:141-174``)."""
    import torch.distributed as dist
    from braidinfer.layers import linear_distributed as ld
    from braidinfer.models import llama

    class RowParallelLocalShard(ld.RowParallelLinear):
        """The reference's distributed row-parallel linear; the checkpoint
        already holds this rank's input shard, so the loader copies as is."""

        def __init__(self, input_size: int, output_size: int, bias: bool = False):
            super().__init__(input_size * dist.get_world_size(), output_size, bias)
            self.weight.weight_loader = self._copy_loader
            if self.bias is not None:
                self.bias.weight_loader = self._copy_loader

        @staticmethod
        def _copy_loader(param, loaded_weight):
            param.data.copy_(loaded_weight)

    llama.RowParallelLinear = RowParallelLocalShard


# ---------------------------------------------------------------- timing
def _decode_requests(llm, prompts, sp, warmup: int, steps: int):
    """Decode each prompt alone through ``generate(stream=True)``; returns
    (device ms over the timed tokens, wall s, tokens)."""
    import torch

    dev_ms, wall, toks = 0.0, 0.0, 0
    for p in prompts:
        evs, times = [], []
        with contextlib.redirect_stdout(io.StringIO()):
            for rec in llm.generate(p, sp, stream=True):
                # The reference yields one record per engine step from the
                # second step on (the first carries two tokens; the last token
                # arrives only in the final record): consecutive non-final
                # records are exactly one decode step apart.
                if rec.get("finished"):
                    continue
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                evs.append(e)
                times.append(time.perf_counter())
        torch.cuda.synchronize()
        a, b = warmup, warmup + steps  # records 0..warmup-1 untimed, then `steps` one-step intervals
        if len(evs) <= b:
            raise RuntimeError("reference produced fewer tokens than requested")
        dev_ms += evs[a].elapsed_time(evs[b])
        wall += times[b] - times[a]
        toks += steps
    return dev_ms, wall, toks


def _prompts(batch: int, plen: int, vocab: int, seed: int = 3):
    import torch

    g = torch.Generator(device="cpu").manual_seed(seed)
    # the reference sets the default device to CUDA; these ids are built on the host
    return [torch.randint(3, vocab, (plen,), generator=g, device="cpu").tolist() for _ in range(batch)]


def _line(args, n, dev_ms, wall, toks, clocks, published, note):
    value = toks / (dev_ms / 1e3)
    return {
        "metric": f"decode tok/s (bs{args.batch}) {args.model} TP{n}", "value": round(value, 2), "unit": "tokens/s",
        "n_gpus": n, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dev_ms / args.steps, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": round(value / published, 3) if args.batch == 8 else None, "dtype": "bf16",
        "data": "synthetic token ids (seed 3), random-init N(0,0.02) weights",
        "config": {"model": args.model, "global_batch": args.batch, "seq_len": args.prompt_len,
                   "parallelism": f"tp{n}", "note": note},
        "clocks": clocks, "e2e": {"value": round(toks / wall, 2), "unit": "tokens/s", "h2d_bytes_per_step": None,
                                  "d2h_bytes_per_step": None, "api": "braidinfer.LLM.generate(stream=True)"},
        "impl": "reference"}


def _engine_kwargs(args):
    max_len = args.prompt_len + args.warmup + args.steps + 68
    return dict(num_kvcache_blocks=-(-max_len // 256) + 4, max_model_len=max_len, kvcache_block_size=256)


def run_tp1(args, clock_sampler, published: float) -> None:
    import tempfile

    import torch

    sys.path.insert(0, REF)
    apply_rope_config_shim()
    from braidinfer import LLM, SamplingParams  # the unmodified reference

    d = write_checkpoint(os.path.join(tempfile.gettempdir(), f"braid_ref_{args.model}_tp1"), args.model)
    prompts = _prompts(args.batch, args.prompt_len, ARCH[args.model]["vocab_size"])
    llm = LLM(d, **_engine_kwargs(args))
    sp = SamplingParams(temperature=0.0, max_tokens=args.warmup + args.steps + 3, ignore_eos=True)
    with clock_sampler(torch.cuda.current_device()) as clocks:
        e0 = time.time()
        dev_ms, wall, toks = _decode_requests(llm, prompts, sp, args.warmup, args.steps)
        clocks.mark(e0, time.time())
    note = ("reference cannot batch (NotImplementedError for batch > 1): requests decoded one at a time, "
            "a lower bound; transformers-5.5 rope_scaling shim applied to AutoConfig in this process")
    line = _line(args, 1, dev_ms, wall, toks, clocks.summary(), published, note)
    if not (getattr(args, "no_extras", False) or getattr(args, "model_given", False) or
            getattr(args, "batch_given", False)):
        line["other_configs"] = _extras(LLM, SamplingParams)
    print(json.dumps(line), flush=True)


# Secondary points of the baseline configurations that the reference can run
# (same labels as the other arm's ``other_configs``).
REF_EXTRAS = [  # label, model, batch, prompt tokens, warm-up, timed steps
    ("qwen3-0.6b bs1 (k_norm |w|<=100)", "qwen3-0.6b", 1, 512, 8, 64),
    ("tinyllama-1.1b bs8", "tinyllama-1.1b", 8, 2048, 4, 32),
]


def _extras(LLM, SamplingParams) -> dict:
    import tempfile
    import types

    out = {}
    for label, model, batch, plen, warmup, steps in REF_EXTRAS:
        try:
            d = write_checkpoint(os.path.join(tempfile.gettempdir(), f"braid_ref_{model}_tp1"), model)
            a = types.SimpleNamespace(prompt_len=plen, warmup=warmup, steps=steps)
            with contextlib.redirect_stdout(io.StringIO()):
                llm = LLM(d, **_engine_kwargs(a))
            sp = SamplingParams(temperature=0.0, max_tokens=warmup + steps + 3, ignore_eos=True)
            dev_ms, wall, toks = _decode_requests(llm, _prompts(batch, plen, ARCH[model]["vocab_size"]), sp,
                                                  warmup, steps)
            out[label] = {"value": round(toks / (dev_ms / 1e3), 2), "unit": "tokens/s",
                          "ms_per_step": round(dev_ms / toks, 4), "e2e": round(toks / wall, 2), "steps": steps,
                          "warmup": warmup, "prompt_len": plen,
                          "note": "requests decoded one at a time (the reference cannot batch)"}
            del llm
        except Exception as e:  # noqa: BLE001 - a secondary point never breaks the headline line
            out[label] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return out


def run_tp(args, clock_sampler, published: float) -> None:
    n = args.gpus
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    os.environ["CUDA_VISIBLE_DEVICES"] = str(local)  # the reference hard-wires cuda:0
    import tempfile

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(0)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", 0))
    if n != dist.get_world_size():
        raise RuntimeError("--gpus must equal the torchrun world size")
    sys.path.insert(0, REF)
    apply_rope_config_shim()
    from braidinfer import LLM, SamplingParams

    install_tp_row_parallel()
    d = os.path.join(tempfile.gettempdir(), f"braid_ref_{args.model}_tp{n}")
    if rank == 0:
        write_checkpoint(d, args.model, tp=n)
    dist.barrier()
    prompts = _prompts(args.batch, args.prompt_len, ARCH[args.model]["vocab_size"])
    llm = LLM(d, **_engine_kwargs(args))
    sp = SamplingParams(temperature=0.0, max_tokens=args.warmup + args.steps + 3, ignore_eos=True)
    dist.barrier()
    torch.cuda.synchronize()
    with clock_sampler(0) as clocks:
        e0 = time.time()
        dev_ms, wall, toks = _decode_requests(llm, prompts, sp, args.warmup, args.steps)
        clocks.mark(e0, time.time())
    t = torch.tensor([dev_ms, wall], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        note = (f"NCCL all-reduce tensor parallelism built from the reference's linear_distributed.RowParallelLinear "
                f"over its Llama model (per-rank shard checkpoint: {ARCH[args.model]['num_attention_heads'] // n} q "
                f"heads, {ARCH[args.model]['num_key_value_heads'] // n} kv heads); requests decoded one at a time "
                "(the reference cannot batch): a lower bound")
        print(json.dumps(_line(args, n, float(t[0]), float(t[1]), toks, clocks.summary(), published, note)),
              flush=True)
    dist.barrier()
    dist.destroy_process_group()
