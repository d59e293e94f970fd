"""Reference arm of bench.py: the unmodified reference (baseline/_ref) on the same workload.

What runs is the reference's own code path: its recipe engine
``recipes.qwen3.engine.qwen3_engine.Qwen3Engine`` (Engine.__init__ ->
prepare_parallel / ParallelMesh, prepare_model -> LLMModelKit (HF Qwen3 with
flash_attention_2) -> FLOPs patch -> chunked token-loss patch -> fp32 masters
-> HF gradient checkpointing -> parallelize_model (torch FSDP2, or DDP when the
shard dimension is 1), OptimKit AdamW + cosine, and per micro-batch its
train_pre_step (prepare_packed_model_inputs -> FA2 varlen kwargs) and
train_exec_step (forward / token-normalised backward / optimizer step).

Substitutions, forced by the offline environment: the reference's dataset
runtime (``mvp_dataset``) is absent, so batches come from the same synthetic
packs this benchmark feeds its own arm, collated by the reference's
``LLMBatchCollator``; ``omegaconf`` / ``accelerate`` / ``hydra`` are replaced
by the small stand-ins in ``baseline/shims`` (config conversion and seeding
only); the HF config for Qwen3-8B-Base is written locally (no hub access).
None of this engine's models, kernels or runtime are imported.
"""

from __future__ import annotations

import json
import os
import random
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
SHIMS = os.path.join(HERE, "shims")

QWEN3_8B_BASE_CONFIG = {
    "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": 151936, "hidden_size": 4096,
    "intermediate_size": 12288, "num_hidden_layers": 36, "num_attention_heads": 32, "num_key_value_heads": 8,
    "head_dim": 128, "hidden_act": "silu", "max_position_embeddings": 32768, "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0, "rope_scaling": None, "attention_bias": False, "attention_dropout": 0.0,
    "tie_word_embeddings": False, "initializer_range": 0.02, "use_cache": False, "torch_dtype": "bfloat16",
    "bos_token_id": 151643, "eos_token_id": 151643, "sliding_window": None, "use_sliding_window": False,
}


def _unavailable(reason: str) -> None:
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason[:300]}), flush=True)


def _packs(n: int, seq_len: int, vocab: int, seed: int, rank: int):
    """Packed sequences with per-document segment ids / positions, the reference's pack format."""
    import torch

    rng = random.Random(seed * 1000003 + rank)
    out = []
    for _ in range(n):
        ids, seg, pos, doc = [], [], [], 0
        while len(ids) < seq_len:
            L = min(rng.randint(256, 4096), seq_len - len(ids))
            doc += 1
            ids += [rng.randrange(vocab) for _ in range(L)]
            seg += [doc] * L
            pos += list(range(L))
        t = torch.tensor(ids)
        out.append({"input_ids": t, "attention_mask": torch.ones_like(t), "labels": t.clone(),
                    "pack_segment_ids": torch.tensor(seg), "position_ids": torch.tensor(pos),
                    "source_sample_num": doc})
    return out


# Workloads of bench.py the reference cannot run, with the reason (printed as its `unavailable` line).
NOT_IN_REFERENCE = {
    "qwen3-8b-cp-ring": "the reference has no context parallelism (only a 'cp' mesh-role name, "
                        "mvp_engine/distributed/parallel_mesh.py:15-22; no context mesh field in config/schema.py)",
    "qwen3-8b-cp-ulysses": "the reference has no context parallelism (only a 'cp' mesh-role name, "
                           "mvp_engine/distributed/parallel_mesh.py:15-22; no context mesh field in config/schema.py)",
    "qwen3-32b-tp": "the reference ships no TP_MODULE_CONFIG for Qwen3 (recipes/qwen3 binds none), so its "
                    "tensor-parallel path cannot shard this model",
    "qwen3-vl-8b": "the reference's Qwen3-VL recipe loads weights and processor files with from_pretrained "
                   "(recipes/qwen3_vl/engine/qwen3_vl_engine.py:166-170, kit/mllm/data) and reads a Lance dataset; "
                   "none of them exist offline",
}


def run(args) -> None:
    workload = getattr(args, "workload", "qwen3-8b-fsdp")
    if workload in NOT_IN_REFERENCE:
        _unavailable(f"workload {workload}: {NOT_IN_REFERENCE[workload]}")
        return
    if not os.path.isdir(os.path.join(REF, "mvp_engine")):
        _unavailable("reference not installed: run baseline/install_reference.sh (pip --no-deps into baseline/_ref)")
        return
    if not os.path.isdir(os.path.join(REF, "recipes")):
        _unavailable("reference recipes/ missing under baseline/_ref (baseline/install_reference.sh copies them)")
        return
    # transformers probes for `accelerate` when first imported; do that before the
    # stand-ins are importable so the probe sees the real (absent) package.
    import transformers  # noqa: F401
    import transformers.modeling_utils  # noqa: F401

    for k, v in (("MASTER_ADDR", "127.0.0.1"), ("MASTER_PORT", "29531"), ("RANK", "0"), ("WORLD_SIZE", "1"),
                 ("LOCAL_RANK", "0")):
        os.environ.setdefault(k, v)
    # The reference package is also called mvp_engine: put it (and the stand-ins) first.
    root = os.path.dirname(HERE)
    sys.path[:] = [REF, SHIMS] + [p for p in sys.path if os.path.abspath(p or ".") != root]
    for name in list(sys.modules):
        if name == "mvp_engine" or name.startswith("mvp_engine."):
            del sys.modules[name]
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    if not torch.cuda.is_available():
        _unavailable("no CUDA device: the reference trains with flash_attention_2, which runs on CUDA only")
        return
    try:
        import flash_attn  # noqa: F401
    except ImportError:
        _unavailable("flash_attn (the reference's attention backend) is not importable")
        return
    import mvp_engine

    assert os.path.abspath(mvp_engine.__file__).startswith(os.path.abspath(REF)), mvp_engine.__file__
    from mvp_engine.engine import TrainStepContext
    from mvp_engine.kit.llm.data.collator import LLMBatchCollator
    from recipes.qwen3.engine.qwen3_engine import Qwen3Engine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    cfg_dir = tempfile.mkdtemp(prefix="qwen3_8b_cfg_")
    with open(os.path.join(cfg_dir, "config.json"), "w") as f:
        json.dump(QWEN3_8B_BASE_CONFIG, f)
    import yaml

    with open(os.path.join(REF, "mvp_engine", "config", "default.yaml")) as f:
        cfg = yaml.safe_load(f)
    with open(os.path.join(REF, "recipes", "qwen3", "configs", "train.yaml")) as f:
        recipe = yaml.safe_load(f)
    from omegaconf import OmegaConf

    cfg = OmegaConf.merge(cfg, recipe)
    steps_total = args.warmup + 2 * args.steps + 2
    cfg["model"]["pretrained_model_name_or_path"] = cfg_dir
    cfg["data"]["max_seq_len"] = args.seq_len
    cfg["data"]["batch_size"] = 1
    cfg["data"]["num_workers"] = 0
    cfg["data"]["packing_isolate_attention"] = True
    cfg["data"]["packing_isolate_position_ids"] = True
    cfg["optim"]["global_batch_size"] = 8 * world
    cfg["optim"]["gradient_accumulation_steps"] = -1
    cfg["loop"]["total_steps"] = steps_total
    cfg["log"]["backends"] = ["terminal"]
    cfg["log"]["interval"] = 1000000
    cfg["checkpoint"]["interval"] = 1000000
    cfg["checkpoint"]["hf_enable"] = False
    cfg["project"]["dir"] = os.environ.get("MVP_BENCH_OUT", "/tmp/mvp_bench_ref")
    try:
        engine = Qwen3Engine(cfg)
        ga = int(engine.config.optim.gradient_accumulation_steps)
        collate = LLMBatchCollator(pad_token_id=151643)
        engine.prepare_dataloader = lambda workflow="train": None
        engine.before_train()
    except torch.OutOfMemoryError as exc:
        _unavailable(f"reference OOM while building model/optimizer at N={world}: {exc}".replace("\n", " "))
        return
    host = [collate([p]) for p in _packs((args.warmup + 2 * args.steps) * ga, args.seq_len, 151936, 42, rank)]
    for b in host:
        for k, v in list(b.items()):
            if isinstance(v, torch.Tensor):
                b[k] = v.pin_memory()

    def micro(b):
        ctx = TrainStepContext(data=dict(b), step=engine.step, epoch=0, micro_step=engine.ga_state.micro_step)
        prepared = engine.train_pre_step(ctx)
        if prepared is not None and prepared is not ctx:
            ctx.data = prepared
        engine.train_exec_step(ctx)
        return ctx

    def step(i):
        ctx = None
        for b in host[i * ga:(i + 1) * ga]:
            ctx = micro(b)
        engine.step += 1
        return ctx

    try:
        engine.model.train()
        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()

        def timed(first: int) -> tuple[float, float]:
            if dist.is_initialized():
                dist.barrier()
            torch.cuda.synchronize()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            loss = None
            for i in range(args.steps):
                ctx = step(first + i)
                out = ctx.outputs
                loss = float(out["global_loss_sum"]) / max(1, int(out["global_effective_token_count"]))
            e.record()
            torch.cuda.synchronize()
            ms = s.elapsed_time(e) / args.steps
            t = torch.tensor([ms], device=engine.device, dtype=torch.float64)
            if dist.is_initialized():
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item()), loss

        ms, _ = timed(args.warmup)
        e_ms, loss = timed(args.warmup + args.steps)
    except torch.OutOfMemoryError as exc:
        _unavailable(f"reference OOM during training steps at N={world}: {str(exc)[:200]}".replace("\n", " "))
        return
    tokens = args.seq_len * ga * world
    flops = engine.unwrapped_model.calculate_model_flops(
        batch_size=1, seq_len=args.seq_len, attention_mask=host[0]["pack_segment_ids"], is_training=True) * ga * world
    line = {
        "impl": "reference",
        "metric": "tokens/s (Qwen3-8B FSDP pretraining, 8192-token packed sequences; whole job)",
        "value": round(tokens / (ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic packs (uniform ids, docs U[256,4096]) through the reference's LLMBatchCollator",
        "config": {"model": "Qwen3-8B", "global_batch": 8 * world, "seq_len": args.seq_len,
                   "parallelism": f"{'fsdp2' if world > 1 else 'ddp'}{world}", "grad_accum": ga,
                   "attention": "flash_attention_2 (flash_attn library)", "activation_checkpointing": "all layers"},
        "tokens_per_s_per_gpu": round(tokens / (ms / 1e3) / world, 1),
        "mfu": round(flops / (ms / 1e3) / (2250e12 * world), 4),
        "e2e": {"value": round(tokens / (e_ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(e_ms, 3)},
        "loss_last": round(loss, 4) if loss is not None else None,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
