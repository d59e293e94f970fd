#!/usr/bin/env python
"""Headline benchmark: Qwen3-8B dense-decoder pretraining throughput with FSDP on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Workload (weak scaling, fixed per-GPU work): Qwen3-8B architecture (36 layers,
hidden 4096, 32 q / 8 kv heads, head_dim 128, SwiGLU 12288, QK-norm, RoPE 1e6,
vocab 151936, untied), random-init weights, bf16 compute with fp32 master
weights and AdamW; synthetic data: token ids uniform over the vocabulary,
documents with lengths uniform in [256, 4096] packed into 8192-token sequences
with a causal mask per document; 8 sequences per GPU per optimizer step
(micro-batch 1 x 8 accumulation steps), i.e. a global batch of 64 sequences on
8 GPUs.  Every step runs forward, backward, the gradient reduce-scatter,
global-norm clip and the AdamW update.

Timing: W warm-up steps, then K steps bracketed by a barrier and
``torch.cuda.synchronize()`` on both sides and timed with CUDA events on the
compute stream; the reported step time is the max over ranks.  Weights,
optimizer state and activations are far larger than the 126 MB L2, so no
explicit flush is needed between steps.  A second timed pass measures the same
steps end to end through ``Engine.train_step`` (host batches in pinned memory
copied to the device every step, the step's loss read back to the host).
Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEQ_LEN = 8192
PER_GPU_SEQS = 8
MODEL = "Qwen/Qwen3-8B-Base"
METRIC = "tokens/s (Qwen3-8B FSDP pretraining, 8192-token packed sequences; whole job)"

# Named workloads.  The default is the headline benchmark; the others are the long-context
# context-parallel and the tensor-parallel configurations (all ranks form one context / tensor
# group up to its size, data parallelism over the rest).
WORKLOADS = {
    "qwen3-8b-fsdp": dict(model=MODEL, seq=SEQ_LEN, seqs_per_dp=PER_GPU_SEQS, docs=(256, 4096), metric=METRIC,
                          model_name="Qwen3-8B"),
    "qwen3-8b-cp-ring": dict(model=MODEL, seq=131072, seqs_per_dp=1, docs=(4096, 65536), cp="ring", ckpt_all=True,
                             metric="tokens/s (Qwen3-8B, 131072-token packed sequences, ring context parallel; "
                                    "whole job)", model_name="Qwen3-8B"),
    "qwen3-8b-cp-ulysses": dict(model=MODEL, seq=131072, seqs_per_dp=1, docs=(4096, 65536), cp="ulysses",
                                ckpt_all=True,
                                metric="tokens/s (Qwen3-8B, 131072-token packed sequences, Ulysses context "
                                       "parallel; whole job)", model_name="Qwen3-8B"),
    "qwen3-vl-8b": dict(model="Qwen/Qwen3-VL-8B-Instruct", seq=16384, seqs_per_dp=4, docs=(448, 1344),
                        recipe="qwen3_vl", config="recipes/qwen3_vl/configs/train.yaml", reserve_gb=12,
                        metric="tokens/s (Qwen3-VL-8B SFT, 16384-token packs of 1-4 images + text; whole job)",
                        model_name="Qwen3-VL-8B"),
    "qwen3-32b-tp": dict(model="Qwen/Qwen3-32B", seq=4096, global_batch=32, docs=(256, 4096), tp=8, ckpt_all=True,
                         metric="tokens/s (Qwen3-32B, TP + sequence parallel + FSDP, 4096-token packed sequences; "
                                "whole job)", model_name="Qwen3-32B"),
}


def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.gpus = gpu_indices
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self) -> None:
        for line in self.proc.stdout:  # type: ignore[union-attr]
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if self.gpus and idx not in self.gpus:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        loaded = [s for s in sm if s > 500] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def _measured_peak() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def _bytes_of(batch: dict) -> int:
    import torch

    return sum(v.numel() * v.element_size() for v in batch.values() if isinstance(v, torch.Tensor))


def _vocab_of(model: str) -> int:
    from mvp_engine.models.qwen3 import load_qwen3_config

    return load_qwen3_config(model).vocab_size


def run_ours(args) -> None:
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from mvp_engine.config.loader import compose_config
    from mvp_engine.engine import TrainStepContext
    from mvp_engine.launch import import_recipe_modules
    from mvp_engine.ops import _ext

    world = _env_int("WORLD_SIZE", 1)
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    rank = _env_int("RANK", 0)
    wl = WORKLOADS[args.workload]
    recipe = wl.get("recipe", "qwen3")
    import_recipe_modules(__import__("pathlib").Path(ROOT) / "recipes" / recipe)
    if recipe == "qwen3_vl":
        from recipes.qwen3_vl.engine.qwen3_vl_engine import Qwen3VLEngine as EngineClass
    else:
        from recipes.qwen3.engine.qwen3_engine import Qwen3Engine as EngineClass

    steps_total = args.warmup + 2 * args.steps + 2
    if args.model == MODEL:
        args.model = wl["model"]
    if args.seq_len == SEQ_LEN:
        args.seq_len = wl["seq"]
    cp = world if wl.get("cp") else 1
    tp = min(world, wl.get("tp", 1))
    dp = world // (cp * tp)
    global_batch = wl.get("global_batch", wl.get("seqs_per_dp", PER_GPU_SEQS) * dp)
    lo, hi = wl["docs"]
    mesh = []
    if cp > 1:
        mesh = [f"parallel.mesh.context={cp}", "parallel.mesh.shard=1", "parallel.mesh.replicate=1",
                f"parallel.backend_kwargs.context_parallel.impl={wl['cp']}"]
    elif tp > 1:
        mesh = [f"parallel.mesh.tensor={tp}", "parallel.mesh.shard=-1", "parallel.mesh.replicate=1",
                "parallel.backend_kwargs.sequence_parallel=true"]
    if recipe == "qwen3_vl":  # 1-4 images, sides multiples of 32 in [lo, hi] px; text (~1/3 of tokens) supervised
        data = [f"data.train_path=synthetic://mm?min_px={lo}&max_px={hi}&min_images=1&max_images=4"
                f"&min_text=256&max_text=2048&loss_fraction=1.0", "data.dataset_source=synthetic_mm",
                f"model.image_max_pixels={hi * hi}", "parallel.mesh.replicate=1", "parallel.mesh.shard=-1",
                "log.backends=[terminal]"]
    else:
        data = [f"data.train_path=synthetic://text?vocab={_vocab_of(args.model)}&min_len={lo}&max_len={hi}"]
    overrides = mesh + data + [
        f"model.pretrained_model_name_or_path={args.model}",
        f"data.max_seq_len={args.seq_len}",
        f"optim.global_batch_size={global_batch}",
        "data.batch_size=1",
        "optim.gradient_accumulation_steps=-1",
        f"loop.total_steps={steps_total}",
        "log.backends=[terminal]",
        "log.interval=1000000",
        f"project.dir={os.environ.get('MVP_BENCH_OUT', '/tmp/mvp_bench')}",
        "checkpoint.interval=1000000",
        "data.num_workers=0",
        "model.gradient_checkpointing.enabled=false",
    ] + list(args.override or [])
    cfg = compose_config(os.path.join(ROOT, wl.get("config", "recipes/qwen3/configs/synthetic_8b.yaml")), overrides)
    engine = EngineClass(cfg)
    ga = int(engine.config.optim.gradient_accumulation_steps)

    # Decide how many layers recompute activations from the memory left after
    # weights and optimizer state: build, measure, then enable checkpointing.
    engine.train_loader = engine.prepare_dataloader("train")
    engine.model = engine.prepare_model()
    engine.optimizer = engine.prepare_optimizer()
    from mvp_engine.utils.training import GradientAccumulationState, GradientScaler
    from mvp_engine.utils.log.timer import Timer

    engine.ga_state = GradientAccumulationState(ga)
    engine.scheduler = engine.prepare_scheduler()
    engine.scaler = GradientScaler(enabled=True, dtype=engine.dtype, device=engine.device_type)
    engine.timer = Timer(total_progress=engine.total_steps)
    inner = engine.unwrapped_model
    cfgm = getattr(inner.config, "text_config", inner.config)
    torch.cuda.synchronize()
    free, _total = torch.cuda.mem_get_info()
    H, F, L = cfgm.hidden_size, cfgm.intermediate_size, cfgm.num_hidden_layers
    qkv = (cfgm.num_attention_heads + 2 * cfgm.num_key_value_heads) * cfgm.head_dim
    local_tokens = args.seq_len // cp  # context ranks hold 1/cp of the row
    # saved per token and layer (bf16): the two residual sums, qkv, the attention output and the SwiGLU
    # input.  The normalised GEMM inputs, the normalised + rotated q / k and the SwiGLU activation are
    # recomputed in the backward (single-rank, data-parallel and ring layers); the tensor-parallel and
    # Ulysses layers keep the norm outputs and q / k as well.
    plain = tp == 1 and wl.get("cp") != "ulysses"
    kept = 4 * H + qkv + 2 * F
    if not plain:
        kept += 2 * H + (cfgm.num_attention_heads + cfgm.num_key_value_heads) * cfgm.head_dim
    per_layer = local_tokens * 2 * kept * 1.1
    head_ws = 4096 * cfgm.vocab_size * 2 * 2 + args.seq_len * H * 16
    # 7 GiB of slack (the one-GPU headline peaked at 160.7 of 178 GiB with 3 layers recomputed); the
    # multimodal workload also keeps the vision tower's per-block checkpoint inputs,
    # the image embeddings and a block's recomputed activations, which vary with the images of a pack
    budget = free - head_ws - (7 << 30) - int(wl.get("reserve_gb", 0)) * (1 << 30)
    keep = max(0, min(L, int(budget // per_layer)))
    ckpt_layers = L - keep if args.ckpt_layers < 0 else args.ckpt_layers
    if wl.get("ckpt_all") and args.ckpt_layers < 0:  # long sequences / activation checkpointing on by config
        ckpt_layers = L
    if ckpt_layers > 0:
        inner.gradient_checkpointing_enable({"num_layers": ckpt_layers})
    engine.model.train()

    it = iter(engine.train_loader)
    n_host = (args.warmup + 2 * args.steps) * ga  # the end-to-end pass gets fresh batches
    host_batches = [next(it) for _ in range(n_host)]
    h2d_bytes = sum(_bytes_of(b) for b in host_batches[:ga])
    # context / tensor ranks of a group share their samples: count each sample once
    tokens_per_step = sum(int(b["total_tokens"]) for b in host_batches[:ga]) * dp

    def step_host(i: int) -> dict:
        return engine.train_step(host_batches[i * ga:(i + 1) * ga])

    for i in range(args.warmup):
        step_host(i)
    torch.cuda.synchronize()
    if args.profile:
        # One step inside an NVTX range for `ncu --nvtx --nvtx-include profile_step`.
        # start/end (not push/pop) range: it spans threads, so autograd's backward
        # kernels are inside it too
        rid = torch.cuda.nvtx.range_start("profile_step")
        step_host(args.warmup)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_end(rid)
        if rank == 0:
            print(json.dumps({"profile_step": "done", "ga": ga, "ckpt_layers": ckpt_layers}), flush=True)
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()
        return

    # ---- device-timed pass: inputs staged on the device beforehand
    staged = []
    for i in range(args.steps):
        row = []
        for b in host_batches[(args.warmup + i) * ga:(args.warmup + i + 1) * ga]:
            ctx = TrainStepContext(data=b, step=0, epoch=0, micro_step=0)
            engine.train_pre_step(ctx)
            row.append(ctx.data)
        staged.append(row)
    torch.cuda.synchronize()
    sampler = ClockSampler([_env_int("LOCAL_RANK", 0)] if world == 1 else list(range(world)))
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    if rank == 0:
        sampler.start()
        time.sleep(0.5)
    engine.mfu_kit.reset()
    _ext.start_counting()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for row in staged:
        for d in row:
            ctx = TrainStepContext(data=d, step=engine.step, epoch=0, micro_step=engine.ga_state.micro_step)
            engine.train_exec_step(ctx)
        engine.step += 1
    end.record()
    torch.cuda.synchronize()
    launches = _ext.stop_counting()
    if dist.is_initialized():
        dist.barrier()
    clocks = sampler.stop() if rank == 0 else {}
    ms = start.elapsed_time(end) / args.steps
    ms_t = torch.tensor([ms], device=engine.device, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    fl = torch.tensor([engine.mfu_kit.accumulated_model_flops], device=engine.device, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(fl)
    flops_per_step = float(fl.item()) / args.steps  # logical FLOPs summed over ranks (reference formula)
    engine.mfu_kit.reset()

    # ---- end-to-end pass through the public step API (H2D from pinned memory, loss read back)
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    e_start.record()
    losses = []
    for i in range(args.steps):
        out = step_host(args.warmup + args.steps + i)
        losses.append(float(out["global_loss_sum"]) / max(1, int(out["global_effective_token_count"])))
    e_end.record()
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_end) / args.steps
    e_t = torch.tensor([e_ms], device=engine.device, dtype=torch.float64)
    if dist.is_initialized():
        dist.all_reduce(e_t, op=dist.ReduceOp.MAX)
    e_ms = float(e_t.item())

    peaks = _measured_peak()
    value = tokens_per_step / (ms / 1e3)
    line = {
        "metric": wl["metric"],
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": True,
        "scaling": "weak" if cp == 1 and "global_batch" not in wl else "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": (f"synthetic: 1-4 images per sample, sides multiples of 32 in [{lo},{hi}] px, N(0,1) pixels, "
                 f"interleaved with uniform-random text tokens, packed to {args.seq_len} tokens, loss on text "
                 f"positions; random-init {wl['model_name']} weights" if recipe == "qwen3_vl" else
                 f"synthetic: uniform token ids over 151936, document lengths U[{lo},{hi}] packed to "
                 f"{args.seq_len} tokens (causal mask per document); random-init {wl['model_name']} weights"),
        "config": {"model": wl["model_name"], "global_batch": global_batch, "seq_len": args.seq_len,
                   "parallelism": (f"fsdp{world}" if cp == 1 and tp == 1 else
                                   f"cp{cp}-{wl['cp']}" if cp > 1 else f"tp{tp}-sp x fsdp{dp}"),
                   "micro_batch": 1, "grad_accum": ga, "workload": args.workload,
                   "activation_checkpoint_layers": ckpt_layers,
                   "l2": "no flush: weights, optimizer state and activations >> 126 MB L2",
                   "optimizer": "AdamW (fp32 master, fused flat-shard kernel), clip 1.0, cosine"},
        "tokens_per_s_per_gpu": round(value / world, 1),
        "mfu": round(flops_per_step / (ms / 1e3) / (2250e12 * world), 4),
        "mfu_vs_measured_bf16_sustained": (round(flops_per_step / (ms / 1e3) / (peaks["bf16_tflops_sustained"] * 1e12
                                                                                 * world), 4)
                                           if peaks.get("bf16_tflops_sustained") else None),
        "clocks": clocks,
        "e2e": {"value": round(tokens_per_step / (e_ms / 1e3), 1), "unit": "tokens/s", "ms_per_step": round(e_ms, 3),
                "h2d_bytes_per_step": int(h2d_bytes),
                "d2h_bytes_per_step": 8 * 2 + 4 * 1,
                "api": f"recipes.{recipe} {EngineClass.__name__}.train_step(host micro-batches)"},
        "gpu_launches": int(launches),
        "peak_mem_gib": round(torch.cuda.max_memory_allocated(engine.device) / 2**30, 1),
        "loss_last": round(losses[-1], 4) if losses else None,
        "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def run_reference(args) -> None:
    from baseline.reference_arm import run as ref_run

    ref_run(args)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="qwen3-8b-fsdp",
                    help="default: the headline Qwen3-8B FSDP benchmark")
    ap.add_argument("--model", default=MODEL)
    ap.add_argument("--seq-len", type=int, default=SEQ_LEN)
    ap.add_argument("--ckpt-layers", type=int, default=-1, help="-1: choose from free memory")
    ap.add_argument("--override", action="append", help="extra config override k=v (repeatable)")
    ap.add_argument("--profile", action="store_true", help="warm up, then run one step in an NVTX range and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        import torch

        if not torch.cuda.is_available():
            raise SystemExit("bench.py times B200 kernels: no CUDA device is visible")
        run_ours(args)


if __name__ == "__main__":
    main()
