"""Kernel microbenchmarks timed with CUDA events (warm-up, L2 flush between runs).

Usage::

    python -m mvp_engine.ops.microbench gemm            # Qwen3-8B layer shapes, ours vs cuBLAS
    python -m mvp_engine.ops.microbench gemm --shape 8192,24576,4096 --iters 20
    python -m mvp_engine.ops.microbench vision          # Qwen3-VL ViT LayerNorm / bias+GELU / RoPE
    torchrun --nproc-per-node 2 -m mvp_engine.ops.microbench cp_attention --tokens 131072

Prints one JSON line per case with the kernel time and achieved TFLOP/s.
cuBLAS (``torch.matmul``) is timed alongside only as the comparison column.
"""

from __future__ import annotations

import argparse
import json

import torch

L2_FLUSH_BYTES = 256 << 20  # twice the B200 L2


def _time(fn, iters: int, warmup: int = 3) -> float:
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        flush.zero_()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


QWEN3_8B_SHAPES = {
    # name: (M, N, K) of Y[M,N] = X[M,K] W[N,K]^T for an 8192-token micro-batch
    "qkv": (8192, 6144, 4096),
    "o_proj": (8192, 4096, 4096),
    "gate_up": (8192, 24576, 4096),
    "down": (8192, 4096, 12288),
    "lm_head_chunk": (4096, 151936, 4096),
}


_WITH_REF = True


def bench_gemm(shapes: dict[str, tuple[int, int, int]], iters: int) -> None:
    from mvp_engine import ops

    for name, (M, N, K) in shapes.items():
        x = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        dy = torch.randn(M, N, device="cuda").bfloat16()
        acc = torch.zeros(N, K, device="cuda")  # fp32 weight-gradient accumulator (training path)
        flops = 2.0 * M * N * K
        cases = {
            "fwd": (lambda: ops.gemm(x, w), lambda: torch.matmul(x, w.t())),
            "dgrad": (lambda: ops.gemm(dy, w, b_mn=True), lambda: torch.matmul(dy, w)),
            "wgrad": (
                lambda: ops.gemm(dy, x, a_mn=True, b_mn=True, out_dtype=torch.float32),
                lambda: torch.matmul(dy.t(), x),
            ),
            "wgrad_acc": (
                lambda: ops.gemm(dy, x, a_mn=True, b_mn=True, out=acc, accumulate=True),
                lambda: torch.matmul(dy.t(), x),
            ),
        }
        for kind, (ours, ref) in cases.items():
            t_ours = _time(ours, iters)
            t_ref = _time(ref, iters) if _WITH_REF else float("nan")
            print(
                json.dumps(
                    {
                        "kernel": "gemm_bf16_sm100",
                        "case": f"{name}.{kind}",
                        "M": M,
                        "N": N,
                        "K": K,
                        "ms": round(t_ours, 4),
                        "tflops": round(flops / t_ours / 1e9, 1),
                        "cublas_ms": round(t_ref, 4),
                        "cublas_tflops": round(flops / t_ref / 1e9, 1),
                    }
                ),
                flush=True,
            )
        del x, w, dy, acc
        torch.cuda.empty_cache()


def _doc_lens(total: int, lo: int, hi: int, seed: int = 0) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    lens, used = [], 0
    while used < total:
        n = int(torch.randint(lo, hi + 1, (1,), generator=g))
        n = min(n, total - used)
        lens.append(n)
        used += n
    return lens


def bench_attention(T: int, Hq: int, Hkv: int, iters: int, lo: int = 256, hi: int = 4096) -> None:
    from mvp_engine.ops import _ext

    lens = _doc_lens(T, lo, hi)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    q = torch.randn(T, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(T, Hkv, 128, device="cuda").bfloat16()
    do = torch.randn(T, Hq, 128, device="cuda").bfloat16()
    pairs = sum(n * (n + 1) // 2 for n in lens)
    fwd_flops = 4.0 * pairs * 128 * Hq
    ext = _ext.ext()
    st = _ext.status_buffer().data_ptr()
    scale = 128**-0.5
    o, lse = ext.flash_attn_fwd(q, k, v, cu, scale, True, st)
    t_f = _time(lambda: ext.flash_attn_fwd(q, k, v, cu, scale, True, st), iters)
    t_b = _time(lambda: ext.flash_attn_bwd(do, q, k, v, o, lse, cu, scale, True, st), iters)
    row = {"kernel": "flash_attn_varlen_sm100", "T": T, "Hq": Hq, "Hkv": Hkv, "docs": len(lens),
           "fwd_ms": round(t_f, 4), "fwd_tflops": round(fwd_flops / t_f / 1e9, 1),
           "bwd_ms": round(t_b, 4), "bwd_tflops": round(2.5 * fwd_flops / t_b / 1e9, 1)}
    try:  # comparison column: the FlashAttention-2 library the reference trains with
        if not _WITH_REF:
            raise RuntimeError("skipped (--no-ref)")
        from flash_attn import flash_attn_varlen_func

        mx = max(lens)
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        t_rf = _time(lambda: flash_attn_varlen_func(q, k, v, cu, cu, mx, mx, causal=True), iters)
        out = flash_attn_varlen_func(qq, kk, vv, cu, cu, mx, mx, causal=True)
        t_rb = _time(lambda: torch.autograd.grad(out, (qq, kk, vv), do, retain_graph=True), iters)
        row.update({"fa2_fwd_ms": round(t_rf, 4), "fa2_fwd_tflops": round(fwd_flops / t_rf / 1e9, 1),
                    "fa2_bwd_ms": round(t_rb, 4), "fa2_bwd_tflops": round(2.5 * fwd_flops / t_rb / 1e9, 1)})
    except Exception as exc:  # pragma: no cover - library availability
        row["fa2"] = f"unavailable: {type(exc).__name__}: {exc}"[:200]
    print(json.dumps(row), flush=True)


def bench_peer_rs(mbytes: int, iters: int) -> None:
    """Pull reduce-scatter of one fp32 gradient unit over NVLink vs NCCL's reduce-scatter (launch with
    torchrun, one rank per GPU).  Device time per call, max over ranks; roofline = bytes this rank pulls
    from its peers ((W-1)/W of the unit) at the measured 770 GB/s per-direction peer copy rate."""
    import os

    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm

    from mvp_engine import ops
    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.ops import _ext

    initialize_process_group()
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    n = (mbytes << 20) // 4 // (64 * world) * (64 * world)
    shard = n // world
    buf = symm.empty(n, dtype=torch.float32, device=dev)
    buf.normal_()
    slots = symm.empty(8, dtype=torch.int64, device=dev)
    slots.zero_()
    torch.cuda.synchronize()
    hb, hs = symm.rendezvous(buf, dist.group.WORLD), symm.rendezvous(slots, dist.group.WORLD)
    hs.barrier()
    peers, pslots = [int(x) for x in hb.buffer_ptrs], [int(x) for x in hs.buffer_ptrs]
    out = torch.empty(shard, device=dev)
    seq = [0]

    def ours():
        seq[0] += 1
        ops.peer_reduce_scatter(peers, pslots, slots.data_ptr(), rank, 0, shard, seq[0], out)

    plain = torch.empty(n, device=dev).normal_()

    def nccl():
        dist.reduce_scatter_tensor(out, plain)

    res = {}
    for name, fn in (("peer_pull", ours), ("nccl", nccl)):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ts = []
        for _ in range(iters):
            dist.barrier()
            torch.cuda.synchronize()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            fn()
            e_.record()
            torch.cuda.synchronize()
            ts.append(s_.elapsed_time(e_))
        t = torch.tensor([sorted(ts)[len(ts) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = float(t)
    _ext.check_status(dev)
    wire = (world - 1) / world * n * 4
    if rank == 0:
        print(json.dumps({"kernel": "rs_pull_kernel", "world": world, "unit_mb": round(n * 4 / 2**20, 1),
                          "peer_pull_ms": round(res["peer_pull"], 4), "nccl_ms": round(res["nccl"], 4),
                          "peer_pull_gbs": round(wire / res["peer_pull"] / 1e6, 1),
                          "nccl_gbs": round(wire / res["nccl"] / 1e6, 1),
                          "roofline_frac_of_770": round(wire / res["peer_pull"] / 1e6 / 770.0, 3)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def bench_fsdp_gather(tokens: int, iters: int, copy_ctas: int, loopback_world: int) -> None:
    """FSDP parameter gather of one Qwen3-8B decoder unit (193 M bf16 parameters), alone and carried by
    copy CTAs of the unit's QKV GEMM ([tokens, 4096] x [6144, 4096]^T).

    With torchrun (one rank per GPU) every shard is read from its owner over NVLink; run as one process,
    the ``loopback_world`` "ranks" are local buffers (the kernel's own cost, for ncu).  Device time per
    call, max over ranks.  Roofline of the fused kernel: the slower of the GEMM at the measured cuBLAS
    burst rate and the remote bytes at the measured 770 GB/s peer copy rate."""
    import os

    import torch.distributed as dist

    from mvp_engine import ops
    from mvp_engine.ops import _ext

    multi = int(os.environ.get("WORLD_SIZE", "1")) > 1
    if multi:
        import torch.distributed._symmetric_memory as symm

        from mvp_engine.distributed.init import initialize_process_group

        initialize_process_group()
        rank, world = dist.get_rank(), dist.get_world_size()
    else:
        rank, world = 0, loopback_world
    dev = torch.device("cuda", torch.cuda.current_device())
    unit = 192_937_984  # Qwen3-8B layer: qkv + o + gate_up + down
    shard = -(-unit // (64 * world)) * 64
    if multi:
        buf = symm.empty(shard, dtype=torch.bfloat16, device=dev)
        flags = symm.empty(8, dtype=torch.int64, device=dev)
        buf.normal_()
        flags.fill_(1)
        torch.cuda.synchronize()
        hb, hf = symm.rendezvous(buf, dist.group.WORLD), symm.rendezvous(flags, dist.group.WORLD)
        hf.barrier()
        bufs, fl = [int(x) for x in hb.buffer_ptrs], [int(x) for x in hf.buffer_ptrs]
    else:
        local = [torch.randn(shard, device=dev).bfloat16() for _ in range(world)]
        flags = torch.ones(world, dtype=torch.int64, device=dev)
        bufs, fl = [t.data_ptr() for t in local], [flags.data_ptr() + 8 * r for r in range(world)]
    slot = torch.empty(world * shard, dtype=torch.bfloat16, device=dev)
    x = torch.randn(tokens, 4096, device=dev).bfloat16()
    w = torch.randn(6144, 4096, device=dev).bfloat16()
    y = torch.empty(tokens, 6144, device=dev, dtype=torch.bfloat16)
    st = _ext.status_buffer(dev).data_ptr()
    ext = _ext.ext()

    cases = {
        "qkv_gemm": lambda: ext.gemm(x, False, w, False, y, False, st),
        "gather_kernel": lambda: ext.peer_gather_shards(bufs, fl, 0, shard, 1, slot, st, 10**10),
        "gemm_carrying_gather": lambda: ext.gemm_pair_gather(x, False, w, False, y, False, st, bufs, fl, 0, shard, 1,
                                                             slot, copy_ctas, 10**10),
    }
    if multi:
        plain = torch.empty(shard, dtype=torch.bfloat16, device=dev)
        cases["nccl_all_gather"] = lambda: dist.all_gather_into_tensor(slot, plain)
    res = {}
    for name, fn in cases.items():
        if multi:
            dist.barrier()
        t = _time(fn, iters)
        if multi:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt)
        res[name] = t
    _ext.check_status(dev)
    # sanity: the carried gather produced every rank's shard
    ok = True if multi else bool(torch.equal(slot, torch.cat(local)))
    remote = (world - 1) * shard * 2 if multi else 0
    flops = 2.0 * tokens * 6144 * 4096
    gemm_peak = 1666.3e12
    roof_ms = max(flops / gemm_peak, remote / 770e9) * 1e3
    if rank == 0:
        print(json.dumps({
            "kernel": "gemm2sm_kernel + shard_gather_cta_bulk", "ranks": world, "mode": "peers" if multi else "loopback",
            "unit_mb": round(unit * 2 / 2**20, 1), "copy_ctas": copy_ctas, "tokens": tokens,
            **{f"{k}_ms": round(v, 4) for k, v in res.items()},
            "gather_gbs_remote": round(remote / res["gather_kernel"] / 1e6, 1) if multi else None,
            "gather_gbs_written": round(world * shard * 2 / res["gather_kernel"] / 1e6, 1),
            "fused_roofline_ms": round(roof_ms, 4),
            "fused_frac_of_roofline": round(roof_ms / res["gemm_carrying_gather"], 3),
            "fused_vs_serial": round((res["qkv_gemm"] + res["gather_kernel"]) / res["gemm_carrying_gather"], 3),
            "gather_correct": ok}), flush=True)
    if multi:
        dist.barrier()
        dist.destroy_process_group()


def bench_comm_loopback(tokens: int, hidden: int, mbytes: int, iters: int) -> None:
    """The fused-collective kernels in one process, every "peer" a local buffer and every ready flag
    published before launch (no wait can depend on another process): the kernels' own cost, for ncu.

    * ``rs_pull_kernel``: pull reduce-scatter of an fp32 gradient unit of ``mbytes`` over two local "ranks";
    * ``gemm_pair_tp`` column: [tokens, hidden] x [hidden, hidden]^T with per-256-row-slice readiness waits
      (two slices, already published);
    * ``gemm_pair_tp`` row: the same GEMM with its output rows routed to two destination buffers."""
    from mvp_engine.ops import _ext

    dev = torch.device("cuda", torch.cuda.current_device())
    ext = _ext.ext()
    st = _ext.status_buffer(dev).data_ptr()
    world = 2
    n = (mbytes << 20) // 4 // (64 * world) * (64 * world)
    shard = n // world
    bufs = [torch.randn(n, device=dev) for _ in range(world)]
    slots = [torch.zeros(8, dtype=torch.int64, device=dev) for _ in range(world)]
    slots[0][1] = 1 << 60  # the other "rank" has published every sequence number already
    out = torch.empty(shard, device=dev)
    seq = [0]

    def rs():
        seq[0] += 1
        ext.peer_reduce_scatter([b.data_ptr() for b in bufs], [sl.data_ptr() for sl in slots], slots[0].data_ptr(),
                                0, 0, shard, seq[0], 1.0, out, None, st, 10**10)

    x = torch.randn(tokens, hidden, device=dev).bfloat16()
    w = torch.randn(hidden, hidden, device=dev).bfloat16()
    y = torch.empty(tokens, hidden, device=dev, dtype=torch.bfloat16)
    ready = torch.full((8,), 1 << 60, dtype=torch.int64, device=dev)
    half = tokens // world
    routed = [torch.empty(half, hidden, device=dev, dtype=torch.bfloat16) for _ in range(world)]

    def col():
        ext.gemm_pair_tp(x, w, False, y, hidden, ready.data_ptr(), 1, half, 0, [], 0, 0, st, 10**10)

    def row():
        ext.gemm_pair_tp(x, w, False, None, hidden, 0, 0, 0, 0, [t.data_ptr() for t in routed], half, 0, st, 10**10)

    res = {name: _time(fn, iters) for name, fn in (("rs_pull", rs), ("tp_column", col), ("tp_row_routed", row))}
    _ext.check_status(dev)
    ok = bool(torch.allclose(out, bufs[0][:shard] + bufs[1][:shard], atol=1e-5))
    print(json.dumps({"mode": "loopback", "unit_mb": round(n * 4 / 2**20, 1), "tokens": tokens, "hidden": hidden,
                      **{k + "_ms": round(v, 4) for k, v in res.items()},
                      "rs_pull_gbs_read": round(n * 4 / res["rs_pull"] / 1e6, 1),
                      "tp_tflops": round(2.0 * tokens * hidden * hidden / res["tp_column"] / 1e9, 1),
                      "rs_correct": ok}), flush=True)


def bench_tp_gemm(tokens: int, hidden: int, iters: int) -> None:
    """Tensor-parallel GEMMs with the collective fused over NVLink vs NCCL + GEMM (launch with torchrun).

    column: y[T, H] = all_gather_seq(x[T/W, H]) @ Wc^T;  row: y[T/W, H] = reduce_scatter_seq(x[T, H] @ Wr^T).
    Device time per call, median of `iters`, max over ranks; roofline = max(FLOPs at the measured bf16
    burst peak, this rank's NVLink bytes at 770 GB/s)."""
    import torch.distributed as dist

    from mvp_engine import ops
    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.tensor_parallel import TensorParallel, _AGLinear, _RSLinear

    initialize_process_group()
    W, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    tp = TensorParallel(dist.group.WORLD, sequence_parallel=True, fused=True)
    rows = tokens // W
    x_sp = torch.randn(rows, hidden, device=dev).bfloat16()
    x_full = torch.randn(tokens, hidden, device=dev).bfloat16()
    wc = torch.randn(hidden, hidden, device=dev).bfloat16()
    wr = torch.randn(hidden, hidden, device=dev).bfloat16()
    gathered = torch.empty(tokens, hidden, device=dev, dtype=torch.bfloat16)
    out_sp = torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16)

    def nccl_col():
        dist.all_gather_into_tensor(gathered, x_sp)
        return ops.gemm(gathered, wc)

    def nccl_row():
        dist.reduce_scatter_tensor(out_sp, ops.gemm(x_full, wr))

    cases = {"column_fused": lambda: _AGLinear.apply(x_sp, wc, tp), "column_nccl": nccl_col,
             "row_fused": lambda: _RSLinear.apply(x_full, wr, tp), "row_nccl": nccl_row}
    res = {}
    for name, fn in cases.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            dist.barrier()
            torch.cuda.synchronize()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            fn()
            e_.record()
            torch.cuda.synchronize()
            ts.append(s_.elapsed_time(e_))
        t = torch.tensor([sorted(ts)[len(ts) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = float(t)
    _ext.check_status(dev)
    flops = 2.0 * tokens * hidden * hidden
    wire = (W - 1) / W * tokens * hidden * 2
    peak = 1675e12
    roof_ms = max(flops / peak, wire / 770e9) * 1e3
    if r == 0:
        print(json.dumps({"kernel": "gemm_pair_tp", "world": W, "tokens": tokens, "hidden": hidden,
                          **{k + "_ms": round(v, 4) for k, v in res.items()},
                          "roofline_ms": round(roof_ms, 4),
                          "column_fused_frac_of_roofline": round(roof_ms / res["column_fused"], 3),
                          "row_fused_frac_of_roofline": round(roof_ms / res["row_fused"], 3)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def bench_cp_attention(tokens: int, hq: int, hkv: int, iters: int, impls: list[str]) -> None:
    """One attention layer (forward + backward) under context parallelism (launch with torchrun).

    Workload: one packed row of ``tokens`` tokens, documents U[4096, 65536] (causal per document),
    zig-zag sharded over the W ranks; cases ``ring`` / ``ulysses`` (NCCL collectives) and
    ``ring_fused`` (K/V pulled over NVLink by copy CTAs of the attention kernel, dK/dV written into
    the owners' slots).  Device time per call (CUDA events, median of ``iters``, max over ranks).
    Roofline of the fused ring: max(attention FLOPs of this rank at the measured bf16 burst peak,
    NVLink bytes into this rank at 770 GB/s) where the bytes are the other ranks' K/V (twice: forward
    and backward) and the fp32 dK/dV partials of this rank's keys."""
    import torch.distributed as dist

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import PackedContext
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.context import ContextParallel

    initialize_process_group()
    W, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    lens = _doc_lens(tokens, 4096, 65536)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(7 + r)
    L = tokens // W
    q = torch.randn(L, hq, 128, device=dev, generator=g).bfloat16().requires_grad_()
    k = torch.randn(L, hkv, 128, device=dev, generator=g).bfloat16().requires_grad_()
    v = torch.randn(L, hkv, 128, device=dev, generator=g).bfloat16().requires_grad_()
    do = torch.randn(L, hq, 128, device=dev, generator=g).bfloat16()
    res = {}
    for name in impls:
        impl, fused = name.split("_")[0], name.endswith("_fused")
        cp = ContextParallel(dist.group.WORLD, impl=impl, fused=fused)
        ctx = PackedContext(torch.zeros(1, L, dtype=torch.long, device=dev), cu, max(lens), None, cp=cp)

        def step():
            o = cp.attention(q, k, v, ctx, 128**-0.5)
            o.backward(do)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            dist.barrier()
            torch.cuda.synchronize()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            step()
            e_.record()
            torch.cuda.synchronize()
            ts.append(s_.elapsed_time(e_))
        t = torch.tensor([sorted(ts)[len(ts) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = float(t)
    _ext.check_status(dev)
    causal_pairs = sum(n * (n + 1) / 2 for n in lens)
    flops = 4.0 * causal_pairs * 128 * hq * 3.5 / W  # fwd (2 GEMMs) + bwd (5 GEMMs), per rank
    wire = (W - 1) / W * (2 * 2 * tokens * hkv * 128 * 2 + 2 * tokens * hkv * 128 * 4)
    roof_ms = max(flops / 1675e12, wire / 770e9) * 1e3
    if r == 0:
        line = {"kernel": "cp_attention_fwd_bwd", "world": W, "tokens": tokens, "heads": [hq, hkv],
                "docs": len(lens), **{k_ + "_ms": round(v_, 3) for k_, v_ in res.items()},
                "roofline_ms": round(roof_ms, 3), "link_ms": round(wire / 770e9 * 1e3, 3)}
        for k_, v_ in res.items():
            line[k_ + "_frac_of_roofline"] = round(roof_ms / v_, 3)
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def bench_cp_layer(tokens: int, iters: int, impls: list[str]) -> None:
    """One Qwen3-8B decoder layer (forward + backward) under context parallelism (launch with torchrun).

    The layer sees this rank's zig-zag share of one ``tokens``-token packed row (documents U[4096, 65536]);
    cases ``ulysses`` (NCCL all-to-alls around the attention), ``ulysses_fused`` (the all-to-alls folded
    into the QKV GEMM, attention and QK-norm/RoPE kernels), ``ring`` and ``ring_fused``.  Device time per
    call (median of ``iters``, max over ranks)."""
    import torch.distributed as dist

    from mvp_engine import ops
    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.models.qwen3 import PackedContext, Qwen3DecoderLayer, load_qwen3_config, positions_from_cu_seqlens
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.context import ContextParallel

    initialize_process_group()
    W, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = load_qwen3_config("Qwen/Qwen3-8B-Base")
    layer = Qwen3DecoderLayer(cfg, 0).to(dev).to(torch.bfloat16)
    with torch.no_grad():
        for name, p_ in layer.named_parameters():
            p_.copy_(torch.randn_like(p_) * 0.02 + (1.0 if "norm" in name else 0.0))
    lens = _doc_lens(tokens, 4096, 65536)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
    L = tokens // W
    x = (torch.randn(L, cfg.hidden_size, device=dev) * 0.5).bfloat16().requires_grad_()
    dy1 = torch.randn(L, cfg.hidden_size, device=dev).bfloat16()
    rope = ops.RopeCache(cfg.head_dim, cfg.rope_theta, max_positions=max(lens))
    res = {}
    for name in impls:
        impl, fused = name.split("_")[0], name.endswith("_fused")
        cp = ContextParallel(dist.group.WORLD, impl=impl, fused=fused)
        idx = cp.local_indices(tokens).to(dev)
        pos = positions_from_cu_seqlens(cu, tokens)[idx].view(1, -1).to(torch.int32)
        ctx = PackedContext(pos, cu, max(lens), rope, cp=cp)

        def step():
            out, _ = layer(x, None, ctx)
            out.backward(dy1)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            dist.barrier()
            torch.cuda.synchronize()
            s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s_.record()
            step()
            e_.record()
            torch.cuda.synchronize()
            ts.append(s_.elapsed_time(e_))
        t = torch.tensor([sorted(ts)[len(ts) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = float(t)
    _ext.check_status(dev)
    if r == 0:
        print(json.dumps({"kernel": "cp_decoder_layer_fwd_bwd", "model": "Qwen3-8B", "world": W, "tokens": tokens,
                          "docs": len(lens), **{k_ + "_ms": round(v_, 3) for k_, v_ in res.items()}}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def bench_vision(tokens: int, iters: int) -> None:
    """Vision-tower kernels on Qwen3-VL ViT shapes (hidden 1152, MLP 4304, 16 heads of 72), ours vs eager.

    ``tokens`` patches (28224 = four 1344x1344 images).  Bytes are the algorithmic HBM traffic of each op.
    """
    from mvp_engine import ops

    H, Fd, nh, D = 1152, 4304, 16, 72
    N = tokens
    x = torch.randn(N, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    b = (0.1 * torch.randn(H, device="cuda")).bfloat16()
    h = torch.randn(N, Fd, device="cuda").bfloat16()
    bf = (0.1 * torch.randn(Fd, device="cuda")).bfloat16()
    qkv = torch.randn(N, 3 * H, device="cuda").bfloat16()
    ang = torch.rand(N, D // 2, device="cuda") * 30
    cos, sin = ang.cos(), ang.sin()
    e = _ext_mod()
    y, mean, rstd = e.layernorm_fwd(x, w, b, 1e-6)
    # distinct gradient tensors: aliased inputs would be served from L2 and overstate the bandwidth
    dy = torch.randn(N, H, device="cuda").bfloat16()
    dh = torch.randn(N, Fd, device="cuda").bfloat16()
    dq, dk, dv = (torch.randn(N, nh, 128, device="cuda").bfloat16() for _ in range(3))

    def eager_rope():
        t = qkv.view(N, 3, nh, D)
        c = torch.cat([cos, cos], -1).unsqueeze(1)
        sn = torch.cat([sin, sin], -1).unsqueeze(1)
        out = []
        for i in range(2):
            xf = t[:, i].float()
            a, bb = xf.chunk(2, dim=-1)
            out.append((xf * c + torch.cat((-bb, a), -1) * sn).to(qkv.dtype))
        out.append(t[:, 2])
        return [torch.nn.functional.pad(o, (0, 128 - D)) for o in out]

    cases = {
        # name: (ours, eager, algorithmic bytes)
        "layernorm_fwd": (lambda: e.layernorm_fwd(x, w, b, 1e-6),
                          lambda: torch.nn.functional.layer_norm(x, (H,), w, b, 1e-6), 2 * N * H * 2 + N * 8),
        "layernorm_bwd": (lambda: e.layernorm_bwd(dy, x, mean, rstd, w),
                          None, 3 * N * H * 2 + N * 8),
        "bias_gelu_fwd_tanh": (lambda: e.bias_gelu_fwd(h, bf, True),
                               lambda: torch.nn.functional.gelu(h + bf, approximate="tanh"), 2 * N * Fd * 2),
        "bias_gelu_bwd_tanh": (lambda: e.bias_gelu_bwd(dh, h, bf, True), None, 3 * N * Fd * 2),
        "bias_residual_fwd": (lambda: e.bias_residual_fwd(x, b, dy), lambda: dy + (x + b), 3 * N * H * 2),
        "bias_grad": (lambda: e.bias_grad(dy), lambda: dy.float().sum(0), N * H * 2),
        "vision_rope_fwd": (lambda: e.vision_rope_fwd(qkv, nh, cos, sin, 128), eager_rope,
                            N * 3 * H * 2 + 3 * N * nh * 128 * 2 + 2 * N * (D // 2) * 4),
        # reads the first D columns of each padded gradient row, writes dqkv
        "vision_rope_bwd": (lambda: e.vision_rope_bwd(dq, dk, dv, cos, sin, D), None,
                            3 * N * nh * D * 2 + N * 3 * H * 2 + 2 * N * (D // 2) * 4),
    }
    peak = _hbm_peak()
    for name, (ours, eager, nbytes) in cases.items():
        t = _time(ours, iters)
        row = {"case": name, "tokens": N, "ms": round(t, 4), "GB/s": round(nbytes / t / 1e6, 1),
               "frac_of_measured_hbm": round(nbytes / t / 1e6 / peak, 3) if peak else None}
        if eager is not None and _WITH_REF:
            te = _time(eager, iters)
            row["eager_ms"] = round(te, 4)
            row["speedup_vs_eager"] = round(te / t, 2)
        print(json.dumps(row), flush=True)


def _ext_mod():
    from mvp_engine.ops import _ext

    return _ext.ext()


def _hbm_peak() -> float:
    """Measured HBM copy bandwidth (GB/s) from the repository's peaks file, if present."""
    import os

    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 0.0


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attention", "peer_rs", "tp_gemm", "cp_attention", "cp_layer", "vision",
                                     "fsdp_gather", "comm_loopback"])
    ap.add_argument("--copy-ctas", type=int, default=24, help="fsdp_gather: copy CTAs carried by the GEMM")
    ap.add_argument("--loopback-world", type=int, default=2, help="fsdp_gather: local 'ranks' when run alone")
    ap.add_argument("--impls", default="ring,ring_fused,ulysses", help="cp_attention: cases to time")
    ap.add_argument("--docs", default="256,4096", help="attention: document lengths U[lo, hi]")
    ap.add_argument("--hidden", type=int, default=5120, help="tp_gemm: hidden size (square weights)")
    ap.add_argument("--mbytes", type=int, default=768, help="peer_rs: unit size in MiB")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--heads", default="32,8")
    ap.add_argument("--shape", default=None, help="M,N,K")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--no-ref", action="store_true", help="skip the library comparison columns")
    args = ap.parse_args()
    global _WITH_REF
    _WITH_REF = not args.no_ref
    if args.what == "gemm":
        shapes = QWEN3_8B_SHAPES
        if args.shape:
            M, N, K = (int(v) for v in args.shape.split(","))
            shapes = {"custom": (M, N, K)}
        bench_gemm(shapes, args.iters)
    elif args.what == "tp_gemm":
        bench_tp_gemm(args.tokens if args.tokens != 8192 else 4096, args.hidden, args.iters)
    elif args.what == "peer_rs":
        bench_peer_rs(args.mbytes, args.iters)
    elif args.what == "comm_loopback":
        bench_comm_loopback(args.tokens, args.hidden, args.mbytes, args.iters)
    elif args.what == "fsdp_gather":
        bench_fsdp_gather(args.tokens, args.iters, args.copy_ctas, args.loopback_world)
    elif args.what == "cp_layer":
        bench_cp_layer(args.tokens, args.iters, args.impls.split(","))
    elif args.what == "cp_attention":
        hq, hkv = (int(v) for v in args.heads.split(","))
        bench_cp_attention(args.tokens, hq, hkv, args.iters, args.impls.split(","))
    elif args.what == "vision":
        bench_vision(args.tokens if args.tokens != 8192 else 28224, args.iters)
    elif args.what == "attention":
        hq, hkv = (int(v) for v in args.heads.split(","))
        lo, hi = (int(v) for v in args.docs.split(","))
        bench_attention(args.tokens, hq, hkv, args.iters, lo, hi)


if __name__ == "__main__":
    main()
