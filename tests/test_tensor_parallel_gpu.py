"""Fused tensor-parallel GEMMs over NVLink (push all-gather into the GEMM, routed-epilogue
reduce-scatter) against the NCCL path, on 2 GPUs."""

import pytest
import torch

from mvp_engine.testing import spawn_workers

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 CUDA devices")


def _worker(rank, world, port, fused):
    import os

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist

    import mvp_engine.parallel.tensor_parallel as tpm

    tpm._FUSED_ROW = True  # exercise both fused halves

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.kit.llm.data.collator import varlen_metadata
    from mvp_engine.models.qwen3 import build_qwen3
    from mvp_engine.ops import _ext
    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.tensor_parallel import apply_native_tensor_parallel

    initialize_process_group()
    dev = torch.device("cuda", torch.cuda.current_device())
    model = build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=512, hidden_size=512, intermediate_size=1024,
                        num_attention_heads=4, num_key_value_heads=2, num_hidden_layers=2)
    tp = apply_native_tensor_parallel(model, group=dist.group.WORLD, sequence_parallel=True, fused=fused)
    fsdp = NativeFSDP(model.to(dev), group=None, device=dev, param_dtype=torch.bfloat16, tp_group=dist.group.WORLD)
    g = torch.Generator().manual_seed(4)
    T = 1024
    ids = torch.randint(0, 512, (1, T), generator=g).to(dev)
    seg = torch.tensor([[1] * 400 + [2] * 624])
    cu, mx, pos = varlen_metadata(seg)
    out = fsdp(input_ids=ids, labels=ids, position_ids=pos.to(dev), cu_seq_lens_q=cu.to(dev), max_length_q=mx)
    loss = out["loss"].sum()
    loss.backward()
    fsdp.finish_grad_sync()
    torch.cuda.synchronize()
    _ext.check_status(dev)
    total = loss.detach().float().clone()
    dist.all_reduce(total)
    grads = [u.grad.detach().float().cpu().clone() for u in fsdp.units if u.trainable]
    used_peer = getattr(tp, "_peer", None) is not None
    dist.barrier()
    return float(total), grads, used_peer


@two_gpus
def test_fused_tensor_parallel_matches_nccl_path():
    fused = spawn_workers(_worker, 2, True, timeout=300)
    plain = spawn_workers(_worker, 2, False, timeout=300)
    for (lf, gf, used), (lp, gp, used_p) in zip(fused, plain):
        assert used and not used_p
        assert abs(lf - lp) < 2e-3 * abs(lp), (lf, lp)
        for a, b in zip(gf, gp):
            assert ((a - b).norm() / (b.norm() + 1e-12)).item() < 2e-2
