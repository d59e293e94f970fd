"""End-to-end numerics of the Qwen3 path on the native kernels (GPU)."""

import copy
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def _tiny(vocab=512, layers=2):
    from mvp_engine.models.qwen3 import build_qwen3

    return build_qwen3("mvp/qwen3-tiny", seed=3, vocab_size=vocab, num_hidden_layers=layers)


def _batch(T, vocab, cuts, device):
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, vocab, (1, T), generator=g)
    cu = torch.tensor([0] + cuts + [T], dtype=torch.int32)
    pos = torch.cat([torch.arange(int(b - a)) for a, b in zip(cu[:-1], cu[1:])]).view(1, T)
    return ids.to(device), cu.to(device), pos.to(device)


def _wrap(model):
    from mvp_engine.parallel.fsdp import NativeFSDP

    return NativeFSDP(model, group=None, device=torch.device("cuda"), param_dtype=torch.bfloat16)


@cuda
def test_native_forward_matches_eager_fp32():
    cpu_model = _tiny()
    gpu = _wrap(copy.deepcopy(cpu_model).cuda())
    T = 1024
    ids, cu, pos = _batch(T, 512, [300, 700], "cuda")
    with torch.no_grad():
        out = gpu(input_ids=ids, labels=ids, position_ids=pos, cu_seq_lens_q=cu, max_length_q=400)["loss"]
        ref = cpu_model(input_ids=ids.cpu(), labels=ids.cpu(), position_ids=pos.cpu(), cu_seq_lens_q=cu.cpu(),
                        max_length_q=400)["loss"]
    out = out.float().cpu()
    assert abs(out.mean().item() - ref.mean().item()) < 2e-2 * ref.mean().item()
    assert torch.corrcoef(torch.stack([out, ref]))[0, 1] > 0.98
    # untrained model on uniform tokens: loss ~ ln(V)
    assert abs(ref.mean().item() - math.log(512)) < 0.2


@cuda
def test_native_path_is_causal_within_documents():
    gpu = _wrap(_tiny(vocab=1000))
    T = 1024
    ids, cu, pos = _batch(T, 1000, [300, 700], "cuda")
    with torch.no_grad():
        a = gpu(input_ids=ids, labels=ids, position_ids=pos, cu_seq_lens_q=cu, max_length_q=400)["loss"].clone()
        ids2 = ids.clone()
        ids2[0, 500:] = (ids2[0, 500:] + 7) % 1000
        b = gpu(input_ids=ids2, labels=ids2, position_ids=pos, cu_seq_lens_q=cu, max_length_q=400)["loss"]
    # positions < 499 see neither the changed tokens nor a changed label
    assert torch.equal(a[:499], b[:499])
    # document isolation: a change inside doc 2 ([300, 700)) leaves doc 3 ([700, T)) depending only on itself,
    # and changing doc 3 only leaves docs 1-2 untouched
    ids3 = ids.clone()
    ids3[0, 800:] = (ids3[0, 800:] + 3) % 1000
    with torch.no_grad():
        c = gpu(input_ids=ids3, labels=ids3, position_ids=pos, cu_seq_lens_q=cu, max_length_q=400)["loss"]
    assert torch.equal(a[:799], c[:799])


@cuda
def test_native_grads_match_eager_fp32():
    cpu_model = _tiny()
    gpu = _wrap(copy.deepcopy(cpu_model).cuda())
    T = 512
    ids, cu, pos = _batch(T, 512, [200], "cuda")
    loss = gpu(input_ids=ids, labels=ids, position_ids=pos, cu_seq_lens_q=cu, max_length_q=312)["loss"].sum() / T
    loss.backward()
    ref = cpu_model(input_ids=ids.cpu(), labels=ids.cpu(), position_ids=pos.cpu(), cu_seq_lens_q=cu.cpu(),
                    max_length_q=312)["loss"].sum() / T
    ref.backward()
    grads = {}
    for u in gpu.units:
        for e in u.entries:
            grads[e.fqns[0]] = u.grad[e.offset:e.offset + e.numel].view(e.shape).cpu()
    for name, p in cpu_model.named_parameters():
        g = grads[name]
        rel = ((g - p.grad).norm() / (p.grad.norm() + 1e-12)).item()
        assert rel < 6e-2, (name, rel)


@cuda
def test_checkpointed_layers_accumulate_into_the_flat_buffer():
    """Activation checkpointing recomputes layers with detached aliases of the weights; their
    gradients must still land in the runtime's fp32 buffer through the GEMM epilogue (no bf16
    per-parameter .grad) and agree with the run without checkpointing."""
    model = _tiny(layers=3)
    runs = []
    for ckpt in (False, True):
        gpu = _wrap(copy.deepcopy(model).cuda())
        if ckpt:
            gpu.module.gradient_checkpointing_enable({"num_layers": 2})
        gpu.train()
        folded = []  # weights whose gradient came back through autograd's .grad (bf16) instead
        for u in gpu.units:
            for e in u.entries:
                if e.shape.numel() > 4096:  # matrices: every one goes through a native GEMM
                    for mod, pname in e.owners[:1]:
                        getattr(mod, pname).register_hook(
                            lambda g, n=e.fqns[0]: folded.append(n) if g is not None else None)
        T = 512
        ids, cu, pos = _batch(T, 512, [200], "cuda")
        loss = gpu(input_ids=ids, labels=ids, position_ids=pos, cu_seq_lens_q=cu, max_length_q=312)["loss"].sum()
        (loss / T).backward()
        torch.cuda.synchronize()
        assert not folded, f"gradients bypassed the fp32 buffer: {folded}"
        runs.append(torch.cat([u.grad.float().cpu() for u in gpu.units if u.trainable]))
    a, b = runs
    assert ((a - b).norm() / b.norm()).item() < 1e-3


@cuda
def test_ce_large_vocab():
    from mvp_engine import ops

    torch.manual_seed(0)
    h = (torch.randn(256, 512, device="cuda") * 0.5).bfloat16()
    w = (torch.randn(151936, 512, device="cuda") * 0.05).bfloat16()
    labels = torch.randint(0, 151936, (256,), device="cuda")
    loss = ops.fused_linear_cross_entropy(h, w, labels, chunk_size=128)
    ref = torch.nn.functional.cross_entropy(h.float() @ w.float().t(), labels, reduction="none")
    assert ((loss - ref).abs().max() < 5e-2), (loss - ref).abs().max()


@cuda
def test_vit_native_bf16_matches_fp32_and_trains():
    """ViT on the tcgen05 GEMM + padded flash attention under the native runtime vs fp32 eager on CPU;
    every parameter (biases, LayerNorm, CLS token included) receives gradient and moves."""
    from mvp_engine.models.vit import build_vit
    from mvp_engine.parallel.optim import FlatAdamW

    cpu = build_vit("vit-tiny-patch16-224", seed=1, num_hidden_layers=4, num_labels=100)
    gpu = _wrap(copy.deepcopy(cpu).cuda())
    g = torch.Generator().manual_seed(0)
    px = torch.randn(4, 3, 224, 224, generator=g)
    y = torch.randint(0, 100, (4,), generator=g)
    out = gpu(pixel_values=px.cuda(), labels=y.cuda())
    ref = cpu(pixel_values=px, labels=y)
    assert abs(out["loss"].item() - ref["loss"].item()) < 3e-2 * ref["loss"].item()
    assert torch.corrcoef(torch.stack([out["logits"].float().cpu().flatten(), ref["logits"].flatten()]))[0, 1] > 0.99
    before = {k: v.float().clone() for k, v in gpu.checkpoint_state_dict(full=True).items()}
    opt = FlatAdamW(gpu, lr=1e-3)
    out["loss"].backward()
    gpu.clip_grad_norm_(1e9)
    opt.step()
    torch.cuda.synchronize()
    after = gpu.checkpoint_state_dict(full=True)
    unchanged = [k for k, v in before.items() if torch.equal(v, after[k].float())]
    assert not unchanged, unchanged[:5]
