"""Qwen3-VL model on CPU: vision metadata, forward/backward, image-token scatter, FLOPs."""

import torch

from mvp_engine.models.qwen3_vl import build_qwen3_vl, vision_metadata


def _inputs(model, grids):
    c = model.config
    vc = c.vision_config
    n_patches = sum(t * h * w for t, h, w in grids)
    pix = torch.randn(n_patches, vc.in_channels * vc.temporal_patch_size * vc.patch_size ** 2)
    ids = []
    for t, h, w in grids:
        n_tok = t * h * w // vc.spatial_merge_size ** 2
        ids += [5, 6, c.vision_start_token_id] + [c.image_token_id] * n_tok + [c.vision_end_token_id]
    ids += list(range(7, 40))
    ids = torch.tensor(ids).view(1, -1)
    labels = ids.clone()
    labels[ids == c.image_token_id] = -100
    return ids, labels, pix, torch.tensor(grids)


def test_vision_metadata_layout():
    from mvp_engine.models.qwen3_vl import Qwen3VLVisionConfig

    m = vision_metadata([[1, 4, 6]], Qwen3VLVisionConfig(num_position_embeddings=256), 16, 36)
    assert m["rope_angles"].shape == (24, 36)
    assert m["pos_idx"].shape == (4, 24) and torch.allclose(m["pos_w"].sum(0), torch.ones(24))
    assert m["cu_seqlens"].tolist() == [0, 24]


def test_forward_backward_and_image_scatter():
    torch.manual_seed(0)
    model = build_qwen3_vl("mvp/qwen3-vl-tiny", seed=0)
    ids, labels, pix, grid = _inputs(model, [[1, 4, 4], [1, 4, 8]])
    out = model(input_ids=ids, labels=labels, pixel_values=pix, image_grid_thw=grid)
    loss = out["loss"]
    n_sup = int((torch.nn.functional.pad(labels, (0, 1), value=-100)[..., 1:] != -100).sum())
    assert loss.shape == (ids.numel(),) and int((loss != 0).sum()) <= n_sup
    loss.sum().backward()
    g = model.model.visual.patch_embed.proj.weight.grad
    assert g is not None and g.abs().sum() > 0, "vision tower must receive gradient through the image tokens"
    assert model.model.visual.deepstack_merger_list[0].linear_fc2.weight.grad.abs().sum() > 0
    fl = model.calculate_model_flops(batch_size=1, seq_len=ids.shape[1], image_grid_thw=grid)
    assert fl > 0


def test_vision_op_fallbacks_match_eager_math():
    """CPU paths of the vision-tower ops (LayerNorm, bias + GELU, padded RoPE) equal the eager formulas."""
    from mvp_engine import ops

    torch.manual_seed(0)
    N, nh, D = 7, 2, 8
    qkv = torch.randn(N, 3 * nh * D)
    ang = torch.rand(N, D // 2) * 10
    q, k, v = ops.vision_rope_pad(qkv, nh, ang.cos(), ang.sin(), 16)
    t = qkv.view(N, 3, nh, D)
    c = torch.cat([ang.cos(), ang.cos()], -1).unsqueeze(1)
    s = torch.cat([ang.sin(), ang.sin()], -1).unsqueeze(1)
    rq = t[:, 0] * c + torch.cat((-t[:, 0, :, D // 2:], t[:, 0, :, :D // 2]), -1) * s
    assert torch.allclose(q[..., :D], rq, atol=1e-6) and q[..., D:].abs().max() == 0
    assert torch.equal(v[..., :D], t[:, 2])
    x, b = torch.randn(5, 16), torch.randn(16)
    assert torch.allclose(ops.bias_gelu(x, b, "tanh"), torch.nn.functional.gelu(x + b, approximate="tanh"))
    w = torch.randn(16)
    assert torch.allclose(ops.layer_norm(x, w, b, 1e-6), torch.nn.functional.layer_norm(x, (16,), w, b, 1e-6))
