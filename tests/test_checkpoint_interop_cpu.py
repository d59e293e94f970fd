"""Checkpoint format: the native runtime and torch FSDP2 read each other's DCP checkpoints (gloo, world 2),
the DCP keys follow ``model.<fqn>`` / ``optimizer.state.<fqn>.<field>``, and ``hf_model/model.safetensors``
loads into Hugging Face's own Qwen3 class (reference layout: mvp_engine/utils/checkpointing/
parallel_sl_util.py:224-440)."""

import pytest
import torch

from mvp_engine.testing import spawn_workers

TINY = dict(seed=5, vocab_size=256, hidden_size=128, intermediate_size=256, num_attention_heads=2,
            num_key_value_heads=1, num_hidden_layers=2)


def _model():
    from mvp_engine.models.qwen3 import build_qwen3

    return build_qwen3("mvp/qwen3-tiny", **TINY)


def _train(model, opt, steps, rank, seed=9):
    g = torch.Generator().manual_seed(seed)
    for _ in range(steps):
        x = torch.randint(0, 256, (2, 32), generator=g)[rank:rank + 1]
        out = model(input_ids=x, labels=x)
        (out["loss"].sum() / 31).backward()
        opt.step()
        opt.zero_grad(set_to_none=True)


def _native(mesh):
    import torch.distributed as dist

    from mvp_engine.parallel.fsdp import NativeFSDP
    from mvp_engine.parallel.optim import FlatAdamW

    m = NativeFSDP(_model(), group=dist.group.WORLD, device=torch.device("cpu"), param_dtype=torch.float32,
                   shard_mesh=mesh)
    return m, FlatAdamW(m, lr=1e-2, weight_decay=0.0)


def _torch_fsdp2(mesh):
    from torch.distributed.fsdp import fully_shard

    m = _model()
    for layer in m.model.layers:
        fully_shard(layer, mesh=mesh)
    fully_shard(m, mesh=mesh)
    return m, torch.optim.AdamW(m.parameters(), lr=1e-2, weight_decay=0.0)


def _full_params(model):
    from mvp_engine.utils.checkpointing.parallel_sl_util import model_state_dict

    return {k: v.detach().float().clone() for k, v in model_state_dict(model, full=True).items()}


def _exp_avg(model, opt):
    from mvp_engine.utils.checkpointing.parallel_sl_util import optimizer_state_dict

    st = optimizer_state_dict(model, opt, full=True).get("state", {})  # torch fills rank 0 only
    return {k: v["exp_avg"].detach().float().clone() for k, v in st.items() if "exp_avg" in v}


def _roundtrip(rank, world, port, src_kind, dst_kind, path):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    from mvp_engine.utils.checkpointing.parallel_sl_util import load_checkpoint, save_checkpoint
    from mvp_engine.distributed.init import initialize_process_group

    initialize_process_group()
    mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("shard",))
    build = {"native": _native, "fsdp2": _torch_fsdp2}
    src, src_opt = build[src_kind](mesh)
    _train(src, src_opt, 2, rank)
    save_checkpoint(mesh, path, src, src_opt, step=2)
    dist.barrier()
    want_p, want_m = _full_params(src), _exp_avg(src, src_opt)
    dst, dst_opt = build[dst_kind](mesh)
    if dst_kind == "fsdp2":  # torch optimizers create their state lazily: take one zero-lr step first
        for g in dst_opt.param_groups:
            g["lr"] = 0.0
        _train(dst, dst_opt, 1, rank, seed=1)
        for g in dst_opt.param_groups:
            g["lr"] = 1e-2
    load_checkpoint(mesh, path, dst, dst_opt, restore_engine_state=False)
    got_p, got_m = _full_params(dst), _exp_avg(dst, dst_opt)
    dist.barrier()
    if rank != 0:  # torch gathers full state dicts on rank 0 only
        return {}, {}, [], []
    return ({k: float((got_p[k] - v).abs().max()) for k, v in want_p.items()},
            {k: float((got_m[k] - v).abs().max()) for k, v in want_m.items()}, sorted(want_p), sorted(got_p))


@pytest.mark.parametrize("src,dst", [("native", "fsdp2"), ("fsdp2", "native")])
def test_dcp_checkpoint_loads_across_runtimes(tmp_path, src, dst):
    res = spawn_workers(_roundtrip, 2, src, dst, str(tmp_path / "iter_2"), timeout=300)
    for pdiff, mdiff, want_keys, got_keys in res[:1]:  # full state dicts are gathered on rank 0
        assert want_keys == got_keys
        assert pdiff and max(pdiff.values()) < 1e-6, pdiff
        assert mdiff and max(mdiff.values()) < 1e-6, mdiff
    # DCP key layout of the saved files
    import torch.distributed.checkpoint as dcp

    mkeys = set(dcp.FileSystemReader(str(tmp_path / "iter_2" / "model")).read_metadata().state_dict_metadata)
    okeys = set(dcp.FileSystemReader(str(tmp_path / "iter_2" / "optimizer")).read_metadata().state_dict_metadata)
    assert "model.model.layers.1.self_attn.q_proj.weight" in mkeys
    assert "model.lm_head.weight" in mkeys
    for field in ("step", "exp_avg", "exp_avg_sq"):
        assert f"optimizer.state.model.layers.0.mlp.down_proj.weight.{field}" in okeys, sorted(okeys)[:8]


def _hf_export(rank, world, port, path):
    import torch.distributed as dist
    from torch.distributed.device_mesh import init_device_mesh

    from mvp_engine.distributed.init import initialize_process_group
    from mvp_engine.utils.checkpointing.parallel_sl_util import save_checkpoint

    initialize_process_group()
    mesh = init_device_mesh("cpu", (world,), mesh_dim_names=("shard",))
    model, opt = _native(mesh)
    _train(model, opt, 1, rank)
    save_checkpoint(mesh, path, model, opt, step=1, hf_enable=True)
    dist.barrier()
    return _full_params(model)


def test_hf_export_loads_into_transformers_qwen3(tmp_path):
    transformers = pytest.importorskip("transformers")
    from safetensors.torch import load_file

    from mvp_engine.models.qwen3 import load_qwen3_config

    full = spawn_workers(_hf_export, 2, str(tmp_path / "iter_1"), timeout=300)[0]
    sd = load_file(str(tmp_path / "iter_1" / "hf_model" / "model.safetensors"))
    cfg = load_qwen3_config("mvp/qwen3-tiny", **{k: v for k, v in TINY.items() if k != "seed"})
    hf_cfg = transformers.Qwen3Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                                      intermediate_size=cfg.intermediate_size,
                                      num_hidden_layers=cfg.num_hidden_layers,
                                      num_attention_heads=cfg.num_attention_heads,
                                      num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                                      tie_word_embeddings=False)
    hf = transformers.Qwen3ForCausalLM(hf_cfg)
    missing, unexpected = hf.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert not [k for k in missing if "rotary" not in k], missing
    for k, v in full.items():
        assert torch.equal(sd[k].float(), v), k
