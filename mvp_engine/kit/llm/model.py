"""Text-LM model kit (reference: mvp_engine/kit/llm/model.py:19-156).

``build_model`` constructs the engine's own decoder (HF-compatible parameter
names, native kernels) from a preset name or a local HF directory: with
``load_pretrained_model`` it then loads ``*.safetensors`` weights from that
directory, otherwise it random-initialises with ``random_init_seed``.
"""

from __future__ import annotations

import glob
import os
from typing import Any, Callable, Literal

import torch

from ...models import build_causal_lm


def _matches(name: str, prefixes: tuple[str, ...]) -> bool:
    return any(name.startswith(p) for p in prefixes)


class LLMModelKit:
    def build_model(self, pretrained_model_name_or_path: str, *, load_pretrained_model: bool = True,
                    random_init_seed: int = 42, trust_remote_code: bool = True,
                    torch_dtype: str | torch.dtype = "auto", attn_implementation: str | None = None,
                    device: torch.device | str | None = None, **kwargs: Any):
        dtype = torch.float32 if torch_dtype in ("auto", None) else (
            getattr(torch, torch_dtype) if isinstance(torch_dtype, str) else torch_dtype)
        model = build_causal_lm(pretrained_model_name_or_path, seed=random_init_seed, dtype=dtype, device=device,
                                **kwargs)
        if load_pretrained_model:
            files = sorted(glob.glob(os.path.join(pretrained_model_name_or_path, "*.safetensors")))
            if not files:
                raise FileNotFoundError(f"no *.safetensors under {pretrained_model_name_or_path!r}")
            from safetensors.torch import load_file

            sd: dict[str, torch.Tensor] = {}
            for f in files:
                sd.update(load_file(f))
            missing, _ = model.load_state_dict(sd, strict=False)
            if missing:
                raise KeyError(f"pretrained weights miss {len(missing)} parameters, e.g. {missing[:3]}")
        return model

    def apply_freeze_policy(self, model: torch.nn.Module, freeze_llm: bool = False,
                            llm_prefixes: tuple[str, ...] | None = None) -> torch.nn.Module:
        if not freeze_llm:
            return model
        prefixes = llm_prefixes or ("model.", "transformer.", "backbone.", "decoder.", "language_model.", "lm_head.")
        for name, p in model.named_parameters():
            if _matches(name, prefixes):
                p.requires_grad = False
        return model

    def apply_gradient_checkpointing(self, model: torch.nn.Module, use_reentrant: bool = False,
                                     mode: Literal["hf", "custom", "hf_with_custom"] = "hf",
                                     target_modules: list[str] | None = None,
                                     num_layers: int | None = None) -> torch.nn.Module:
        """``hf`` mode checkpoints every decoder layer (or the first ``num_layers``);
        ``custom`` wraps ``Parent:child`` modules with torch's checkpoint wrapper."""
        if mode in ("hf", "hf_with_custom"):
            if not hasattr(model, "gradient_checkpointing_enable"):
                raise AttributeError(f"{type(model).__name__} does not support gradient checkpointing.")
            model.gradient_checkpointing_enable(
                gradient_checkpointing_kwargs={"use_reentrant": use_reentrant, "num_layers": num_layers})
            if mode == "hf":
                return model
        if not target_modules:
            raise ValueError("`target_modules` is required when gradient checkpointing mode uses custom wrappers.")
        from torch.distributed.algorithms._checkpoint.checkpoint_wrapper import CheckpointImpl, checkpoint_wrapper

        impl = CheckpointImpl.REENTRANT if use_reentrant else CheckpointImpl.NO_REENTRANT
        pairs = []
        for spec in target_modules:
            if ":" not in spec:
                raise ValueError(f"Invalid target module name '{spec}'. Expected format 'parent_module:child_module'.")
            parent, child = (s.strip() for s in spec.split(":"))
            pairs.append((parent, child))
        for parent in model.modules():
            for pname, cname in pairs:
                if type(parent).__name__ != pname:
                    continue
                for name, child in list(parent.named_children()):
                    if name == cname and not hasattr(child, "_checkpoint_wrapped_module"):
                        parent.add_module(name, checkpoint_wrapper(child, checkpoint_impl=impl,
                                                                   preserve_rng_state=False))
        return model

    def apply_model_compile(self, model: torch.nn.Module, backend: str, mode: str) -> torch.nn.Module:
        """``model.compile`` as the reference offers it; the native kernels are opaque to the compiler."""
        model.compile(backend=backend, mode=mode)
        return model

    def apply_model_patches(self, model: torch.nn.Module,
                            patch_fns: Callable | list[Callable]) -> torch.nn.Module:
        for fn in (patch_fns if isinstance(patch_fns, list) else [patch_fns]):
            model = fn(model)
        return model
