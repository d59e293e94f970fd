"""Multimodal model kit (reference: mvp_engine/kit/mllm/model.py:19-145)."""

from __future__ import annotations

from typing import Any, Callable, Literal

import torch

from ..llm.model import LLMModelKit, _matches


class MLLMModelKit:
    def build_model(self, pretrained_model_name_or_path: str, *, trust_remote_code: bool = True,
                    torch_dtype: str | torch.dtype = "auto", attn_implementation: str | None = None,
                    load_pretrained_model: bool = False, random_init_seed: int = 42,
                    device: torch.device | str | None = None, **kwargs: Any):
        """The engine's Qwen3-VL (HF names); pretrained ``*.safetensors`` loaded when requested."""
        return LLMModelKit().build_model(pretrained_model_name_or_path, load_pretrained_model=load_pretrained_model,
                                         random_init_seed=random_init_seed, torch_dtype=torch_dtype, device=device,
                                         **kwargs)

    def apply_freeze_policy(self, model: torch.nn.Module, freeze_vit: bool = False, freeze_projector: bool = False,
                            freeze_llm: bool = False, vit_prefixes: tuple[str, ...] | None = None,
                            projector_prefixes: tuple[str, ...] | None = None,
                            llm_prefixes: tuple[str, ...] | None = None) -> torch.nn.Module:
        vit = vit_prefixes or ("model.visual.patch_embed.", "model.visual.blocks.", "model.visual.pos_embed.")
        proj = projector_prefixes or ("model.visual.merger.", "model.visual.deepstack_merger_list.")
        llm = llm_prefixes or ("model.language_model.", "lm_head.")
        for name, p in model.named_parameters():
            if (freeze_vit and _matches(name, vit)) or (freeze_projector and _matches(name, proj)) or \
                    (freeze_llm and _matches(name, llm)):
                p.requires_grad = False
        return model

    def apply_gradient_checkpointing(self, model: torch.nn.Module, use_reentrant: bool = False,
                                     mode: Literal["hf", "custom", "hf_with_custom"] = "hf",
                                     target_modules: list[str] | None = None,
                                     num_layers: int | None = None) -> torch.nn.Module:
        return LLMModelKit().apply_gradient_checkpointing(model, use_reentrant, mode, target_modules, num_layers)

    def apply_model_compile(self, model: torch.nn.Module, backend: str, mode: str) -> torch.nn.Module:
        """Compile the language model only; the vision forward stays eager (variable image shapes)."""
        visual = getattr(getattr(model, "model", model), "visual", None)
        if visual is not None:
            visual.forward = torch.compiler.disable(visual.forward)
        model.compile(backend=backend, mode=mode)
        return model

    def apply_model_patches(self, model: torch.nn.Module, patch_fns: Callable | list[Callable]) -> torch.nn.Module:
        return LLMModelKit().apply_model_patches(model, patch_fns)
