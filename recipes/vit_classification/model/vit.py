"""ViT classifier builder (reference: recipes/vit_classification/model/vit.py:8-35): the engine's
``ViTForImageClassification`` (HF parameter names) from the recipe's model config, random init unless
``load_pretrained_weights`` points at a local directory of ``*.safetensors``."""

from __future__ import annotations

import glob
import os

from mvp_engine.models.vit import ViTForImageClassification, build_vit


def build_vit_model(model_config, seed: int = 0, device=None) -> ViTForImageClassification:
    c = model_config
    model = build_vit(c.pretrained_model_name_or_path, seed=seed, device=device, image_size=c.image_size,
                      patch_size=c.patch_size, num_channels=c.num_channels, hidden_size=c.hidden_size,
                      intermediate_size=c.intermediate_size, num_hidden_layers=c.num_hidden_layers,
                      num_attention_heads=c.num_attention_heads, hidden_dropout_prob=c.hidden_dropout_prob,
                      attention_probs_dropout_prob=c.attention_dropout_prob, num_labels=c.num_classes)
    if c.load_pretrained_weights:
        files = sorted(glob.glob(os.path.join(c.pretrained_model_name_or_path, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"no *.safetensors under {c.pretrained_model_name_or_path!r}")
        from safetensors.torch import load_file

        sd = {}
        for f in files:
            sd.update(load_file(f))
        sd = {k: v for k, v in sd.items() if not k.startswith("classifier.") or
              v.shape[0] == c.num_classes}  # a new head when the class count differs
        model.load_state_dict(sd, strict=False)
    return model
