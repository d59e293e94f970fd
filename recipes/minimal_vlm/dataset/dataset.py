"""Training stream of the minimal VLM recipe (reference: recipes/minimal_vlm/dataset/dataset.py:14-58):
a resampled source (parquet chat rows, or synthetic image+text rows) mapped through ``process_sample``;
dropped samples are filtered out."""

from __future__ import annotations

from functools import partial
from typing import Any

from mvp_engine.data import Dataset, RuntimeContext

from .preprocess import build_sample_spec, process_sample


def _kept(sample) -> bool:
    return sample is not None


def build_dataset(config: Any, *, processor: Any, parallel_mesh: Any = None):
    path = config.data.train_path
    if path is None:
        raise ValueError("Missing `data.train_path` for the minimal VLM recipe.")
    synthetic = config.data.dataset_source.startswith("synthetic") or path.startswith("synthetic")
    if parallel_mesh is not None and parallel_mesh.device_mesh is not None:
        ctx = RuntimeContext.from_runtime(seed=int(config.seed), device_mesh=parallel_mesh.device_mesh,
                                          dp_dims=parallel_mesh.dp.dim_names or None)
    else:
        ctx = RuntimeContext.from_runtime(seed=int(config.seed))
    source = "synthetic_mm" if synthetic and not config.data.dataset_source.startswith("synthetic") \
        else config.data.dataset_source
    ds = Dataset.from_source(source, path, context=ctx, resample=True)
    spec = build_sample_spec(processor, int(config.data.max_seq_len), synthetic)
    return ds.map(partial(process_sample, spec=spec)).filter(_kept)
