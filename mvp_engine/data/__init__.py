"""Minimal streaming dataset runtime.

The reference builds its pipelines on the external ``mvp_dataset`` package
(imported in mvp_engine/kit/llm/data/data.py:10-11 and
mvp_engine/kit/llm/data/packing.py:9-10), which is not part of the reference
repository.  This module implements the part of that contract the kits use:

* ``Dataset.from_source(kind, path, context=..., resample=..., shuffle_mode=...)``
  followed by ``.map(fn)``, ``.filter(fn)`` and ``.assemble(factory)``;
* ``Assembler`` objects with ``push / finish / state_dict / load_state_dict /
  fingerprint`` (stateful N->M stream transforms such as packers and guards);
* ``RuntimeContext`` carrying the seed and the data-parallel rank/world, so
  each rank (and each loader worker) reads a disjoint slice of the source;
* ``TorchLoader(dataset, ...).batch(batch_size, drop_last, collate_fn)``;
* ``stable_fingerprint``.

Sources: ``synthetic_text`` / ``synthetic_mm`` (the shapes of the benchmark
configurations: uniform token ids, document lengths U[lo, hi], images with
H, W in multiples of 32), ``jsonl``, ``parquet`` (pyarrow) and ``lance`` when
that package is importable.
"""

from .runtime import (Assembler, Dataset, RuntimeContext, TorchLoader, register_source, stable_fingerprint)
from .synthetic import SyntheticTokenizer

__all__ = ["Assembler", "Dataset", "RuntimeContext", "TorchLoader", "register_source", "stable_fingerprint",
           "SyntheticTokenizer"]
