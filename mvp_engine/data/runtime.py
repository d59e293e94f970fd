"""Streaming dataset pipeline, assemblers, rank/worker sharding and the torch loader."""

from __future__ import annotations

import array
import bisect
import hashlib
import itertools
import json
import os
import random
from dataclasses import dataclass, field
from typing import Any, Callable, Generic, Iterable, Iterator, Optional, Sequence, TypeVar

import torch
import torch.distributed as dist

I = TypeVar("I")
O = TypeVar("O")


def stable_fingerprint(obj: Any) -> str:
    """Deterministic short hash of a JSON-able description (resume compatibility checks)."""
    blob = json.dumps(obj, sort_keys=True, default=repr).encode()
    return hashlib.sha256(blob).hexdigest()[:16]


class Assembler(Generic[I, O]):
    """Stateful stream transform: ``push`` one item, get zero or more items back."""

    def push(self, item: I) -> Iterable[O]:
        raise NotImplementedError

    def finish(self, *, drop_last: bool = False) -> Iterable[O]:
        return []

    def state_dict(self) -> dict[str, object]:
        return {}

    def load_state_dict(self, state: dict[str, object]) -> None:
        if state:
            raise ValueError(f"{type(self).__name__} does not have resumable state.")

    def fingerprint(self) -> str:
        return stable_fingerprint({"kind": type(self).__name__})


@dataclass
class RuntimeContext:
    """Seed plus this process's slice of the source (data-parallel rank x loader worker)."""

    seed: int = 42
    dp_rank: int = 0
    dp_world: int = 1
    worker_id: int = 0
    num_workers: int = 1
    epoch: int = 0

    @classmethod
    def from_runtime(cls, seed: int = 42, device_mesh: Any = None,
                     dp_dims: Optional[str | Sequence[str]] = None) -> "RuntimeContext":
        rank, world = 0, 1
        if device_mesh is not None and dp_dims:
            dims = (dp_dims,) if isinstance(dp_dims, str) else tuple(dp_dims)
            dims = tuple(d for d in dims if d in (device_mesh.mesh_dim_names or ()))
            if dims:
                sub = device_mesh[dims[0]] if len(dims) == 1 else device_mesh[dims]
                coords = sub.get_coordinate()
                sizes = [device_mesh[d].size() for d in dims]
                if coords is not None:
                    rank = 0
                    for c, s in zip(coords, sizes):
                        rank = rank * s + c
                world = 1
                for s in sizes:
                    world *= s
        elif dist.is_available() and dist.is_initialized():
            rank, world = dist.get_rank(), dist.get_world_size()
        return cls(seed=seed, dp_rank=rank, dp_world=world)

    @property
    def shard_index(self) -> int:
        return self.dp_rank * self.num_workers + self.worker_id

    @property
    def num_shards(self) -> int:
        return self.dp_world * self.num_workers

    def rng(self, salt: str = "") -> random.Random:
        key = f"{self.seed}:{self.shard_index}:{self.num_shards}:{self.epoch}:{salt}"
        return random.Random(int(hashlib.sha256(key.encode()).hexdigest()[:16], 16))


# ----------------------------------------------------------------- sources
SourceFn = Callable[[str, RuntimeContext, dict], Iterator[dict]]
_SOURCES: dict[str, SourceFn] = {}


def register_source(name: str) -> Callable[[SourceFn], SourceFn]:
    def deco(fn: SourceFn) -> SourceFn:
        _SOURCES[name] = fn
        return fn

    return deco


class _JsonlRows:
    """Rows of a ``.jsonl`` file, parsed on demand: the index holds the byte offset of each non-blank
    line (8 bytes per row), so a corpus is never held as Python objects, on any rank."""

    def __init__(self, path: str) -> None:
        self.path = path
        offsets, pos = [], 0
        with open(path, "rb") as f:
            for line in f:
                if line.strip():
                    offsets.append(pos)
                pos += len(line)
        self.offsets = array.array("q", offsets)

    def __len__(self) -> int:
        return len(self.offsets)

    def take(self, indices: Sequence[int]) -> list[dict]:
        out = []
        with open(self.path, "rb") as f:
            for i in indices:
                f.seek(self.offsets[i])
                out.append(json.loads(f.readline()))
        return out


class _ParquetRows:
    """Rows of a ``.parquet`` file: one memory-mapped Arrow table, rows converted per chunk."""

    def __init__(self, path: str) -> None:
        import pyarrow.parquet as pq

        self.table = pq.read_table(path, memory_map=True)

    def __len__(self) -> int:
        return self.table.num_rows

    def take(self, indices: Sequence[int]) -> list[dict]:
        return self.table.take(list(indices)).to_pylist()


class _ListRows:
    def __init__(self, rows: list) -> None:
        self.rows = rows

    def __len__(self) -> int:
        return len(self.rows)

    def take(self, indices: Sequence[int]) -> list[dict]:
        return [self.rows[i] for i in indices]


class _ConcatRows:
    """Several row sources seen as one, global index = offset of the part + index within it."""

    def __init__(self, parts: list) -> None:
        self.parts = parts
        self.starts = list(itertools.accumulate((len(p) for p in parts), initial=0))

    def __len__(self) -> int:
        return self.starts[-1]

    def take(self, indices: Sequence[int]) -> list[dict]:
        out = []
        for i in indices:
            k = bisect.bisect_right(self.starts, i) - 1
            out.extend(self.parts[k].take([i - self.starts[k]]))
        return out


_ROW_SOURCES: dict[tuple, Any] = {}


def _open_rows(path: str):
    """Row source of a file (``.jsonl``, ``.parquet``, ``.json`` list, or a ``.json`` manifest
    ``{"files": [...]}`` of such files, relative to the manifest), built once per process and file
    version and shared by every epoch."""
    st = os.stat(path)
    key = (os.path.abspath(path), st.st_size, st.st_mtime_ns)
    src = _ROW_SOURCES.get(key)
    if src is not None:
        return src
    if path.endswith(".jsonl"):
        src = _JsonlRows(path)
    elif path.endswith(".parquet"):
        src = _ParquetRows(path)
    elif path.endswith(".json"):
        with open(path) as f:
            data = json.load(f)
        if isinstance(data, dict) and "files" in data:
            base = os.path.dirname(path)
            src = _ConcatRows([_open_rows(os.path.join(base, fp)) for fp in data["files"]])
        else:
            src = _ListRows(list(data))
    else:
        raise ValueError(f"Unsupported file source: {path}")
    _ROW_SOURCES[key] = src
    return src


def _read_rows(path: str) -> list[dict]:
    """Every row of a file source, in file order."""
    src = _open_rows(path)
    return src.take(range(len(src)))


@register_source("jsonl")
@register_source("json")
@register_source("parquet")
def _file_source(path: str, ctx: RuntimeContext, opts: dict) -> Iterator[dict]:
    src = _open_rows(path)
    if opts.get("shuffle_mode", "none") != "none":
        order = list(range(len(src)))
        RuntimeContext(seed=ctx.seed, epoch=ctx.epoch).rng("order").shuffle(order)
        mine = order[ctx.shard_index::ctx.num_shards]
    else:  # file order: this shard's indices without materialising the others
        mine = range(ctx.shard_index, len(src), ctx.num_shards)
    for s in range(0, len(mine), 256):
        chunk = mine[s:s + 256]
        for i, row in zip(chunk, src.take(chunk)):
            yield dict(row, __global_index__=i)


@register_source("lance")
def _lance_source(path: str, ctx: RuntimeContext, opts: dict) -> Iterator[dict]:
    try:
        import lance  # type: ignore
    except ImportError as exc:  # pragma: no cover - optional dependency
        raise RuntimeError("the 'lance' source needs the lance package; use jsonl/parquet/synthetic") from exc
    ds = lance.dataset(path)
    n = ds.count_rows()
    idx = list(range(n))
    if opts.get("shuffle_mode", "none") != "none":
        RuntimeContext(seed=ctx.seed, epoch=ctx.epoch).rng("order").shuffle(idx)
    mine = idx[ctx.shard_index::ctx.num_shards]
    for s in range(0, len(mine), 256):
        tbl = ds.take(mine[s:s + 256])
        for j, row in enumerate(tbl.to_pylist()):
            yield dict(row, __global_index__=mine[s + j])


# ---------------------------------------------------------------- pipeline
@dataclass
class _Stage:
    kind: str  # map | filter | assemble
    fn: Any


class Dataset:
    """Lazily composed stream: source -> stages.  Iterating builds fresh stage state."""

    def __init__(self, kind: str, path: str, context: RuntimeContext, resample: bool = False,
                 shuffle_mode: str = "none", stages: Optional[list[_Stage]] = None, options: Optional[dict] = None):
        if kind not in _SOURCES:
            from . import synthetic  # noqa: F401  (registers the synthetic sources)
        if kind not in _SOURCES:
            raise ValueError(f"Unknown dataset source {kind!r}; known: {sorted(_SOURCES)}")
        self.kind = kind
        self.path = path
        self.context = context
        self.resample = resample
        self.shuffle_mode = shuffle_mode
        self.stages: list[_Stage] = list(stages or [])
        self.options = dict(options or {})
        self._live_assemblers: list[Assembler] = []

    @classmethod
    def from_source(cls, kind: str, path: str, *, context: Optional[RuntimeContext] = None, resample: bool = False,
                    shuffle_mode: str = "none", **options: Any) -> "Dataset":
        return cls(kind, path, context or RuntimeContext(), resample, shuffle_mode, options=options)

    def _with(self, stage: _Stage) -> "Dataset":
        return Dataset(self.kind, self.path, self.context, self.resample, self.shuffle_mode,
                       self.stages + [stage], self.options)

    def map(self, fn: Callable[[Any], Any]) -> "Dataset":
        return self._with(_Stage("map", fn))

    def filter(self, fn: Callable[[Any], bool]) -> "Dataset":
        return self._with(_Stage("filter", fn))

    def assemble(self, factory: Callable[..., Assembler]) -> "Dataset":
        return self._with(_Stage("assemble", factory))

    def with_context(self, context: RuntimeContext) -> "Dataset":
        return Dataset(self.kind, self.path, context, self.resample, self.shuffle_mode, self.stages, self.options)

    def _rows(self) -> Iterator[dict]:
        ctx = RuntimeContext(**{**self.context.__dict__})
        opts = {"shuffle_mode": self.shuffle_mode, **self.options}
        for epoch in itertools.count():
            ctx.epoch = epoch
            yield from _SOURCES[self.kind](self.path, ctx, opts)
            if not self.resample:
                return

    def __iter__(self) -> Iterator[Any]:
        stream: Iterable[Any] = self._rows()
        self._live_assemblers = []
        for st in self.stages:
            if st.kind == "map":
                stream = map(st.fn, stream)
            elif st.kind == "filter":
                stream = filter(st.fn, stream)
            else:
                asm = st.fn(self.context) if _accepts_context(st.fn) else st.fn()
                self._live_assemblers.append(asm)
                stream = _run_assembler(asm, stream)
        return iter(stream)

    def consume(self, factory: Callable[[RuntimeContext], Any]) -> Any:
        """Feed the (finite) stream into ``factory(context)``: ``push(item)`` returns False to stop
        early; the consumer's ``finish()`` value is returned."""
        consumer = factory(self.context)
        for item in self:
            if consumer.push(item) is False:
                break
        return consumer.finish()

    def state_dict(self) -> dict:
        return {"assemblers": [a.state_dict() for a in self._live_assemblers],
                "fingerprints": [a.fingerprint() for a in self._live_assemblers]}


def _accepts_context(factory: Any) -> bool:
    import functools
    import inspect

    fn = factory.func if isinstance(factory, functools.partial) else factory
    try:
        params = list(inspect.signature(fn).parameters.values())
    except (TypeError, ValueError):
        return False
    bound = len(factory.args) if isinstance(factory, functools.partial) else 0
    positional = [p for p in params if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD) and p.name != "self"]
    return len(positional) > bound and positional[bound].name in ("assemble_context", "context")


def _run_assembler(asm: Assembler, stream: Iterable[Any]) -> Iterator[Any]:
    for item in stream:
        yield from asm.push(item)
    yield from asm.finish()


# ------------------------------------------------------------------ loader
class _IterWrapper(torch.utils.data.IterableDataset):
    def __init__(self, dataset: Dataset):
        super().__init__()
        self.dataset = dataset

    def __iter__(self):
        info = torch.utils.data.get_worker_info()
        ds = self.dataset
        if info is not None and info.num_workers > 1:
            ctx = RuntimeContext(**{**ds.context.__dict__, "worker_id": info.id, "num_workers": info.num_workers})
            ds = ds.with_context(ctx)
        return iter(ds)


class MappedLoader:
    """Iterable of ``fn(batch)`` over another loader's batches (host-side, in the training process)."""

    def __init__(self, loader: Any, fn: Callable) -> None:
        self.loader, self.fn = loader, fn

    def __iter__(self):
        for b in self.loader:
            yield self.fn(b)

    def map(self, fn: Callable) -> "MappedLoader":
        return MappedLoader(self, fn)

    def state_dict(self) -> Optional[dict]:
        inner = getattr(self.loader, "state_dict", None)
        return inner() if callable(inner) else None

    def load_state_dict(self, state: dict) -> None:
        inner = getattr(self.loader, "load_state_dict", None)
        if callable(inner):
            inner(state)


class BatchLoader(torch.utils.data.DataLoader):
    """torch ``DataLoader`` with ``map(fn)`` for per-batch host transforms and a resumable position.

    The position is the number of batches handed out since the current pass began.  Sources are
    seeded and the pipeline is deterministic, so a restored loader reproduces its stream by drawing
    and dropping that many batches at the start of its next pass (exact, at the cost of re-reading
    them)."""

    _handed_out = 0
    _fast_forward = 0

    def map(self, fn: Callable) -> MappedLoader:
        return MappedLoader(self, fn)

    def __iter__(self):
        source = super().__iter__()
        skip, self._fast_forward = self._fast_forward, 0
        self._handed_out = 0
        return self._positioned(source, skip)

    def _positioned(self, source, skip: int):
        for _ in range(skip):
            try:
                next(source)
            except StopIteration:
                return
            self._handed_out += 1
        for batch in source:
            self._handed_out += 1
            yield batch

    def state_dict(self) -> dict:
        return {"batches_into_pass": int(self._handed_out)}

    def load_state_dict(self, state: dict) -> None:
        self._fast_forward = int(state.get("batches_into_pass", 0))


class TorchLoader:
    """torch DataLoader front-end over a :class:`Dataset` (workers shard the stream)."""

    def __init__(self, dataset: Dataset, num_workers: int = 0, pin_memory: bool = False,
                 persistent_workers: bool = False, multiprocessing_context: Optional[str] = "spawn"):
        self.dataset = dataset
        self.num_workers = int(num_workers)
        self.pin_memory = bool(pin_memory)
        self.persistent_workers = bool(persistent_workers) and self.num_workers > 0
        self.multiprocessing_context = multiprocessing_context if self.num_workers > 0 else None

    def batch(self, batch_size: int, drop_last: bool = True, collate_fn: Optional[Callable] = None):
        return BatchLoader(
            _IterWrapper(self.dataset), batch_size=batch_size, drop_last=drop_last, collate_fn=collate_fn,
            num_workers=self.num_workers, pin_memory=self.pin_memory, persistent_workers=self.persistent_workers,
            multiprocessing_context=self.multiprocessing_context)
