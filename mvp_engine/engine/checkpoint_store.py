"""Checkpoint directory bookkeeping: tags, completion markers and retention.

The on-disk layout inside each checkpoint directory is written by
``mvp_engine.utils.checkpointing.save_checkpoint`` (the reference's layout,
``mvp_engine/utils/checkpointing/parallel_sl_util.py:224-316`` there).  This module
owns the level above it, ``<project>/checkpoints/<policy>_<n>/``, and makes the
directory set safe to resume from after a crash at any point:

* a directory counts as a checkpoint only once its ``COMPLETE`` marker exists; the
  marker is written last, through a temporary file and an atomic rename, and holds
  the optimizer step it belongs to;
* before a directory is (re)written its marker is removed, so a rewrite that dies
  half way is never taken for a complete checkpoint;
* a save whose directory already carries a marker for the same step is skipped
  (the interval save and the final save of a run often coincide);
* retention runs after the new marker is in place and counts complete directories
  only: the newest ``keep_n`` complete ones stay, older complete ones and every
  incomplete directory older than the newest complete one are deleted.

Rank 0 does all file-system work; the other ranks only join the barriers.
"""

from __future__ import annotations

import os
import shutil
from pathlib import Path
from typing import Callable, Optional, Union

import torch.distributed as dist

COMPLETE_MARKER = "COMPLETE"


def _tag_number(name: str) -> Optional[int]:
    head, sep, tail = name.rpartition("_")
    return int(tail) if sep and head and tail.isdigit() else None


def _marker_step(path: Path) -> Optional[int]:
    try:
        text = (path / COMPLETE_MARKER).read_text().strip()
    except OSError:
        return None
    try:
        return int(text)
    except ValueError:
        return -1  # a marker without a readable step still marks a complete directory


def latest_complete_checkpoint(root: Union[str, os.PathLike]) -> Optional[str]:
    """Newest ``<policy>_<n>`` directory under ``root`` that holds a completion marker, or None."""
    root = Path(root)
    if not root.is_dir():
        return None
    numbered = [(n, p) for p in root.iterdir() if p.is_dir() and (n := _tag_number(p.name)) is not None]
    for _, p in sorted(numbered, key=lambda x: x[0], reverse=True):
        if (p / COMPLETE_MARKER).is_file():
            return str(p)
    return None


class CheckpointStore:
    """The ``checkpoints/`` folder of one run."""

    def __init__(self, root: Union[str, os.PathLike], keep_n: int, *, is_writer: bool,
                 barrier: Optional[Callable[[], None]] = None) -> None:
        self.root = Path(root)
        self.keep_n = max(1, int(keep_n))
        self.is_writer = bool(is_writer)
        self._barrier = barrier or (lambda: dist.barrier() if dist.is_available() and dist.is_initialized() else None)

    def directory(self, tag: str) -> Path:
        return self.root / tag

    def is_current(self, tag: str, step: int) -> bool:
        """True when ``tag`` already holds a complete checkpoint of ``step``."""
        return _marker_step(self.directory(tag)) == int(step)

    def begin(self, tag: str) -> Path:
        """Prepare ``tag`` for writing: drop its old marker, create it, wait for every rank."""
        path = self.directory(tag)
        if self.is_writer:
            self.root.mkdir(parents=True, exist_ok=True)
            (path / COMPLETE_MARKER).unlink(missing_ok=True)
            path.mkdir(parents=True, exist_ok=True)
        self._barrier()
        return path

    def commit(self, tag: str, step: int) -> None:
        """Mark ``tag`` complete (after every rank finished writing), then apply retention."""
        self._barrier()
        if self.is_writer:
            path = self.directory(tag)
            tmp = path / f".{COMPLETE_MARKER}.tmp"
            tmp.write_text(str(int(step)))
            os.replace(tmp, path / COMPLETE_MARKER)
            self.prune(protect=path)
        self._barrier()

    def prune(self, protect: Optional[Path] = None) -> list[str]:
        """Apply the retention rule; returns the names removed (writer rank only)."""
        if not self.is_writer or not self.root.is_dir():
            return []
        numbered = sorted(((n, p) for p in self.root.iterdir() if p.is_dir()
                           and (n := _tag_number(p.name)) is not None), key=lambda x: x[0])
        complete = [(n, p) for n, p in numbered if (p / COMPLETE_MARKER).is_file()]
        keep = {p for _, p in complete[-self.keep_n:]}
        if protect is not None:
            keep.add(protect)
        newest_complete = complete[-1][0] if complete else None
        removed = []
        for n, p in numbered:
            if p in keep:
                continue
            stale_partial = newest_complete is not None and n < newest_complete
            if (p / COMPLETE_MARKER).is_file() or stale_partial:
                shutil.rmtree(p, ignore_errors=True)
                removed.append(p.name)
        return removed
