"""Host-side fault injection for failure-detection tests.

Every failure is made on the host: a rank that exits without warning, a store key
that is deleted or never written, a damaged checkpoint file, a device status word
that a bounded wait would have set.  Nothing here faults, traps or hangs a GPU;
device-side waits are exercised by withholding the flag they wait for (see the
peer-collective tests), which the kernels turn into a status code.
"""

from __future__ import annotations

import os
from pathlib import Path
from typing import Union


def exit_abruptly(code: int = 17) -> None:
    """Leave the process immediately (no atexit handlers, no process-group teardown), like a crash."""
    os._exit(code)


def drop_store_key(store, key: str) -> bool:
    """Delete ``key`` from a c10d store; returns whether it existed."""
    return bool(store.delete_key(key))


def corrupt_file(path: Union[str, os.PathLike], *, keep_bytes: int = 16) -> None:
    """Truncate a file to its first ``keep_bytes`` bytes (a torn write)."""
    p = Path(path)
    data = p.read_bytes()[:keep_bytes]
    p.write_bytes(data)


def remove_completion_marker(ckpt_dir: Union[str, os.PathLike]) -> None:
    """Make a checkpoint look interrupted mid-save."""
    from ..engine.engine import COMPLETE_MARKER

    m = Path(ckpt_dir) / COMPLETE_MARKER
    if m.exists():
        m.unlink()


def set_status_word(code: int, device=None) -> None:
    """Write a bounded-wait status code into the device status word (as a timed-out kernel would)."""
    from ..ops import _ext

    _ext.status_buffer(device).fill_(int(code))
