"""Result type of a runtime patch (reference: mvp_engine/patches/types.py:11-17)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

PatchStatus = Literal["applied", "skipped", "failed"]


@dataclass(frozen=True)
class PatchResult:
    """What applying one patch did: ``applied``, ``skipped`` (not needed / not applicable, with the reason)
    or ``failed`` (the reason is the error)."""

    name: str
    status: PatchStatus
    reason: str = ""

    @property
    def applied(self) -> bool:
        return self.status == "applied"
