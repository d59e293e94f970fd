"""Name -> object registry used for engines (reference: mvp_engine/utils/registry.py:6-68)."""

from __future__ import annotations

from typing import Any, Callable, Optional, TypeVar

T = TypeVar("T")


class Registry:
    """Map string keys to classes or factories.

    ``@reg.register()`` registers under ``obj.__name__``; ``@reg.register("name")``
    under an explicit key; bare ``@reg.register`` is accepted too.
    """

    def __init__(self, name: str = "registry") -> None:
        self.name = name
        self.mapper: dict[str, Any] = {}

    def register(self, key: Optional[str] | Callable = None) -> Callable[[T], T]:
        if callable(key):
            self.mapper[key.__name__] = key
            return key  # type: ignore[return-value]

        def _add(obj: T) -> T:
            self.mapper[key if key is not None else obj.__name__] = obj  # type: ignore[attr-defined]
            return obj

        return _add

    def get(self, key: str) -> Any:
        try:
            return self.mapper[key]
        except KeyError:
            raise KeyError(f"No object named '{key}' found!") from None

    def __getitem__(self, key: str) -> Any:
        return self.get(key)

    def __contains__(self, key: str) -> bool:
        return key in self.mapper

    def keys(self):
        return self.mapper.keys()
