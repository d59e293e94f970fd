from typing import Generic, TypeVar

I = TypeVar("I")
O = TypeVar("O")


class Assembler(Generic[I, O]):
    pass


class RuntimeContext:
    @classmethod
    def from_runtime(cls, *a, **k):
        return cls()
