"""Named auxiliary-target bundles (schema + values).

Same role as avgen/core/tensors.py:79-333: a batch can carry extra supervised
targets (depth, flow, ...) described by a hashable spec of names, semantics,
shapes and portable dtype names.
"""
from __future__ import annotations

from enum import Enum

import torch
from torch.utils import _pytree

from avgen_b200.core._validate import require_name, require_unique_names

__all__ = ["TensorBundle", "TensorBundleSpec", "TensorDType"]


class TensorDType(str, Enum):
    BOOL = "bool"
    INT32 = "int32"
    INT64 = "int64"
    BF16 = "bf16"
    FP16 = "fp16"
    FP32 = "fp32"

    @property
    def torch_dtype(self) -> torch.dtype:
        return _DTYPES[self]

    @classmethod
    def from_torch(cls, dtype: torch.dtype) -> TensorDType:
        for key, value in _DTYPES.items():
            if value is dtype:
                return key
        raise KeyError(f"dtype {dtype} has no portable name")


_DTYPES = {
    TensorDType.BOOL: torch.bool,
    TensorDType.INT32: torch.int32,
    TensorDType.INT64: torch.int64,
    TensorDType.BF16: torch.bfloat16,
    TensorDType.FP16: torch.float16,
    TensorDType.FP32: torch.float32,
}


class TensorBundleSpec:
    """Immutable schema of a tensor bundle."""

    __slots__ = ("dtypes", "names", "semantics", "shapes")

    def __init__(self, names: tuple[str, ...] = (), semantics: tuple[str, ...] = (),
                 shapes: tuple[tuple[int, ...], ...] = (), dtypes: tuple[TensorDType, ...] = ()) -> None:
        if len({len(names), len(semantics), len(shapes), len(dtypes)}) != 1:
            raise ValueError("tensor bundle spec fields must have equal lengths")
        require_unique_names("names", names)
        for i, sem in enumerate(semantics):
            require_name(f"semantics[{i}]", sem)
        for shape in shapes:
            if any(isinstance(d, bool) or d < 0 for d in shape):
                raise ValueError(f"bundle shapes must be non-negative; got {shape}")
        self.names = tuple(names)
        self.semantics = tuple(semantics)
        self.shapes = tuple(tuple(s) for s in shapes)
        self.dtypes = tuple(TensorDType(d) for d in dtypes)

    def __len__(self) -> int:
        return len(self.names)

    def _key(self) -> tuple:
        return (self.names, self.semantics, self.shapes, self.dtypes)

    def __eq__(self, other: object) -> bool:
        return isinstance(other, TensorBundleSpec) and self._key() == other._key()

    def __hash__(self) -> int:
        return hash(self._key())

    def __repr__(self) -> str:
        return "TensorBundleSpec(" + ", ".join(f"{n}:{d.value}{list(s)}" for n, d, s in
                                             zip(self.names, self.dtypes, self.shapes)) + ")"

    def index_of(self, name: str) -> int:
        try:
            return self.names.index(name)
        except ValueError:
            raise KeyError(f"unknown bundle field {name!r}; available: {', '.join(self.names) or '(none)'}") from None

    def with_batch_size(self, batch: int) -> TensorBundleSpec:
        return TensorBundleSpec(self.names, self.semantics, tuple((batch, *s[1:]) for s in self.shapes), self.dtypes)

    def to_dict(self) -> dict[str, object]:
        return {"names": list(self.names), "semantics": list(self.semantics),
                "shapes": [list(s) for s in self.shapes], "dtypes": [d.value for d in self.dtypes]}

    @classmethod
    def from_dict(cls, values: dict) -> TensorBundleSpec:
        return cls(tuple(values["names"]), tuple(values["semantics"]), tuple(tuple(s) for s in values["shapes"]),
                   tuple(TensorDType(v) for v in values["dtypes"]))


class TensorBundle:
    """Ordered tensors matching a :class:`TensorBundleSpec`."""

    __slots__ = ("values",)

    def __init__(self, values: tuple[torch.Tensor, ...] = ()) -> None:
        self.values = tuple(values)

    def __len__(self) -> int:
        return len(self.values)

    def __repr__(self) -> str:
        return f"TensorBundle({len(self.values)} tensors)"

    def get(self, spec: TensorBundleSpec, name: str) -> torch.Tensor:
        return self.values[spec.index_of(name)]

    def validate(self, spec: TensorBundleSpec, *, device: torch.device | None = None) -> None:
        if len(self.values) != len(spec):
            raise ValueError(f"bundle has {len(self.values)} values for {len(spec)} fields")
        for value, name, shape, dtype in zip(self.values, spec.names, spec.shapes, spec.dtypes):
            if tuple(value.shape) != shape:
                raise ValueError(f"target {name!r} shape must be {shape}; got {tuple(value.shape)}")
            if value.dtype is not dtype.torch_dtype:
                raise TypeError(f"target {name!r} dtype must be {dtype.torch_dtype}; got {value.dtype}")
            if device is not None and value.device != device:
                raise ValueError(f"target {name!r} must be on {device}")


_pytree.register_pytree_node(TensorBundle, lambda b: (list(b.values), None),
                             lambda v, _c: TensorBundle(tuple(v)), serialized_type_name="avgen_b200.TensorBundle")
