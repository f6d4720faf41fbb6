"""Parameter identity and layout metadata.

Same contract as the reference's ``src/zerograd/_manifest.py:17-126``:
ordered, versioned entries; the index of an entry's group is the split index
its perturbation key is drawn from.  Leaves are ``torch.Tensor``.
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, field
from enum import StrEnum
from typing import TypeAlias, Union

import torch

ParameterPath: TypeAlias = tuple[str, ...]
ParameterTree: TypeAlias = Mapping[str, Union["ParameterTree", torch.Tensor]]


class ParameterLayout(StrEnum):
    """Factor algebra of a manifest leaf (``_manifest.py:17-22``)."""

    MATRIX = "matrix"
    TABLE = "table"
    VECTOR = "vector"


LAYOUT_CODE = {ParameterLayout.MATRIX: 0, ParameterLayout.TABLE: 1, ParameterLayout.VECTOR: 2}


@dataclass(frozen=True, slots=True)
class ManifestEntry:
    """One perturbed leaf and its group (``_manifest.py:25-41``)."""

    path: ParameterPath
    layout: ParameterLayout
    group: str

    def __post_init__(self) -> None:
        if not isinstance(self.path, tuple) or not self.path:
            raise ValueError("manifest paths must be non-empty tuples")
        if any(not isinstance(part, str) or not part for part in self.path):
            raise ValueError("manifest path components must be non-empty strings")
        if not isinstance(self.layout, ParameterLayout):
            raise TypeError("manifest layouts must be ParameterLayout values")
        if not isinstance(self.group, str) or not self.group:
            raise ValueError("manifest groups must be non-empty strings")


@dataclass(frozen=True, slots=True)
class Manifest:
    """Versioned ordered manifest (``_manifest.py:44-126``)."""

    version: int
    entries: tuple[ManifestEntry, ...]
    _path_index: dict = field(init=False, repr=False, compare=False, default_factory=dict)
    _group_index: dict = field(init=False, repr=False, compare=False, default_factory=dict)

    def __post_init__(self) -> None:
        if not isinstance(self.version, int) or isinstance(self.version, bool) or self.version < 1:
            raise ValueError(f"manifest version must be a positive integer, got {self.version!r}")
        if not isinstance(self.entries, tuple) or not self.entries:
            raise ValueError("manifest entries must be a non-empty tuple")
        if any(not isinstance(e, ManifestEntry) for e in self.entries):
            raise TypeError("manifest entries must be ManifestEntry instances")
        paths = [e.path for e in self.entries]
        if len(set(paths)) != len(paths):
            raise ValueError("manifest paths must be unique")
        groups = [e.group for e in self.entries]
        if len(set(groups)) != len(groups):
            raise ValueError("manifest groups must be unique; reuse one entry for tied uses")
        object.__setattr__(self, "_path_index", {e.path: e for e in self.entries})
        object.__setattr__(self, "_group_index", {e.group: i for i, e in enumerate(self.entries)})

    def entry(self, path: ParameterPath) -> ManifestEntry:
        try:
            return self._path_index[path]
        except KeyError as error:
            raise KeyError(f"path is not in the manifest: {'.'.join(path)}") from error

    def group_index(self, group: str) -> int:
        try:
            return self._group_index[group]
        except KeyError as error:
            raise KeyError(f"group is not in the manifest: {group}") from error

    def resolve(self, params: ParameterTree, path: ParameterPath) -> torch.Tensor:
        node = params
        for part in path:
            if not isinstance(node, Mapping):
                raise KeyError(f"path traverses an array before {part!r}: {'.'.join(path)}")
            try:
                node = node[part]
            except KeyError as error:
                raise KeyError(f"parameter path is missing: {'.'.join(path)}") from error
        if not isinstance(node, torch.Tensor):
            raise TypeError(f"parameter path does not resolve to a tensor: {'.'.join(path)}")
        return node

    def validate(self, params: ParameterTree) -> None:
        for entry in self.entries:
            parameter = self.resolve(params, entry.path)
            expected = 1 if entry.layout is ParameterLayout.VECTOR else 2
            if parameter.ndim != expected:
                raise ValueError(
                    f"{entry.layout.value} parameter {'.'.join(entry.path)} must be "
                    f"{expected}-D, got shape {tuple(parameter.shape)}")
