"""The plugin's discovery hooks (tensorplay-mlu pyproject.toml:42-50): the
`tensorplay.backends` and `tensorplay.distributed.backends` entry points are
declared in pyproject.toml, resolve to callables of this package, and read
back through importlib.metadata from the distribution's metadata."""

from __future__ import annotations

import importlib
import importlib.metadata as md
import os
import tomllib

from conftest import ROOT


def _entry_points():
    with open(os.path.join(ROOT, "pyproject.toml"), "rb") as f:
        return tomllib.load(f)["project"]["entry-points"]


def test_entry_points_are_declared_and_resolve():
    eps = _entry_points()
    assert eps["tensorplay.backends"] == {"b200": "tensorplay_mlu_b200:_autoload"}
    assert eps["tensorplay.distributed.backends"] == {"nccl_b200": "tensorplay_mlu_b200.distributed:register"}
    for group in eps.values():
        for target in group.values():
            module, attr = target.split(":")
            assert callable(getattr(importlib.import_module(module), attr))


def test_entry_points_read_back_through_importlib_metadata(tmp_path):
    # The metadata an install writes (dist-info with entry_points.txt), read
    # by the same importlib.metadata query TensorPlay's plugin discovery makes.
    dist = tmp_path / "tensorplay_mlu_b200-0.2.0.dist-info"
    dist.mkdir()
    (dist / "METADATA").write_text("Metadata-Version: 2.1\nName: tensorplay-mlu-b200\nVersion: 0.2.0\n")
    lines = []
    for group, entries in _entry_points().items():
        lines.append(f"[{group}]")
        lines += [f"{name} = {target}" for name, target in entries.items()]
        lines.append("")
    (dist / "entry_points.txt").write_text("\n".join(lines))
    found = {}
    for d in md.distributions(path=[str(tmp_path)]):
        for ep in d.entry_points:
            found[(ep.group, ep.name)] = ep
    backend = found[("tensorplay.backends", "b200")]
    dist_backend = found[("tensorplay.distributed.backends", "nccl_b200")]
    assert callable(backend.load()) and callable(dist_backend.load())
    assert backend.load() is importlib.import_module("tensorplay_mlu_b200")._autoload
