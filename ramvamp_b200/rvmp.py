"""Reading an .rvmp install's expert files into the HBM expert table.

The reference streams experts from `experts/layer_XX.bin` through
io::ExpertStream; here every layer is loaded once, at start-up.  This
module reads and validates `experts/layout.json` the way
format/layout.rs does (schema v1: per layer one file of `n_experts` blobs of
`stride` bytes, gate/up/down slabs at 4 KiB-aligned offsets), cross-checks
it against `manifest.json` (layer and expert counts, file sizes), turns it
into the table's layer layouts and hands each layer file to the native
loader (`rv_expert_table_load_file`).

Validation errors raise `FormatError` with the reference's variant name in
`kind` (format/error.rs): InvalidLayout, Misaligned, MissingFileEntry,
UnsafeFileName.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from pathlib import PurePosixPath
from typing import Dict, List, Optional, Sequence

EXPERT_BLOB_ALIGN = 4096  # format/mod.rs:73
LAYOUT_FILE = "experts/layout.json"  # format/mod.rs:82
MANIFEST_FILE = "manifest.json"  # format/mod.rs:76
PROJECTIONS = ("gate", "up", "down")  # ProjectionName, format/layout.rs:59-68


class FormatError(ValueError):
    """format/error.rs: `kind` names the variant; Misaligned also carries
    `what`, `name`, `value`, `align`."""

    def __init__(self, kind: str, message: str, **details):
        super().__init__(f"{kind}: {message}")
        self.kind = kind
        for k, v in details.items():
            setattr(self, k, v)


@dataclass
class Projection:
    """format/layout.rs:45-56."""

    name: str
    offset_in_blob: int
    len: int
    quant: str


@dataclass
class LayerEntry:
    """format/layout.rs:31-42."""

    file: str
    stride: int
    n_experts: int
    projections: List[Projection] = field(default_factory=list)


@dataclass
class ExpertsLayout:
    """`experts/layout.json` (format/layout.rs:23-28)."""

    layers: List[LayerEntry]

    def to_json(self) -> dict:
        return {"layers": [{"file": l.file, "stride": l.stride, "n_experts": l.n_experts,
                            "projections": [{"name": p.name, "offset_in_blob": p.offset_in_blob, "len": p.len,
                                             "quant": p.quant} for p in l.projections]} for l in self.layers]}


def _fields(obj, allowed: Sequence[str], what: str) -> dict:
    """serde(deny_unknown_fields): every key known, every key present."""
    if not isinstance(obj, dict):
        raise FormatError("InvalidLayout", f"{what}: expected an object")
    unknown = set(obj) - set(allowed)
    if unknown:
        raise FormatError("InvalidLayout", f"{what}: unknown field(s) {sorted(unknown)}")
    missing = [k for k in allowed if k not in obj]
    if missing:
        raise FormatError("InvalidLayout", f"{what}: missing field(s) {missing}")
    return obj


def _uint(v, what: str) -> int:
    if not isinstance(v, int) or isinstance(v, bool) or v < 0:
        raise FormatError("InvalidLayout", f"{what}: expected an unsigned integer")
    return v


def parse_layout(obj) -> ExpertsLayout:
    """The JSON object of `experts/layout.json` as an ExpertsLayout."""
    top = _fields(obj, ["layers"], "layout")
    if not isinstance(top["layers"], list):
        raise FormatError("InvalidLayout", "layout: layers must be an array")
    layers = []
    for i, lo in enumerate(top["layers"]):
        lo = _fields(lo, ["file", "stride", "n_experts", "projections"], f"layer {i}")
        if not isinstance(lo["file"], str) or not isinstance(lo["projections"], list):
            raise FormatError("InvalidLayout", f"layer {i}: bad field types")
        projs = []
        for j, po in enumerate(lo["projections"]):
            po = _fields(po, ["name", "offset_in_blob", "len", "quant"], f"layer {i} projection {j}")
            if po["name"] not in PROJECTIONS:
                raise FormatError("InvalidLayout", f"layer {i}: unknown projection {po['name']!r}")
            if not isinstance(po["quant"], str):
                raise FormatError("InvalidLayout", f"layer {i}: quant must be a string")
            projs.append(Projection(po["name"], _uint(po["offset_in_blob"], "offset_in_blob"),
                                    _uint(po["len"], "len"), po["quant"]))
        layers.append(LayerEntry(lo["file"], _uint(lo["stride"], "stride"), _uint(lo["n_experts"], "n_experts"),
                                 projs))
    return ExpertsLayout(layers)


def check_file_name(name: str) -> None:
    """format/manifest.rs:315-326: a non-empty relative path made of plain
    components only (no root, no `.` or `..`)."""
    p = PurePosixPath(name)
    safe = bool(name) and not p.is_absolute() and all(c not in ("", ".", "..") for c in name.split("/")) \
        and "\\" not in name
    if not safe:
        raise FormatError("UnsafeFileName", name, name=name)


def validate_layer(layer: LayerEntry, index: int) -> None:
    """format/layout.rs:132-203."""
    check_file_name(layer.file)
    if layer.stride == 0:
        raise FormatError("InvalidLayout", f"layer {index}: stride is zero")
    if layer.stride % EXPERT_BLOB_ALIGN:
        raise FormatError("Misaligned", f"expert blob stride {layer.stride} of {layer.file}", what="expert blob stride",
                          name=layer.file, value=layer.stride, align=EXPERT_BLOB_ALIGN)
    if layer.n_experts == 0:
        raise FormatError("InvalidLayout", f"layer {index}: n_experts is zero")
    if not layer.projections:
        raise FormatError("InvalidLayout", f"layer {index}: no projections")
    seen = set()
    ranges = []
    for p in layer.projections:
        if p.name in seen:
            raise FormatError("InvalidLayout", f"layer {index}: duplicate {p.name} projection")
        seen.add(p.name)
        if p.len == 0 or not p.quant:
            raise FormatError("InvalidLayout", f"layer {index}: {p.name} projection has a zero length or empty quant")
        if p.offset_in_blob % EXPERT_BLOB_ALIGN:
            raise FormatError("Misaligned", f"projection offset {p.offset_in_blob} of layer {index} {p.name}",
                              what="projection offset", name=f"layer {index} {p.name}", value=p.offset_in_blob,
                              align=EXPERT_BLOB_ALIGN)
        end = p.offset_in_blob + p.len
        if end >= 1 << 64:
            raise FormatError("InvalidLayout", f"layer {index}: {p.name} projection offset + len overflows")
        if end > layer.stride:
            raise FormatError("InvalidLayout",
                              f"layer {index}: {p.name} projection ends at byte {end}, past stride {layer.stride}")
        ranges.append((p.offset_in_blob, end))
    ranges.sort()
    for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
        if b0 < a1:
            raise FormatError("InvalidLayout", f"layer {index}: projections overlap")


def validate_layout(layout: ExpertsLayout) -> None:
    """format/layout.rs:71-80."""
    if not layout.layers:
        raise FormatError("InvalidLayout", "no layers")
    for i, layer in enumerate(layout.layers):
        validate_layer(layer, i)


def validate_against(layout: ExpertsLayout, manifest: dict) -> None:
    """format/layout.rs:86-130: layer count, per-layer expert count, unique
    files with a `files` entry of exactly n_experts * stride bytes."""
    validate_layout(layout)
    arch = manifest.get("arch", {})
    files = manifest.get("files", {})
    n_layers = arch.get("n_layers")
    if len(layout.layers) != n_layers:
        raise FormatError("InvalidLayout", f"layout has {len(layout.layers)} layers, arch has {n_layers}")
    seen = set()
    for i, layer in enumerate(layout.layers):
        if layer.n_experts != arch.get("n_experts"):
            raise FormatError("InvalidLayout",
                              f"layer {i}: n_experts {layer.n_experts} does not match arch.n_experts "
                              f"{arch.get('n_experts')}")
        if layer.file in seen:
            raise FormatError("InvalidLayout", f"layer {i}: file {layer.file!r} already used by an earlier layer")
        seen.add(layer.file)
        entry = files.get(layer.file)
        if entry is None:
            raise FormatError("MissingFileEntry", layer.file, name=layer.file)
        expected = layer.stride * layer.n_experts
        if entry.get("size") != expected:
            raise FormatError("InvalidLayout", f"layer {i} ({layer.file!r}): files entry says {entry.get('size')} "
                                               f"bytes, n_experts * stride is {expected}")


def layer_layouts(layout: ExpertsLayout, hidden: int, moe: int) -> list:
    """The expert table's per-layer layouts (`rv_layer_layout`): the three
    projections of every layer, their quant types as QuantFormat."""
    from . import LayerLayout, QuantFormat

    out = []
    for i, layer in enumerate(layout.layers):
        by = {p.name: p for p in layer.projections}
        missing = [n for n in PROJECTIONS if n not in by]
        if missing:
            raise FormatError("InvalidLayout", f"layer {i}: no {missing[0]} projection")
        fmts = []
        for n in PROJECTIONS:
            q = by[n].quant.lower()
            if q not in ("q4_k", "q5_k", "q6_k"):
                raise FormatError("InvalidLayout", f"layer {i}: {n} projection is {by[n].quant}, the GPU expert "
                                                   "path takes q4_k/q5_k/q6_k")
            fmts.append(int(QuantFormat[q.upper()]))
        g, u, d = by["gate"], by["up"], by["down"]
        out.append(LayerLayout(layer.n_experts, 0, layer.stride, g.offset_in_blob, g.len, u.offset_in_blob, u.len,
                               d.offset_in_blob, d.len, fmts[0], fmts[1], fmts[2], hidden, moe))
    return out


def read_install(install_dir: str, check_manifest: bool = True):
    """(layout, manifest) of an install directory, validated."""
    with open(os.path.join(install_dir, LAYOUT_FILE)) as f:
        layout = parse_layout(json.load(f))
    manifest = None
    mpath = os.path.join(install_dir, MANIFEST_FILE)
    if check_manifest:
        with open(mpath) as f:
            manifest = json.load(f)
        validate_against(layout, manifest)
    else:
        validate_layout(layout)
    return layout, manifest


def load_expert_table(install_dir: str, device: int = 0, hidden: Optional[int] = None,
                      moe: Optional[int] = None, layers: Optional[Sequence[int]] = None):
    """An ExpertTable holding the install's experts (all layers, or the
    listed ones in that order), each layer file read by the native loader.
    hidden / moe default to the manifest's arch.hidden / arch.moe_intermediate."""
    from . import ExpertTable

    layout, manifest = read_install(install_dir)
    arch = manifest["arch"]
    hidden = arch["hidden"] if hidden is None else hidden
    moe = arch["moe_intermediate"] if moe is None else moe
    picks = list(range(len(layout.layers))) if layers is None else list(layers)
    lays = layer_layouts(ExpertsLayout([layout.layers[i] for i in picks]), hidden, moe)
    table = ExpertTable(lays, device=device)
    for li, src in enumerate(picks):
        table.load_file(li, os.path.join(install_dir, layout.layers[src].file))
    return table
