"""Loader of the reference's repacked routed experts (`.gturbo` directory:
packed_experts/layout.json + packed_experts/layer_XX.bin) into HBM-resident
expert pools, the replacement for the reference's SSD expert streaming
(PackedExpertsLayoutReader.load,
Sources/TurboFieldfare/Infrastructure/ModelIO/PackedExpertsLayout.swift:54-143;
the blob order written by RepackPlanner,
Sources/TurboFieldfareRepack/Core/Planning/RepackPlanner.swift:370-445).

layout.json: {"expertStride", "numLayers", "expertsPerLayer", "layers": [{"layer",
"file", "experts": [{"expert", "physicalRank", "offset", "size", "tensors":
{role: {"offset", "size", "dtype", "shape", "bits"?}}}]}]} with the nine roles
gate, gate_scales, gate_biases, up, ..., down_biases; sub-tensor offsets are
relative to the expert's blob.

The pool is laid out in logical expert order (expert e at pool + e*stride,
whatever the physical order of the file) with the nine sub-tensors at the
offsets the kernels need.  When every sub-tensor of the file already starts on
a 16-byte boundary (the reference's own layout for the Gemma 4 shapes) the
blobs are copied unchanged; otherwise each sub-tensor is moved to a 16-byte
aligned offset (edgeexpert_b200.format.expert_layout), so the TMA paths can
read it.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROLES = ("gate", "gate_scales", "gate_biases", "up", "up_scales", "up_biases", "down", "down_scales", "down_biases")
OFFSET_FIELDS = ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b")
MAX_LAYOUT_BYTES = 16 * 1024 * 1024  # the reference's metadata cap (PackedExpertsLayout.swift:53)


class LayoutError(ValueError):
    """layout.json rejected (the reference's ModelError.indexCorrupt / missingFile)."""


@dataclass
class ExpertEntry:
    expert: int
    physical_rank: int
    offset: int
    size: int
    tensors: dict  # role -> {"offset", "size", "dtype", "shape", "bits"?}


@dataclass
class PackedLayout:
    expert_stride: int
    num_layers: int
    experts_per_layer: int
    files: list      # per layer: file name
    experts: list    # per layer: list of ExpertEntry in logical order


def read_layout(directory) -> PackedLayout:
    """Parse and validate packed_experts/layout.json with the reference's checks."""
    path = Path(directory) / "packed_experts" / "layout.json"
    if not path.exists():
        raise LayoutError("missing file packed_experts/layout.json")
    if path.stat().st_size > MAX_LAYOUT_BYTES:
        raise LayoutError(f"layout.json size {path.stat().st_size} exceeds metadata cap {MAX_LAYOUT_BYTES}")
    try:
        root = json.loads(path.read_text())
    except json.JSONDecodeError as exc:
        raise LayoutError(f"layout.json: {exc}") from exc
    try:
        stride = int(root["expertStride"])
        num_layers = int(root["numLayers"])
        per_layer = int(root["expertsPerLayer"])
        layers = root["layers"]
    except (KeyError, TypeError, ValueError) as exc:
        raise LayoutError("layout.json: missing top-level keys") from exc
    files, experts = [], []
    for lobj in layers:
        if not isinstance(lobj, dict) or not {"layer", "file", "experts"} <= lobj.keys():
            raise LayoutError("layout.json: malformed layer entry")
        slots: list = [None] * per_layer
        for n, eobj in enumerate(lobj["experts"]):
            if not isinstance(eobj, dict) or not {"offset", "size", "tensors"} <= eobj.keys():
                raise LayoutError("layout.json: malformed expert entry")
            tensors = {}
            for role, t in eobj["tensors"].items():
                if not isinstance(t, dict) or not {"offset", "size", "dtype", "shape"} <= t.keys():
                    raise LayoutError(f"layout.json: malformed tensor {role}")
                if "bits" in t and not isinstance(t["bits"], int):
                    raise LayoutError(f"layout.json: malformed tensor bits {role}")
                tensors[role] = t
            eid = int(eobj.get("expert", sum(s is not None for s in slots)))
            if not 0 <= eid < per_layer:
                raise LayoutError("layout.json: expert id out of range")
            rank = int(eobj.get("physicalRank", eid))
            if not 0 <= rank < per_layer:
                raise LayoutError("layout.json: physicalRank out of range")
            slots[eid] = ExpertEntry(eid, rank, int(eobj["offset"]), int(eobj["size"]), tensors)
        if any(s is None for s in slots):
            raise LayoutError("layout.json: missing expert entries")
        files.append(lobj["file"])
        experts.append(slots)
    return PackedLayout(stride, num_layers, per_layer, files, experts)


def _shape_of(entry: ExpertEntry) -> tuple[int, int, int]:
    """(d, f, bits) from the gate and down weight tensors' logical shapes."""
    g = entry.tensors["gate"]
    dn = entry.tensors["down"]
    f, d = int(g["shape"][-2]), int(g["shape"][-1])
    if [int(v) for v in dn["shape"][-2:]] != [d, f]:
        raise LayoutError("layout.json: gate and down shapes disagree")
    return d, f, int(g.get("bits", 4))


def load_layer_host(directory, layer: int, layout: PackedLayout | None = None):
    """One layer's experts as a host byte pool in logical order:
    (pool uint8 [E * stride], stride, tf_expert_offsets, d, f, scale dtype name).
    2/3/4-bit routed experts (the rebits output keeps the same layout with
    smaller weight tensors); `bits` is the gate tensor's "bits" field."""
    from .format import expert_layout
    layout = layout or read_layout(directory)
    entries = layout.experts[layer]
    for role in ROLES:
        if role not in entries[0].tensors:
            raise LayoutError(f"layout.json: expert tensor {role} missing")
    d, f, bits = _shape_of(entries[0])
    if bits not in (2, 3, 4):
        raise LayoutError(f"layout.json: {bits}-bit routed experts are not supported by this loader")
    sdtype = entries[0].tensors["gate_scales"]["dtype"].lower()
    data = np.fromfile(Path(directory) / "packed_experts" / layout.files[layer], dtype=np.uint8)
    E = layout.experts_per_layer
    src_off = [int(entries[0].tensors[r]["offset"]) for r in ROLES]
    aligned = all(o % 16 == 0 for o in src_off) and layout.expert_stride % 16 == 0
    for e in entries:
        if [int(e.tensors[r]["offset"]) for r in ROLES] != src_off:
            raise LayoutError("layout.json: sub-tensor offsets differ between experts")
        if e.offset + layout.expert_stride > data.size:
            raise LayoutError(f"{layout.files[layer]}: expert {e.expert} beyond the end of the file")
    from ._lib import ExpertOffsets
    if aligned:
        stride = layout.expert_stride
        pool = np.empty(E * stride, np.uint8)
        for e in entries:
            pool[e.expert * stride:(e.expert + 1) * stride] = data[e.offset:e.offset + stride]
        offsets = ExpertOffsets(*src_off)
    else:  # 16-byte realignment of every sub-tensor
        lay = expert_layout(d, f, bits=bits)
        stride = lay.stride
        pool = np.zeros(E * stride, np.uint8)
        dst_off = [getattr(lay.offsets, n) for n in OFFSET_FIELDS]
        for e in entries:
            base = e.expert * stride
            for r, so, do in zip(ROLES, src_off, dst_off):
                n = int(e.tensors[r]["size"])
                pool[base + do:base + do + n] = data[e.offset + so:e.offset + so + n]
        offsets = lay.offsets
    return pool, stride, offsets, d, f, sdtype


def load_layer_pool(directory, layer: int, device, layout: PackedLayout | None = None):
    """One layer's routed experts as an HBM-resident ExpertPool."""
    import torch

    from .moe import ExpertPool
    layout = layout or read_layout(directory)
    pool, stride, offsets, d, f, sdtype = load_layer_host(directory, layer, layout)
    bits = _shape_of(layout.experts[layer][0])[2]
    blob = torch.from_numpy(pool).to(device)
    sd = torch.float16 if sdtype in ("f16", "fp16", "float16") else torch.bfloat16
    return ExpertPool(blob, stride, len(pool) // stride, offsets, d, f, sd, bits)
