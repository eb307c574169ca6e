"""The packed-experts loader (edgeexpert_b200.gturbo) on CPU: a directory in
the reference's repacked layout (packed_experts/layout.json + layer files,
PackedExpertsLayout.swift:54-143; blob order of RepackPlanner.swift:370-445)
with experts stored in a permuted physical order is read back into a pool in
logical order, byte for byte; sub-tensors off a 16-byte boundary are
realigned; malformed layouts raise the reference's errors."""
import json

import numpy as np
import pytest

import oracle as O

D, F, E = 128, 64, 6


def make_experts(seed=0, d=D, f=F, n=E):
    """n experts as dicts role -> bytes (weights, then BF16 scales / biases)."""
    rng = O.seed_tree(seed, "gturbo")
    out = []
    for _ in range(n):
        ex = {}
        for proj, rows, cols in (("gate", f, d), ("up", f, d), ("down", d, f)):
            W, S, B = rng.synthetic_affine(rows, cols, 4, 0)
            ex[proj] = (np.ascontiguousarray(W).view(np.uint8).reshape(-1), [rows, cols])
            ex[proj + "_scales"] = (np.ascontiguousarray(S).view(np.uint8).reshape(-1), [rows, cols // 64])
            ex[proj + "_biases"] = (np.ascontiguousarray(B).view(np.uint8).reshape(-1), [rows, cols // 64])
        out.append(ex)
    return out


def write_packed(directory, layers, gap=0, order=None, page=16384):
    """The repacker's on-disk layout; `gap` bytes between sub-tensors make
    them 2-byte aligned only; `order` is the physical order of the experts."""
    from edgeexpert_b200.gturbo import ROLES
    pdir = directory / "packed_experts"
    pdir.mkdir(parents=True, exist_ok=True)
    ex0 = layers[0][0]
    offs, cur = {}, 0
    for r in ROLES:
        offs[r] = cur
        cur += ex0[r][0].size + gap
    stride = (cur + page - 1) // page * page
    meta = {"expertStride": stride, "numLayers": len(layers), "expertsPerLayer": len(layers[0]), "layers": []}
    for li, experts in enumerate(layers):
        n = len(experts)
        order_l = order or list(range(n))
        data = np.zeros(n * stride, np.uint8)
        entries = []
        for rank, e in enumerate(order_l):
            base = rank * stride
            tensors = {}
            for r in ROLES:
                b, shape = experts[e][r]
                data[base + offs[r]:base + offs[r] + b.size] = b
                t = {"offset": offs[r], "size": int(b.size), "dtype": "u32" if r in ("gate", "up", "down") else "bf16",
                     "shape": shape}
                if r in ("gate", "up", "down"):
                    t["bits"] = 4
                tensors[r] = t
            entries.append({"expert": e, "physicalRank": rank, "offset": base, "size": stride, "tensors": tensors})
        fname = f"layer_{li:02d}.bin"
        data.tofile(pdir / fname)
        meta["layers"].append({"layer": li, "file": fname, "experts": entries})
    (pdir / "layout.json").write_text(json.dumps(meta))
    return stride


@pytest.mark.parametrize("gap", [0, 2])
def test_loader_restores_logical_order_and_alignment(tmp_path, gap):
    from edgeexpert_b200.gturbo import OFFSET_FIELDS, ROLES, load_layer_host, read_layout
    layers = [make_experts(1), make_experts(2)]
    order = [3, 0, 5, 1, 4, 2]
    write_packed(tmp_path, layers, gap=gap, order=order)
    lay = read_layout(tmp_path)
    assert lay.num_layers == 2 and lay.experts_per_layer == E
    for li in range(2):
        pool, stride, offsets, d, f, sdt = load_layer_host(tmp_path, li, lay)
        assert (d, f, sdt) == (D, F, "bf16")
        for name in OFFSET_FIELDS:
            assert getattr(offsets, name) % 16 == 0
        for e in range(E):
            for r, name in zip(ROLES, OFFSET_FIELDS):
                b = layers[li][e][r][0]
                o = e * stride + getattr(offsets, name)
                assert np.array_equal(pool[o:o + b.size], b), (li, e, r)
        if gap == 0:  # already aligned: the file's own offsets are kept
            assert offsets.gate_s == layers[0][0]["gate"][0].size


def test_loader_rejects_malformed_layouts(tmp_path):
    from edgeexpert_b200.gturbo import LayoutError, read_layout
    with pytest.raises(LayoutError, match="missing file"):
        read_layout(tmp_path)
    write_packed(tmp_path, [make_experts(3)])
    path = tmp_path / "packed_experts" / "layout.json"
    good = json.loads(path.read_text())

    def check(mutate, msg):
        bad = json.loads(json.dumps(good))
        mutate(bad)
        path.write_text(json.dumps(bad))
        with pytest.raises(LayoutError, match=msg):
            read_layout(tmp_path)

    check(lambda m: m.pop("expertStride"), "missing top-level keys")
    check(lambda m: m["layers"][0].pop("file"), "malformed layer entry")
    check(lambda m: m["layers"][0]["experts"][0].update(expert=E), "expert id out of range")
    check(lambda m: m["layers"][0]["experts"][0].update(physicalRank=-1), "physicalRank out of range")
    check(lambda m: m["layers"][0]["experts"].pop(), "missing expert entries")
    check(lambda m: m["layers"][0]["experts"][0]["tensors"]["gate"].update(bits="4"), "malformed tensor bits")
    path.write_text("{not json")
    with pytest.raises(LayoutError):
        read_layout(tmp_path)
