"""CPU tests of the C-ABI library: it loads, and exports every symbol the
public header declares (no compute calls: there is no GPU here)."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"^TF_API\s+[\w\s\*]+?\b(tf_\w+)\s*\(", h.read_text(), flags=re.M))
    return sorted(names)


def test_header_declares_entry_points():
    syms = _declared_symbols()
    for must in ("tf_int4_gemv", "tf_int8_gemv", "tf_router_topk", "tf_moe_phase1", "tf_moe_phase2",
                 "tf_shared_expert", "tf_moe_decode_layer", "tf_context_create"):
        assert must in syms


def test_library_exports_every_declared_symbol():
    from edgeexpert_b200 import _lib
    handle = _lib.lib()
    missing = [s for s in _declared_symbols() if not hasattr(handle, s)]
    assert not missing, f"declared but not exported: {missing}"
    # every symbol the Python binding types must be declared in the header too
    assert set(_lib.exported_symbols()) <= set(_declared_symbols())


def test_status_strings_without_gpu():
    from edgeexpert_b200 import _lib
    assert _lib.status_string(0) == "ok"
    assert _lib.status_string(3) == "unsupported shape"


def test_context_create_reports_no_device_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from edgeexpert_b200 import _lib
    with pytest.raises(_lib.TFError) as ei:
        _lib.Context(0)
    assert ei.value.status in (_lib.TF_ERR_NO_DEVICE, _lib.TF_ERR_CUDA)


def test_expert_layout_matches_reference_blob_sizes():
    from edgeexpert_b200.format import affine_bytes, expert_layout, moe_layer_bytes
    lay = expert_layout(2816, 704)
    # 3,345,408 bytes used per expert (gate+up+down incl. BF16 scales/biases)
    assert lay.used == 3 * affine_bytes(704, 2816) == 3_345_408
    assert lay.stride % 16384 == 0 and lay.stride >= lay.used
    o = lay.offsets
    for name in ("gate_w", "gate_s", "gate_b", "up_w", "up_s", "up_b", "down_w", "down_s", "down_b"):
        assert getattr(o, name) % 16 == 0
    # config-1 algorithmic bytes: 8 routed + shared(2112) + router + activations
    assert moe_layer_bytes() == 8 * 3_345_408 + 10_036_224 + 382_976 + 2 * 2816 + 2 * 128 + 6 * 2816
