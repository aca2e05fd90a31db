"""The C-ABI library builds, loads without a GPU and exports every entry point the header declares
(no compute calls: there is no GPU here)."""

import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _declared() -> set[str]:
    text = (ROOT / "include" / "orthrus_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(orthrus_[a-z0-9_]+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    from orthrus_training_b200 import _lib

    lib = _lib.lib()
    declared = _declared()
    assert len(declared) >= 18
    missing = [s for s in sorted(declared) if not hasattr(lib, s)]
    assert not missing, missing
    assert lib.orthrus_version() >= 100


def test_binding_table_matches_header():
    from orthrus_training_b200 import _lib

    assert set(_lib.exported_symbols()) == _declared()


def test_workspace_queries_are_pure_host_calls():
    from orthrus_training_b200 import _lib

    lib = _lib.lib()
    assert lib.orthrus_attn_bwd_workspace_bytes(8, 16, 1024) == 8 * 16 * 1024 * 4
    assert lib.orthrus_qkv_prep_bwd_workspace_bytes(8, 2048, 128) > 0


def test_ops_refuse_cpu_tensors():
    import pytest
    import torch

    from orthrus_training_b200 import ops

    with pytest.raises(ValueError):
        ops.gemm(torch.zeros(4, 4), torch.zeros(4, 4))
    with pytest.raises(ValueError):
        ops.rms_norm(torch.zeros(2, 8), torch.ones(8), 1e-6)
