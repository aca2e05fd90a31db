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


def test_new_ops_refuse_cpu_tensors():
    """The fused projections, the RoPE table and the tree-mask attention have no CPU path either."""
    import pytest
    import torch

    from orthrus_training_b200 import ops

    x = torch.zeros(128, 64, dtype=torch.bfloat16)
    w = torch.zeros(256, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.linear(x, w)
    with pytest.raises(ValueError):
        ops.linear(x, w, residual=torch.zeros(128, 256, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.linear_swiglu(x, w)
    with pytest.raises(ValueError):
        ops.linear_swiglu(x, w, keep_gate_up=True)
    with pytest.raises(ValueError):
        ops.rope_table(torch.ones(64), 16)
    n = torch.ones(128, dtype=torch.bfloat16)
    rope = (torch.zeros(128, 64, dtype=torch.bfloat16), torch.zeros(128, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        ops.linear_qkv_rope(x, torch.zeros(4 * 128, 64, dtype=torch.bfloat16), n, n, rope, 1, 128, 2, 1, 1e-6)
    q = torch.zeros(1, 2, 4, 64, dtype=torch.bfloat16)
    k = torch.zeros(1, 1, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.attention_fwd(q, k, k, k, k, mask=3, hd=64, scale=0.125,
                          offset=torch.zeros(1, dtype=torch.int32), limit2=torch.ones(4, dtype=torch.int32))


def test_fused_shape_predicates():
    import torch

    from orthrus_training_b200 import ops

    x = torch.zeros(8, 1024, dtype=torch.bfloat16)
    assert ops.fused_linear_supported(x, torch.zeros(4096, 1024, dtype=torch.bfloat16), 4096)
    assert not ops.fused_linear_supported(x, torch.zeros(4000, 1024, dtype=torch.bfloat16), 4000)
    assert not ops.fused_linear_supported(x.float(), torch.zeros(4096, 1024), 4096)
    assert ops.fused_qkv_rope_supported(x, 128, 128, 2048, 16, 8)
    assert not ops.fused_qkv_rope_supported(x, 64, 64, 2048, 16, 8)       # head dim 128 only
    assert not ops.fused_qkv_rope_supported(x, 128, 128, 2000, 16, 8)     # whole 128-row tiles
    assert not ops.fused_qkv_rope_supported(x, 128, 128, 2048, 15, 8)     # two heads per tile
