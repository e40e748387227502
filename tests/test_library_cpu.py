"""torch.library registration of the operators (schema and idempotence; no GPU needed)."""

import pytest

torch = pytest.importorskip("torch")

from loraforge_b200.ops.library import register  # noqa: E402


def test_ops_register_once_with_declared_mutations():
    ops = register()
    assert register() is ops
    schemas = {name: str(getattr(torch.ops.loraforge_b200, name).default._schema)
               for name in ("row_shrink", "row_expand", "lora_shrink_expand")}
    assert "Tensor(a2!) output" in schemas["row_shrink"]
    assert "Tensor(a2!) output" in schemas["row_expand"]
    assert "output" in schemas["lora_shrink_expand"] and "workspace" in schemas["lora_shrink_expand"]
    assert schemas["lora_shrink_expand"].endswith("-> ()")
