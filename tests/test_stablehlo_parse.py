"""Host-side checks of the StableHLO front door (parse + plan, no device):
sb_stablehlo_validate on the module printed in the reference's docs, on
modules in the emitter's text forms (oracle/hlo_emit.py), and rejection of
ops outside the library's surface."""
import json
from pathlib import Path

import pytest

from oracle import hlo_emit, models
from sheaf_b200.runtime import SheafB200Error, validate_stablehlo

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())
UNIMPLEMENTED = 12


def test_docs_module_parses():
    """docs/key-concepts.md:170-184, with wrapped lines and comments."""
    s = validate_stablehlo(GOLD["docs_mlir_forward"])
    assert "forward: 3 ops, 3 args, 1 results" in s


def test_mlp_vag_module_parses():
    s = validate_stablehlo(hlo_emit.mlp_vag_module())
    assert "value_and_grad" in s and "6 args, 5 results" in s


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_nanogpt_vag_module_is_recognised(dt):
    cfg = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
    s = validate_stablehlo(hlo_emit.gpt_vag_module(cfg, dt))
    assert "nanoGPT value_and_grad L=2 H=2 D=128 V=65 B=4 T=64" in s


def test_full_nanogpt_vag_module_plans():
    s = validate_stablehlo(hlo_emit.gpt_vag_module(models.NANOGPT_CHAR, "bf16"))
    assert "L=6 H=6 D=384 V=65 B=64 T=256" in s


def _wrap(body: str, arg="tensor<4xf32>", ret="tensor<4xf32>") -> str:
    return f"module @m {{\n func.func @f(%arg0: {arg}) -> {ret} {{\n{body}\n }}\n}}\n"


def test_unsupported_op_is_unimplemented():
    with pytest.raises(SheafB200Error) as e:
        validate_stablehlo(_wrap("    %0 = stablehlo.cbrt %arg0 : tensor<4xf32>\n    return %0 : tensor<4xf32>"))
    assert e.value.code == UNIMPLEMENTED and "cbrt" in e.value.message


def test_unsupported_types_and_forms():
    for body, arg in [
        ("    return %arg0 : tensor<4xf64>", "tensor<4xf64>"),
        ("    return %arg0 : tensor<?xf32>", "tensor<?xf32>"),
    ]:
        with pytest.raises(SheafB200Error):
            validate_stablehlo(_wrap(body, arg, arg))
    pad = ("    %z = stablehlo.constant dense<0.0> : tensor<f32>\n"
           "    %0 = stablehlo.pad %arg0, %z, low = [0], high = [0], interior = [1] : (tensor<4xf32>, tensor<f32>) -> "
           "tensor<7xf32>\n    return %0 : tensor<7xf32>")
    with pytest.raises(SheafB200Error) as e:
        validate_stablehlo(_wrap(pad, ret="tensor<7xf32>"))
    assert e.value.code == UNIMPLEMENTED


def test_type_errors_are_reported():
    bad = "    %0 = stablehlo.add %arg0, %arg0 : tensor<5xf32>\n    return %0 : tensor<5xf32>"
    with pytest.raises(SheafB200Error):
        validate_stablehlo(_wrap(bad, ret="tensor<5xf32>"))
    undefined = "    %0 = stablehlo.add %arg0, %7 : tensor<4xf32>\n    return %0 : tensor<4xf32>"
    with pytest.raises(SheafB200Error):
        validate_stablehlo(_wrap(undefined))
