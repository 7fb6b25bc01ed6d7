"""Host-side checks of the StableHLO front door (parse + plan, no device):
sb_stablehlo_validate on the module printed in the reference's docs, on
modules in the emitter's text forms (oracle/hlo_emit.py), and rejection of
ops outside the library's surface."""
import json
import re
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


@pytest.mark.parametrize("dt,key,hp", [("bf16", False, {}), ("bf16", True, {}),
                                       ("f32", False, dict(b1=0.8, b2=0.99, eps=1e-6, wd=0.01, max_norm=0.5))])
def test_nanogpt_train_step_module_is_recognised(dt, key, hp):
    """train-step (examples/nanogpt/train.shf:26-33): the state leaves, x, y, lr;
    the AdamW / clip literals are read off the ops that use them."""
    cfg = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
    s = validate_stablehlo(hlo_emit.gpt_train_module(cfg, dt, with_key=key, **hp))
    want = dict(b1=0.9, b2=0.95, eps=1e-8, wd=0.1, max_norm=1.0, **hp) if not hp else hp
    assert "nanoGPT train_step L=2 H=2 D=128 V=65 B=4 T=64" in s, s
    got = dict(re.findall(r"(b1|b2|eps|wd|max_norm)=([0-9.e+-]+)", s))
    for k, v in want.items():
        assert abs(float(got[k]) - v) <= 1e-6 * v, (k, got[k], v)
    assert ("(key leaf)" in s) == key


def test_train_step_with_a_missing_literal_is_not_recognised():
    """Without the weight-decay multiply the hyperparameters cannot all be read:
    the function stays on the generic executor."""
    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=2, seq=64)
    text = hlo_emit.gpt_train_module(cfg, "f32")
    # the weight-decay term wd * p: replace it by p itself
    lines = text.splitlines()
    for i, ln in enumerate(lines):
        m = re.match(r"\s+(%\d+) = stablehlo\.multiply (%\d+), (%arg\d+) : (tensor<[^>]*>)", ln)
        if m:
            lines[i] = f"    {m.group(1)} = stablehlo.add {m.group(3)}, {m.group(3)} : {m.group(4)}"
    s = validate_stablehlo("\n".join(lines) + "\n")
    assert "train_step" in s and "nanoGPT train_step" not in s


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


# The emitter's forms for reverse, dynamic slices and top_k's sort
# (sheaf/src/lowering/stablehlo/indexing_ops.rs:184-343,486-550).
INDEXING = """module @idx {
  func.func @f(%arg0: tensor<4x6xf32>, %arg1: tensor<i32>, %arg2: tensor<i32>, %arg3: tensor<1x2xf32>) -> (tensor<4x6xf32>, tensor<2x3xf32>, tensor<4x6xf32>, tensor<4x6xf32>) {
    %0 = stablehlo.reverse %arg0, dims = [1] : (tensor<4x6xf32>) -> tensor<4x6xf32>
    %1 = "stablehlo.dynamic_slice"(%arg0, %arg1, %arg2) { slice_sizes = array<i64: 2, 3> } : (tensor<4x6xf32>, tensor<i32>, tensor<i32>) -> tensor<2x3xf32>
    %2 = "stablehlo.dynamic_update_slice"(%arg0, %arg3, %arg1, %arg2) : (tensor<4x6xf32>, tensor<1x2xf32>, tensor<i32>, tensor<i32>) -> tensor<4x6xf32>
    %3 = stablehlo.dynamic_update_slice %arg0, %arg3, %arg2, %arg1 : (tensor<4x6xf32>, tensor<1x2xf32>, tensor<i32>, tensor<i32>) -> tensor<4x6xf32>
    return %0, %1, %2, %3 : tensor<4x6xf32>, tensor<2x3xf32>, tensor<4x6xf32>, tensor<4x6xf32>
  }
}
"""


def top_k_module(rows: int, n: int, k: int, direction: str = "GT", key: str = "f32") -> str:
    """top_k as emit_top_k prints it: iota, the two-operand stable sort with a
    comparator region, slices of the first k, indices converted to f32."""
    t = f"tensor<{rows}x{n}x{key}>"
    ti = f"tensor<{rows}x{n}xi32>"
    return f"""module @topk {{
  func.func @top_k(%arg0: {t}) -> (tensor<{rows}x{k}x{key}>, tensor<{rows}x{k}xf32>) {{
    %0 = stablehlo.iota dim = 1 : {ti}
    %1, %2 = "stablehlo.sort"(%arg0, %0) ({{
    ^bb0(%3: tensor<{key}>, %4: tensor<{key}>, %5: tensor<i32>, %6: tensor<i32>):
      %7 = "stablehlo.compare"(%3, %4) {{comparison_direction = #stablehlo<comparison_direction {direction}>}} : (tensor<{key}>, tensor<{key}>) -> tensor<i1>
      "stablehlo.return"(%7) : (tensor<i1>) -> ()
    }}) {{dimension = 1 : i64, is_stable = true}} : ({t}, {ti}) -> ({t}, {ti})
    %8 = stablehlo.slice %1 [0:{rows}, 0:{k}] : ({t}) -> tensor<{rows}x{k}x{key}>
    %9 = stablehlo.slice %2 [0:{rows}, 0:{k}] : ({ti}) -> tensor<{rows}x{k}xi32>
    %10 = stablehlo.convert %9 : (tensor<{rows}x{k}xi32>) -> tensor<{rows}x{k}xf32>
    return %8, %10 : tensor<{rows}x{k}x{key}>, tensor<{rows}x{k}xf32>
  }}
}}
"""


def test_indexing_forms_parse():
    s = validate_stablehlo(INDEXING)
    assert "f: 4 ops, 4 args, 4 results" in s


def test_top_k_sort_parses():
    s = validate_stablehlo(top_k_module(3, 65, 5))
    assert "top_k: 5 ops, 1 args, 2 results" in s
    validate_stablehlo(top_k_module(1, 50304 // 4, 200, "LT", "bf16"))


def test_sort_and_dynamic_slice_rejections():
    bad_cmp = top_k_module(3, 65, 5).replace('"stablehlo.compare"(%3, %4)', '"stablehlo.compare"(%5, %6)')
    too_long = top_k_module(1, (1 << 24) + 8, 5)
    eq = top_k_module(3, 65, 5, "EQ")
    bad_start = INDEXING.replace("%arg1: tensor<i32>", "%arg1: tensor<f32>").replace(
        "tensor<i32>, tensor<i32>) -> tensor<2x3xf32>", "tensor<f32>, tensor<i32>) -> tensor<2x3xf32>")
    for text in (bad_cmp, too_long, eq, bad_start):
        with pytest.raises(SheafB200Error):
            validate_stablehlo(text)
