"""Extracts the reference's own golden vectors for the fwd+VJP path into
tests/golden/reference_goldens.json.

Sources (read as text from a checkout of the reference, default
/root/reference):
  * sheaf/tests/vag_tests.yaml           - value-and-grad goldens
  * sheaf/tests/interpreter_tests.yaml   - gelu / softmax / log-softmax / tanh forward goldens
  * sheaf/src/core/prng.rs               - Random123 Threefry2x32-20 known answers (tests module)

Run:  python tests/golden/make_reference_goldens.py [REFERENCE_ROOT]
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path

import yaml

HERE = Path(__file__).resolve().parent

VAG_NAMES = [
    "vag-add", "vag-sub", "vag-neg", "vag-mul", "vag-div", "vag-pow", "vag-exp", "vag-log", "vag-sqrt", "vag-abs",
    "vag-tanh", "vag-relu", "vag-sigmoid", "vag-gelu", "vag-softmax", "vag-log-softmax", "vag-sum", "vag-mean",
    "vag-maximum", "vag-matmul", "vag-einsum", "vag-slice", "vag-slice-axis", "vag-ce-slice", "vag-get-embedding",
    "vag-get-embedding-repeated", "vag-shared-embedding-head", "vag-where", "vag-cross-entropy-loss",
    "vag-let-lambda", "vag-dict-capture", "vag-defn-calling-defn", "vag-matmul-batched-transpose",
]
FWD_NAMES = {"tanh", "gelu", "softmax", "log-softmax"}


def main(root: Path) -> None:
    tests = root / "sheaf" / "tests"
    vag = yaml.safe_load((tests / "vag_tests.yaml").read_text())
    by_name = {c["name"]: c for c in vag}
    out = {"source": "sheaf/tests/vag_tests.yaml, sheaf/tests/interpreter_tests.yaml, sheaf/src/core/prng.rs",
           "vag": {}, "forward": [], "threefry_kat": []}
    for name in VAG_NAMES:
        c = by_name[name]
        out["vag"][name] = {"test": " ".join(c["test"].split()), "expected": c["expected"]}
    interp = yaml.safe_load((tests / "interpreter_tests.yaml").read_text())
    for c in interp:
        if c.get("name") in FWD_NAMES:
            out["forward"].append({"name": c["name"], "test": c["test"], "expected": c["expected"]})
    prng_src = (root / "sheaf" / "src" / "core" / "prng.rs").read_text()
    kat_block = prng_src[prng_src.index("fn random123_known_answers"):]
    kat_block = kat_block[:kat_block.index("}\n")]
    hexnum = r"(0x[0-9a-fA-F]+|0|u32::MAX)"
    pat = re.compile(r"\(\[(.*?)\],\s*\[(.*?)\],\s*\[(.*?)\]\)")
    for m in pat.finditer(kat_block):
        def parse(s):
            s = s.strip()
            if s == "u32::MAX; 2":
                return [0xFFFFFFFF, 0xFFFFFFFF]
            return [int(v.strip(), 0) for v in s.split(",")]
        out["threefry_kat"].append({"counter": parse(m.group(1)), "key": parse(m.group(2)),
                                    "expected": parse(m.group(3))})
    # the worked StableHLO example printed in docs/key-concepts.md (a module
    # exactly as the emitter produces it, wrapped lines and comments included)
    doc = (root / "docs" / "key-concepts.md").read_text()
    start = doc.index("```mlir", doc.index("produces typed MLIR")) + len("```mlir")
    out["docs_mlir_forward"] = doc[start:doc.index("```", start)].strip("\n") + "\n"
    (HERE / "reference_goldens.json").write_text(json.dumps(out, indent=1) + "\n")
    print(f"wrote {len(out['vag'])} VAG, {len(out['forward'])} forward, {len(out['threefry_kat'])} KAT cases")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path("/root/reference"))
