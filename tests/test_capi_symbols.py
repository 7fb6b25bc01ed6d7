"""The C-ABI library loads without a GPU and exports every symbol that
include/*.h declares (no compute calls)."""
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
DECL = re.compile(r"SB_API\s+[\w\s\*]+?\b(sb_\w+)\s*\(")


def declared_symbols() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(DECL.findall(h.read_text()))
    return names


def test_headers_declare_the_boundary():
    names = declared_symbols()
    for required in ["sb_session_create", "sb_module_load_stablehlo", "sb_call", "sb_buffer_alloc_copy",
                     "sb_buffer_d2h", "sb_buffer_release", "sb_status_free", "sb_op_matmul"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    import sheaf_b200

    lib = sheaf_b200.lib()  # raises if the library was not built
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_the_headers():
    from sheaf_b200 import _lib

    assert set(_lib.SIGNATURES) == declared_symbols()


def test_no_extra_exports():
    so = ROOT / "sheaf_b200" / "lib" / "libsheaf_b200.so"
    if not so.exists():
        pytest.skip("library not built")
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line and line.split()[-1].startswith("sb_")}
    assert exported == declared_symbols()


def test_session_create_without_gpu_fails_cleanly():
    """On a machine without a CUDA device the session constructor returns a
    status instead of crashing."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from sheaf_b200.runtime import SheafB200Error, Session

    with pytest.raises(SheafB200Error):
        Session(0)
