"""sheaf_b200: B200-native executor for Sheaf's compiled fwd+VJP tensor programs.

The compute path is the sm_100a kernel library ``lib/libsheaf_b200.so``
(built from ``csrc/`` by :mod:`sheaf_b200.build`) reached through its C ABI
(``include/sheaf_b200*.h``); this package is the Python host mirror of that
ABI.
"""
from ._lib import ELEM_BF16, ELEM_F16, ELEM_F32, ELEM_I32, LibraryMissing, lib

__all__ = ["ELEM_BF16", "ELEM_F16", "ELEM_F32", "ELEM_I32", "LibraryMissing", "lib"]
