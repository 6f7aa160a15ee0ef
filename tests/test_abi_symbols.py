"""The C-ABI library loads and exports every entry point include/*.h declares.

CPU only: loads the shared library (no device call) and compares its dynamic
symbol table with the declarations in the public headers, and with the ctypes
signature table of the Python binding.
"""

import ctypes
import glob
import os
import re
import subprocess

import private_genomic_dnagpt_b200 as eng
from private_genomic_dnagpt_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(ckks_\w+)\s*\(", re.M)


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        with open(h) as f:
            text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
        names |= set(DECL.findall(text))
    return names


def test_header_declares_the_boundary():
    names = declared()
    for must in ("ckks_ctx_create", "ckks_keygen", "ckks_rotkey_gen", "ckks_encode", "ckks_encrypt",
                 "ckks_decrypt", "ckks_add", "ckks_mul_pt", "ckks_mul_ct", "ckks_rescale", "ckks_rotate",
                 "ckks_rotate_hoisted", "ckks_accumulate_sum", "ckks_ct_export", "ckks_ct_import"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = build()
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    handle = ctypes.CDLL(lib)
    for name in declared():
        assert hasattr(handle, name)


def test_python_binding_covers_the_header():
    assert declared() == set(eng.exported_symbols())
