"""The C-ABI library loads without a GPU and exports every function include/*.h declares."""
import ctypes as C
import glob
import os
import re

from conftest import ROOT
from nitrorag_b200 import _lib


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(nr_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"nr_engine_create", "nr_step", "nr_forward_prefill", "nr_forward_decode",
            "nr_paged_attention_decode", "nr_q8_matmul"} <= names


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(_lib.LIB_PATH)
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_library_is_built_for_sm100a():
    # the cubin's target is recorded in the ELF notes of the fat binary; cuobjdump is
    # not used on purpose: only the build flags are checked
    from nitrorag_b200 import build
    assert "arch=compute_100a,code=sm_100a" in build.NVCC_FLAGS
