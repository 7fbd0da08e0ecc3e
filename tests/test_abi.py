"""CPU checks of the C-ABI library: it builds, loads without a GPU and exports
every function include/nyion_attn.h declares (no compute calls here)."""
import ctypes
import os
import subprocess

import nyion_rs_b200.attn as A


def test_library_loads_and_version():
    assert A.lib().nyion_attn_version() == 100


def test_every_declared_symbol_is_exported():
    names = A.declared_symbols()
    assert "nyion_attn_decode_paged_f32" in names and "gpu_attention_device" in names
    L = ctypes.CDLL(A.LIB_PATH)
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    out = subprocess.check_output(["nm", "-D", "--defined-only", A.LIB_PATH], text=True)
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(names) <= exported


def test_workspace_size_host_only():
    L = A.lib()
    a = L.nyion_attn_decode_workspace_size(32, 4, 32, 64)
    b = L.nyion_attn_decode_workspace_size(1, 4, 32, 64)
    assert a > b > 0
    assert L.nyion_attn_decode_workspace_size(0, 4, 32, 64) == 0
    # batches beyond one launch's 512 sequences reuse the same workspace
    assert L.nyion_attn_decode_workspace_size(4096, 4, 32, 64) == L.nyion_attn_decode_workspace_size(512, 4, 32, 64)


def test_no_oracle_in_product_path():
    """The product package must not import, load or name the CPU oracle."""
    pkg = os.path.dirname(A.__file__)
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h")):
                text = open(os.path.join(root, f)).read()
                assert "liboracle" not in text and "import oracle" not in text, f
