"""The C-ABI library builds for sm_100a, loads without a GPU, and exports every declared symbol."""
import re
import subprocess

from conftest import ROOT

HEADER = ROOT / "include" / "shardlm_cuda.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(shd_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from shardlm_b200 import _lib, build

    build.build_library()
    names = declared_functions()
    assert len(names) > 10
    out = subprocess.run(["nm", "-D", "--defined-only", str(build.LIB)], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (shd_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    lib = _lib.lib()  # loads without a GPU
    for n in names:
        assert getattr(lib, n) is not None
    # the ctypes table covers exactly the declared entry points
    assert sorted(_lib.SIGNATURES) == names


def test_build_targets_sm100a_only():
    from shardlm_b200 import build

    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_init_fails_loudly_without_gpu():
    import ctypes

    import torch

    from shardlm_b200 import _lib

    if torch.cuda.is_available():
        return
    h = ctypes.c_void_p()
    rc = _lib.lib().shd_init(0, ctypes.byref(h))
    assert rc != 0 and not h.value
