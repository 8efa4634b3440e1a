"""The C-ABI library loads without a GPU and exports every symbol of include/vxb.h."""
import os
import re
import subprocess

import vxb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    with open(os.path.join(ROOT, "include", "vxb.h")) as f:
        src = f.read()
    return sorted(set(re.findall(r"^VXB_API\s+[\w\s\*]+?\b(vxb_\w+)\s*\(", src, re.M)))


def test_header_declares_the_binding_signatures():
    names = declared()
    assert len(names) >= 20
    assert set(names) == set(vxb.SIGNATURES), set(names) ^ set(vxb.SIGNATURES)


def test_library_loads_and_exports_every_declared_symbol():
    L = vxb.lib()  # raises if the library is missing
    out = subprocess.run(["nm", "-D", "--defined-only", vxb.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (vxb_\w+)$", out, re.M))
    for name in declared():
        assert name in exported, f"{name} declared in include/vxb.h but not exported"
        assert getattr(L, name) is not None


def test_open_without_gpu_fails_loudly():
    import torch

    if torch.cuda.is_available():
        return
    try:
        vxb.Decoder(0)
    except vxb.VxbError as e:
        assert e.code == vxb.ERR_BACKEND
    else:
        raise AssertionError("opening a context without a GPU must fail")


def test_last_error_is_thread_local_string():
    assert isinstance(vxb.lib().vxb_last_error(), bytes)
