"""CPU checks of the drop-in boundary: the C-ABI library loads, exports every symbol include/larder_b200.h declares,
and the Python layer refuses CPU tensors and bad shapes loudly (no CPU fallback exists). No compute call runs."""
import ctypes
import os
import re

import pytest
import torch

from larder_b200 import _lib, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "larder_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lb2_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_symbols()
    assert names, "no declarations parsed"
    for n in names:
        assert hasattr(L, n), f"{n} declared in include/larder_b200.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of step with the header"


def declarations():
    """{name: (return type, [parameter types])} of every entry point in include/larder_b200.h."""
    text = open(os.path.join(ROOT, "include", "larder_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"^\s*#[^\n]*", "", text, flags=re.M)  # preprocessor lines
    out = {}
    for ret, name, params in re.findall(r"([A-Za-z_][\w\s\*]*?)\s*\b(lb2_\w+)\s*\(([^)]*)\)\s*;", text):
        types = []
        for prm in [x.strip() for x in params.split(",") if x.strip() and x.strip() != "void"]:
            prm = re.sub(r"\s*\*\s*", "* ", prm)
            types.append(" ".join(prm.replace("*", " * ").split()[:-1]).replace(" *", "*"))
        out[name] = (" ".join(ret.split()), types)
    return out


def ctype_of(c_type):
    """The ctypes type a C parameter or return type binds as."""
    t = c_type.replace("const ", "").strip()
    if t.count("*") == 2:
        return ctypes.POINTER(ctypes.c_void_p)
    if t == "int64_t*":
        return _lib._i64p
    if t == "char*":
        return ctypes.c_char_p
    if t.endswith("*"):
        return ctypes.c_void_p
    return {"int": ctypes.c_int, "float": ctypes.c_float, "size_t": ctypes.c_size_t, "int64_t": ctypes.c_int64,
            "uint32_t": ctypes.c_uint32}[t]


def test_ctypes_signatures_match_the_header():
    """Each binding's argument list is the declaration's, type by type: a wrong count or width would pass every CPU
    check and corrupt the call's arguments on a GPU."""
    decl = declarations()
    assert set(decl) == set(declared_symbols())
    assert set(_lib.SIGNATURES) == set(decl), set(_lib.SIGNATURES) ^ set(decl)
    for name, (ret, params) in decl.items():
        args, res = _lib.SIGNATURES[name]
        want = [ctype_of(p) for p in params]
        assert len(args) == len(want), f"{name}: {len(args)} ctypes arguments, {len(want)} declared"
        for i, (a, w) in enumerate(zip(args, want)):
            assert a == w, f"{name} argument {i}: ctypes {a.__name__}, declared {params[i]}"
        assert res == ctype_of(ret), f"{name}: returns {ret}"


def test_abi_version_and_error_slot():
    L = _lib.lib()
    assert L.lb2_abi_version() == 1
    assert isinstance(L.lb2_error(), bytes)


def test_workspace_size_queries_need_no_gpu():
    L = _lib.lib()
    assert L.lb2_attn_decode_workspace_size(16, 32, 4, 1, 8192, 128, 512) > 0
    assert L.lb2_attn_decode_workspace_size(0, 32, 4, 1, 8192, 128, 512) == 0


def test_cpu_tensors_are_refused():
    q = torch.zeros(1, 8, 1, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 64, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.attn_decode(q, k, k, 0.1)
    with pytest.raises(ValueError, match="CUDA"):
        ops.attn_prefill(q, k, k, 0.1, "causal")
    with pytest.raises(ValueError, match="CUDA"):
        ops.gdn_recurrent(torch.zeros(1, 1, 1, 128), torch.zeros(1, 1, 1, 128), torch.zeros(1, 1, 1, 128),
                          torch.ones(1, 1, 1), torch.ones(1, 1, 1))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "nope.so"))
    with pytest.raises(ImportError, match="no CPU or PyTorch fallback"):
        _lib.lib()
