"""CPU-side checks of the C ABI: the library loads without a GPU, exports every symbol
include/b200fp8.h declares, the ctypes structs mirror the header, and argument validation
rejects bad calls before any launch (no compute calls happen here)."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "b200fp8.h")


def _lib():
    from b200fp8 import _lib
    return _lib


def _declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2f_[a-z0-9_]+)\s*\(", text)))


def test_header_functions_are_exported():
    lib = _lib().lib()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} missing from libb200fp8.so"
    assert set(declared) == set(_lib().EXPORTED_SYMBOLS)


def test_version_and_registry():
    lib = _lib().lib()
    assert lib.b2f_version() == 1
    n = lib.b2f_registry_size()
    names = [lib.b2f_registry_at(i).contents.name.decode() for i in range(n)]
    assert "gemm_fp8" in names and "norm_quant" in names
    for name in names:
        op = lib.b2f_registry_lookup(name.encode())
        assert op and op.contents.abi_version == 1 and op.contents.fn
    assert not lib.b2f_registry_lookup(b"no_such_op")


def _struct_fields(struct_name):
    text = open(HEADER).read()
    m = re.search(r"typedef struct %s \{(.*?)\} %s;" % (struct_name, struct_name), text, re.S)
    assert m, struct_name
    body = re.sub(r"/\*.*?\*/", "", m.group(1), flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = re.sub(r"\b(const|unsigned)\b", "", decl.strip())
        if not decl:
            continue
        parts = decl.replace("*", " ").split()
        names = " ".join(parts[2:]) if parts[0] == "long" else " ".join(parts[1:])
        fields += [x.strip() for x in names.split(",")]
    return fields


STRUCTS = [("b2f_gemm_args", "GemmArgs"), ("b2f_norm_args", "NormArgs"),
           ("b2f_attn_args", "AttnArgs"), ("b2f_rope_args", "RopeArgs")]


@pytest.mark.parametrize("struct,cls", STRUCTS)
def test_ctypes_structs_mirror_header(struct, cls):
    L = _lib()
    if not hasattr(L, cls):
        pytest.skip(f"{cls} not bound")
    assert [f[0] for f in getattr(L, cls)._fields_] == _struct_fields(struct)


def test_args_init_defaults():
    L = _lib()
    a = L.GemmArgs()
    L.lib().b2f_gemm_args_init(ctypes.byref(a))
    assert a.alpha == 1.0 and a.pre_mul == 1.0 and a.post_mul == 1.0 and a.out_scale == 1.0
    assert a.out_dtype == L.DTYPE_BF16 and a.mode == L.GEMM_STORE and a.tile_n == 0
    nrm = L.NormArgs()
    L.lib().b2f_norm_args_init(ctypes.byref(nrm))
    assert nrm.kind == L.NORM_RMS and abs(nrm.eps - 1e-6) < 1e-12 and nrm.q_scale == 1.0


def test_argument_validation_without_gpu():
    L = _lib()
    lib = L.lib()
    a = L.GemmArgs()
    lib.b2f_gemm_args_init(ctypes.byref(a))
    assert lib.b2f_gemm_fp8(ctypes.byref(a), None) == L.B2F_ERR_ARG  # empty shape
    assert b"empty shape" in lib.b2f_last_error()
    a.m, a.n, a.k = 128, 128, 100
    a.a = a.b = a.out = 4096
    a.lda = a.ldb = 112
    a.out_ld = 128
    assert lib.b2f_gemm_fp8(ctypes.byref(a), None) == L.B2F_ERR_ARG  # K % 16
    nrm = L.NormArgs()
    lib.b2f_norm_args_init(ctypes.byref(nrm))
    nrm.rows, nrm.cols = 4, 12
    assert lib.b2f_norm_quant(ctypes.byref(nrm), None) == L.B2F_ERR_ARG  # cols % 8
    nrm.cols = 8200
    nrm.x = nrm.weight = nrm.q_out = 4096
    assert lib.b2f_norm_quant(ctypes.byref(nrm), None) == L.B2F_ERR_UNSUPPORTED


def test_ops_refuse_cpu_tensors():
    import torch
    from b200fp8 import ops
    a = torch.zeros((128, 128), dtype=torch.float8_e4m3fn)
    with pytest.raises(ValueError, match="CUDA"):
        ops.gemm_fp8(a, a)


def test_auto_split_rule(monkeypatch):
    """The Python layer hands its cached split-K workspace to the shapes b2f_gemm_fp8's
    automatic choice may split (few 128 x 128 tiles, K >= 4096); the rest get none."""
    from b200fp8 import ops
    monkeypatch.setattr(ops, "_sm_count", lambda index: 148)
    assert ops._auto_split(128, 8192, 8192, "cuda:0")
    assert not ops._auto_split(128, 8192, 2048, "cuda:0")    # short K
    assert not ops._auto_split(128, 32768, 8192, "cuda:0")   # 256 tiles fill the GPU
    assert not ops._auto_split(8192, 8192, 8192, "cuda:0")   # large M: CTA pairs
    assert ops._auto_split(256, 4096, 8192, "cuda:0")         # 64 tiles, long K, M > 128
    assert not ops._auto_split(256, 8192, 8192, "cuda:0")     # 128 tiles: more than half
    assert ops._auto_split(128, 8192, 3969, "cuda:0")         # ceil(K / 128) = 32
    assert not ops._auto_split(128, 8192, 3968, "cuda:0")     # ceil(K / 128) = 31
