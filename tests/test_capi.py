"""The C-ABI library loads and exports what include/ogx.h declares; host-side guards (no GPU needed)."""

import ctypes
import os
import re

import pytest

from opengenie_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "ogx.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ogx_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.EXPORTED)


def _declared_parameters():
    """name -> list of C parameter types, from the prototypes in include/ogx.h."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for ret, name, params in re.findall(r"\b(int|const char\*)\s+(ogx_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = " ".join(params.split())
        out[name] = [] if params in ("", "void") else [p.strip().rsplit(" ", 1)[0] for p in params.split(",")]
    return out


def _ctype_of(c_type: str):
    if "*" in c_type:
        return "pointer"
    return {"int64_t": ctypes.c_int64, "int": ctypes.c_int, "float": ctypes.c_float}[c_type]


def test_binding_argument_types_match_the_header():
    """Every ctypes signature has the header's parameter count and kinds (an int64 where the prototype has
    int64_t, a pointer where it has a pointer), so no call passes a misread argument."""
    declared = _declared_parameters()
    assert sorted(declared) == sorted(_lib.EXPORTED)
    for name, argtypes in _lib._SIGNATURES.items():
        c_params = declared[name]
        assert len(c_params) == len(argtypes), name
        for i, (c_type, py_type) in enumerate(zip(c_params, argtypes)):
            want = _ctype_of(c_type)
            if want == "pointer":
                assert py_type is ctypes.c_void_p or issubclass(py_type, ctypes._Pointer), (name, i, c_type)
            else:
                assert py_type is want, (name, i, c_type, py_type)


def test_library_exports_every_declared_symbol(ogx_lib):
    for name in declared_functions():
        assert hasattr(ogx_lib, name), name


def test_version(ogx_lib):
    assert ogx_lib.ogx_version() == 1


def _err(ogx_lib):
    return ogx_lib.ogx_last_error().decode()


def test_guards_reject_before_touching_the_device(ogx_lib):
    # tokens < 1 -> the reference's "empty_tokens" reason (triton_ltx_ops.py:1527-1528)
    rc = ogx_lib.ogx_video_qk_rmsnorm_rope(1 << 20, 1 << 20, 0, 4096, 1 << 20, 1 << 20, 0, 1e-6, 1 << 20, 1 << 20, 0,
                                          17 * 64, 64, 1 << 20, 1 << 20, 4096, None)
    assert rc == -1 and _err(ogx_lib) == "empty_tokens"
    # head_dim other than 128
    rc = ogx_lib.ogx_attention_fwd(16, 16, 16, 1, 128, 32, 64, 0, 4096, 0.1, 16, 0, 4096, None)
    assert rc == -1 and "head_dim" in _err(ogx_lib)
    # GEMM K must be a multiple of 16 (TMA row pitch)
    rc = ogx_lib.ogx_fp8_scaled_mm(16, 128, 100, 112, 16, 256, 112, 16, 16, 256, None, 0, 16, 256, None)
    assert rc == -1 and "shape" in _err(ogx_lib)
    # AdaZero column count outside {2048, 4096} (triton_ltx_ops.py:1005)
    rc = ogx_lib.ogx_adazero_from_ada(16, 1, 4, 1024, 16, 1, 1024, 16, 0, 0, 0, 1024, 0, 1, 1e-6, 16, None)
    assert rc == -1 and _err(ogx_lib) == "cols"
    # quantiser dtype must be bf16 or f16 (triton_ltx_ops.py:1021-1022)
    rc = ogx_lib.ogx_fp8_quantize_e4m3(16, 1, 64, 16, 0, 16, None)
    assert rc == -1 and _err(ogx_lib) == "x_dtype"
    # attention over keys of another length: no keys, and a key row stride narrower than the heads
    rc = ogx_lib.ogx_attention_fwd_kv(16, 16, 16, 1, 128, 0, 32, 128, 0, 4096, 0, 4096, 0.1, 16, 0, 4096, None)
    assert rc == -1 and _err(ogx_lib) == "shape"
    rc = ogx_lib.ogx_attention_fwd_kv_e4m3(16, 16, 16, 1, 128, 77, 32, 128, 0, 4096, 0, 2048, 0.1, 16, 16, 0, 4096,
                                           None)
    assert rc == -1 and _err(ogx_lib) == "stride"
    # Q/K RMSNorm without RoPE: rows of 4096 need a row stride of at least 4096
    rc = ogx_lib.ogx_qk_rmsnorm(16, 4, 2048, 16, 4, 4096, 16, 16, 0, 1e-6, 16, 4096, 16, 4096, None)
    assert rc == -1 and _err(ogx_lib) == "qk_stride"


def test_ops_refuse_cpu_tensors():
    import torch

    from opengenie_b200 import ltx_ops

    x = torch.zeros((1, 4, 4096), dtype=torch.bfloat16)
    s = torch.tensor(1.0)
    with pytest.raises(ValueError):
        ltx_ops.fused_fp8_quantize_e4m3(x, s)
    table = torch.zeros((6, 4096))
    ts = torch.zeros((1, 4, 6 * 4096), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="x_device_or_dtype"):
        ltx_ops.fused_adazero_from_ada(x, 1e-6, table, ts, shift_index=0, scale_index=1)
    cos = torch.zeros((1, 32, 4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="qk_device_or_dtype"):
        ltx_ops.fused_video_qk_rmsnorm_rope(x, x, x[0, 0], x[0, 0], 1e-6, cos, cos)


def test_python_surface_exports_every_public_op():
    """``ltx_ops.__all__`` names every public function and class (the reference's op names and this library's
    fused ones, the RopePositions argument type) and the quantiser mode constants, and nothing that does not
    exist."""
    import inspect

    from opengenie_b200 import ltx_ops

    public = {n for n, f in vars(ltx_ops).items()
              if (inspect.isfunction(f) or inspect.isclass(f)) and f.__module__ == ltx_ops.__name__
              and not n.startswith("_")}
    assert public | {"QUANT_SINGLE", "QUANT_TORCH"} == set(ltx_ops.__all__)
