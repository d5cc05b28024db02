"""The C ABI boundary without a GPU: libmt.so loads, exports every function
include/mt.h declares, the ctypes table matches the header's parameter
counts, and argument errors come back as codes with messages before any
CUDA call is made."""
import ctypes as C
import re
from pathlib import Path

import pytest

from metal_autotune_b200 import build, lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "mt.h"


def declared() -> dict[str, int]:
    """name -> parameter count of every function declared in mt.h."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(?:int|size_t|uint64_t|const char\s*\*)\s+(mt_\w+)\s*\(([^)]*)\)\s*;", text):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


@pytest.fixture(scope="module")
def mt():
    build.build_library()
    return lib.load()


def test_header_declares_the_region_entry_points():
    names = declared()
    for required in ("mt_quantized_matmul", "mt_rms_norm", "mt_rope", "mt_swiglu", "mt_sdpa", "mt_diff_reduce",
                     "mt_linear", "mt_layer_norm", "mt_mamba_scan", "mt_last_error_string", "mt_version"):
        assert required in names


def test_every_declared_symbol_is_exported_and_bound(mt):
    names = declared()
    assert set(names) == set(lib.SIGNATURES), set(names) ^ set(lib.SIGNATURES)
    for name, nparams in names.items():
        assert hasattr(mt, name), name
        assert len(lib.SIGNATURES[name][1]) == nparams, name


def test_version_and_error_string(mt):
    assert lib.version() == (0, 1, 0)
    assert isinstance(mt.mt_last_error_string(), bytes)


def test_argument_errors_need_no_gpu(mt):
    rc = mt.mt_rms_norm(None, None, 1e-6, None, 4, 8, 0, None)
    assert rc == -1
    assert b"null pointer" in mt.mt_last_error_string()
    rc = mt.mt_quantized_matmul(None, None, None, None, None, 4, 8, 64, 64, 3, 0, None, 0, None)
    assert rc == -1 and b"x is NULL" in mt.mt_last_error_string()
    rc = mt.mt_sdpa(None, None, None, None, *([1] * 6), 1.0, 1, 0, *([0] * 12), 0, None)
    assert rc == -1
    with pytest.raises(lib.MTError, match="invalid argument"):
        lib.call("mt_swiglu", None, None, None, 8, 0, None)


def test_unsupported_dtype_is_reported(mt):
    p = C.c_void_p(16)  # never dereferenced: the dtype check comes first
    rc = mt.mt_quantized_matmul(p, p, p, p, p, 4, 8, 64, 64, 4, 2, None, 0, None)
    assert rc == -2 and b"not built" in mt.mt_last_error_string()


def test_workspace_queries_are_host_only(mt):
    assert lib.qmm_workspace_bytes(1, 4096, 2560, 4, 0) == 0          # decode runs the vector kernel
    assert lib.qmm_workspace_bytes(128, 6144, 2560, 4, 0) > 0         # prefill may split K
    assert mt.mt_diff_workspace_bytes(1 << 20) >= 256


def test_product_import_does_not_touch_the_oracle():
    import sys
    import subprocess
    code = ("import sys; import metal_autotune_b200.lib, metal_autotune_b200.autotuner_runtime.kernels, "
            "metal_autotune_b200.targets.qwen3; "
            "assert not any(m == 'oracle' or m.startswith('oracle.') for m in sys.modules), 'oracle imported'")
    subprocess.run([sys.executable, "-c", code], check=True, cwd=str(HEADER.parents[1]))


def test_fused_decode_cuts_check_arguments_without_gpu(mt):
    """The fused decode entry points refuse what only the unfused pair serves,
    before any CUDA call: more than 4 tokens (attention), a missing or
    misaligned norm weight (norm + matmul)."""
    p = C.c_void_p(256)  # never dereferenced: the checks come first
    rc = mt.mt_qk_norm_rope_sdpa_decode(p, p, p, 4096, 1024, p, p, 1e-6, p, p, p, 5, 32, 8, 128, 160, 0, 1e6,
                                        0.088, 0, None)
    assert rc == -1 and b"at most 4 tokens" in mt.mt_last_error_string()
    rc = mt.mt_qk_norm_rope_sdpa_decode(p, p, p, 4096, 1024, p, p, 1e-6, p, p, p, 1, 32, 8, 128, 128, 128, 1e6,
                                        0.088, 0, None)
    assert rc == -1 and b"exceeds cache capacity" in mt.mt_last_error_string()
    rc = mt.mt_rms_norm_quantized_matmul_multi(p, None, 1e-6, p, p, p, p, 256, None, None, None, None, 0, None, None,
                                               None, None, 0, 1, 1024, 64, 4, 0, None)
    assert rc == -1 and b"norm weight is NULL" in mt.mt_last_error_string()
    rc = mt.mt_rms_norm_quantized_matmul_swiglu(p, C.c_void_p(258), 1e-6, p, p, p, p, p, p, p, 1, 256, 1024, 64, 4,
                                                0, None)
    assert rc == -1 and b"16-byte aligned" in mt.mt_last_error_string()


def test_conv1d_checks_arguments_without_gpu(mt):
    p = C.c_void_p(256)
    rc = mt.mt_conv1d(p, p, None, p, 1, 100, 48, 64, 3, 1, 1, 1, 1, None)  # Cin not a multiple of 32
    assert rc == -2 and b"multiple of 32" in mt.mt_last_error_string()
    rc = mt.mt_conv1d(p, p, None, p, 1, 1, 64, 64, 5, 1, 1, 0, 1, None)  # input shorter than the kernel
    assert rc == -1 and b"shorter than the kernel" in mt.mt_last_error_string()


def test_rope_strided_checks_arguments_without_gpu(mt):
    import torch
    p = C.c_void_p(256)
    bf = lib.dtype_code(torch.bfloat16)
    rc = mt.mt_rope_strided(None, p, 1, 2, 4, 128, 128, 0, 1e4, 1.0, 0, 1024, 128, 256, 1024, 512, 128, bf, None)
    assert rc == -1 and b"mt_rope_strided: null pointer" in mt.mt_last_error_string()
    rc = mt.mt_rope_strided(p, p, 1, 2, 4, 64, 128, 0, 1e4, 1.0, 0, 512, 64, 128, 512, 256, 64, bf, None)
    assert rc == -1 and b"dims=128" in mt.mt_last_error_string()
    assert mt.mt_rope_strided(p, p, 0, 2, 4, 128, 128, 0, 1e4, 1.0, 0, 0, 0, 0, 0, 0, 0, bf, None) == 0  # empty
