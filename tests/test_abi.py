"""The C-ABI library: it loads without a GPU, exports every function that
include/s3t.h declares, and fails cleanly (status + message) when no GPU is
usable.  No compute is launched here."""

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    text = (ROOT / "include" / "s3t.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(s3t_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def libs3t():
    from sam3cpp_b200 import LIB_PATH, lib
    if not LIB_PATH.exists():
        pytest.skip("libs3t.so not built")
    return lib()


def test_header_declares_the_abi():
    names = declared_functions()
    for required in ["s3t_create", "s3t_destroy", "s3t_last_error", "s3t_set_weight", "s3t_load_gguf",
                     "s3t_finalize_weights", "s3t_trunk_run", "s3t_trunk_run_layers", "s3t_sync",
                     "s3t_dequantize", "s3t_gemm_f16", "s3t_attention", "s3t_layernorm"]:
        assert required in names


def test_library_exports_every_declared_symbol(libs3t):
    missing = [n for n in declared_functions() if not hasattr(libs3t, n)]
    assert not missing, missing


def test_no_gpu_fails_cleanly(libs3t):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    ctx = libs3t.s3t_create(0)
    assert not ctx
    assert libs3t.s3t_last_error().decode()


def test_null_arguments_are_errors(libs3t):
    assert libs3t.s3t_trunk_run(None, None, 1, None, 0, None) == -1
    assert b"null" in libs3t.s3t_last_error()
    assert libs3t.s3t_finalize_weights(None) == -1
    ne = (C.c_int64 * 4)(1, 1, 1, 1)
    assert libs3t.s3t_set_weight(None, b"x", 0, ne, None, 0) == -1


def test_python_mirror_raises_without_gpu(libs3t):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import sam3cpp_b200 as s3t
    with pytest.raises(s3t.S3TError):
        s3t.GgufModel("/nonexistent.gguf")


def test_multi_gpu_handle_fails_cleanly_without_arguments(libs3t):
    assert not libs3t.s3t_multi_create(None, 0, b"x.gguf", None)
    assert b"devices" in libs3t.s3t_last_error()
    assert libs3t.s3t_multi_run(None, None, 1, None, 0, None) == -1
    assert libs3t.s3t_multi_num_devices(None) == 0


def test_dropin_library_resolves_every_symbol(libs3t):
    """The reference linked with the drop-in trunk (oracle/_ref/libsam3ref_s3t.so,
    built by `make -C oracle dropin`) loads with every symbol resolved: the
    harness's neck entries need the reference's own src/vision_neck.cpp."""
    lib = ROOT / "oracle" / "_ref" / "libsam3ref_s3t.so"
    if not lib.exists():
        pytest.skip("drop-in reference library not built")
    # RTLD_LOCAL: this library carries its own ggml build, which must not
    # stand in for the symbols of the reference builds later tests load.
    C.CDLL(str(lib), mode=C.RTLD_LOCAL)
