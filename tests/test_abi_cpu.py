"""CPU-only checks of the C-ABI boundary: the library loads without a GPU and
exports every symbol include/beacon_cuda.h declares (no compute calls)."""
import ctypes
import os
import re

import pytest

from beacon_cuda import _lib as L


def test_library_built():
    assert os.path.exists(L.LIB_PATH), "run __graft_entry__.build() first"


def test_exports_every_header_symbol():
    lib = ctypes.CDLL(L.LIB_PATH)
    names = L.header_symbols()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_table_matches_header():
    assert sorted(L.SIGNATURES) == L.header_symbols()


def test_status_and_dtype_values_match_reference():
    # BeaconStatus (shim/include/beacon_shim.h:24-33) and BeaconDtype
    # (crates/beacon-format/src/dtype.rs:12-29) discriminants
    text = open(L.HEADER).read()
    vals = dict(re.findall(r"(BEACON_CUDA_[A-Z0-9_]+)\s*=\s*(\d+)", text))
    assert vals["BEACON_CUDA_OK"] == "0" and vals["BEACON_CUDA_ERR_INVALID_ARGUMENT"] == "1"
    assert vals["BEACON_CUDA_ERR_OUT_OF_MEMORY"] == "2" and vals["BEACON_CUDA_ERR_SHAPE_MISMATCH"] == "3"
    assert vals["BEACON_CUDA_ERR_UNSUPPORTED_DTYPE"] == "4" and vals["BEACON_CUDA_ERR_UNKNOWN"] == "99"
    assert vals["BEACON_CUDA_DTYPE_Q4_0"] == "100" and vals["BEACON_CUDA_DTYPE_Q4_K"] == "101"
    assert vals["BEACON_CUDA_DTYPE_Q8_0"] == "104" and vals["BEACON_CUDA_DTYPE_Q8_K"] == "110"


def test_null_arguments_rejected_without_gpu():
    lib = L.lib()
    # argument validation happens before any CUDA call
    assert lib.beacon_cuda_context_create(0, None) == L.ERR_INVALID_ARGUMENT
    assert b"null" in lib.beacon_cuda_last_error_message()
    assert lib.beacon_cuda_tensor_shape(None, None, None) == L.ERR_INVALID_ARGUMENT
    assert lib.beacon_cuda_comm_unique_id(None) == L.ERR_INVALID_ARGUMENT


def test_context_create_reports_missing_device():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    st = L.lib().beacon_cuda_context_create(0, ctypes.byref(h))
    assert st != L.OK
    assert L.lib().beacon_cuda_last_error_message()
