"""CPU checks of the drop-in boundary: the shared library loads without a GPU
and exports every entry point include/omeinsum_b200.h declares; host-side
argument validation fails with a status code instead of crashing."""
import ctypes
import os
import re

import pytest

from conftest import ROOT, load_pkg

HEADER = os.path.join(ROOT, "include", "omeinsum_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(om_b200_\w+)\s*\(", text)))


def test_header_lists_match_package():
    om = load_pkg()
    assert sorted(om.EXPORTS) == declared_symbols()


def test_integration_binds_every_declared_symbol():
    """The reference-side FFI declarations shown for a maintainer cover the
    header exactly: every entry point, and none that does not exist."""
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    bound = sorted(set(re.findall(r"pub fn (om_b200_\w+)\s*\(", text)))
    assert bound == declared_symbols()


def test_library_exports_every_declared_symbol():
    om = load_pkg()
    L = ctypes.CDLL(om.LIB_PATH)
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing


def test_name_and_null_argument_errors():
    om = load_pkg()
    L = om.lib()
    assert L.om_b200_name() == b"b200"
    # null backend / out pointers are rejected before any CUDA call
    assert L.om_b200_create(0, None) == 1
    assert L.om_b200_sync(None) == 1
    assert L.om_b200_contract(None, 1, 0, None, 0, None, None, None, None, 0, None, None, None,
                              0, None, None, None, None) == 1
    buf = ctypes.create_string_buffer(256)
    L.om_b200_last_error(buf, 256)
    assert b"null" in buf.value


def test_create_without_gpu_reports_error():
    om = load_pkg()
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(om.OmError):
        om.B200(0)
