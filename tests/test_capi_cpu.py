"""The C-ABI library without a GPU: it loads, exports every symbol that
include/pcb200.h declares, and rejects bad arguments before touching CUDA."""

import os
import re

import pytest

from practice_cuda_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "pcb200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z0-9_]+\*?\s+\*?(pcb_[a-z0-9_]+)\(", text, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for required in ["pcb_quant_per_block", "pcb_quant_per_channel", "pcb_quant_per_tensor",
                     "pcb_bmm_scaled", "pcb_pack_u8", "pcb_get_device_error"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in _declared():
        assert hasattr(lib, name), name
    assert set(_declared()) == set(_lib.exported_symbols())


def test_abi_version_matches_header():
    m = re.search(r"#define PCB200_ABI_VERSION (\d+)", open(HEADER).read())
    assert _lib.lib().pcb_version() == int(m.group(1))


def test_status_names():
    assert _lib.status_name(0) == "PCB_OK"
    assert _lib.status_name(3) == "PCB_ERR_LAYOUT"
    assert _lib.status_name(99) == "PCB_ERR_UNKNOWN"


def test_invalid_arguments_rejected_without_gpu():
    lib = _lib.lib()
    # block sizes must be positive
    st = lib.pcb_quant_per_block(None, 2, 1, 4, 4, 0, 4, 1, None, 3, 0, 4, 1, None, 0, 1, 1, 0, 128, 1e-12, None)
    assert st == _lib.PCB_ERR_INVALID
    # negative sizes
    st = lib.pcb_quant_per_channel(None, 2, 1, -1, 4, 0, 4, 1, None, 3, 0, 4, 1, None, 0, 1, -2, 1e-12, None)
    assert st == _lib.PCB_ERR_INVALID
    # bad channel axis
    st = lib.pcb_quant_per_channel(None, 2, 1, 4, 4, 0, 4, 1, None, 3, 0, 4, 1, None, 0, 1, 0, 1e-12, None)
    assert st == _lib.PCB_ERR_INVALID
    # bad input dtype (fp8 input to a quantizer)
    st = lib.pcb_quant_per_block(1, 3, 1, 4, 4, 0, 4, 1, 1, 3, 0, 4, 1, 1, 0, 1, 1, 1, 128, 1e-12, None)
    assert st == _lib.PCB_ERR_INVALID
    # empty problem is a no-op
    st = lib.pcb_quant_per_block(None, 2, 0, 4, 4, 0, 4, 1, None, 3, 0, 4, 1, None, 0, 1, 1, 1, 128, 1e-12, None)
    assert st == _lib.PCB_OK
    # bmm: bf16 operands are not fp8
    st = lib.pcb_bmm_scaled(1, 0, 16, 1, 1, 0, 1, 16, 2, 1, 16, 16, 16, None, 0, 0, 0, 1, None, 0, 0, 0, 1, 16,
                            None, 0, 0, 0, 0, 1, 2, 0, 16, 1, 0, None)
    assert st == _lib.PCB_ERR_INVALID
    # bmm: non-positive quant block
    st = lib.pcb_bmm_scaled(1, 0, 16, 1, 1, 0, 1, 16, 3, 1, 16, 16, 16, None, 0, 0, 0, 0, None, 0, 0, 0, 1, 16,
                            None, 0, 0, 0, 0, 1, 2, 0, 16, 1, 0, None)
    assert st == _lib.PCB_ERR_INVALID
    # pack: padded width below the source width
    assert lib.pcb_pack_u8(None, 1, 2, 8, 16, 8, 1, None, 16, 4, 4, None) == _lib.PCB_ERR_INVALID
    assert "pack" in _lib.lib().pcb_last_error_text().decode()


def test_check_raises_with_status():
    with pytest.raises(_lib.Pcb200Error) as ei:
        _lib.check(_lib.PCB_ERR_LAYOUT, "op")
    assert ei.value.status == _lib.PCB_ERR_LAYOUT


def test_new_entry_points_reject_bad_arguments_without_gpu():
    lib = _lib.lib()
    # dynamic float8 cast: axiswise must be 0 or 1; fp8 input rejected
    st = lib.pcb_quant_float8_dynamic(None, 2, 1, 4, 4, 0, 4, 1, None, 3, 0, 4, 1, None, 0, 1, 2, 1e-12, None, None)
    assert st == _lib.PCB_ERR_INVALID
    st = lib.pcb_quant_float8_dynamic(1, 3, 1, 4, 4, 0, 4, 1, 1, 3, 0, 4, 1, 1, 0, 1, 1, 1e-12, None, None)
    assert st == _lib.PCB_ERR_INVALID
    # mixed-format BMM: B's dtype must be fp8
    st = lib.pcb_bmm_scaled_mixed(1, 0, 128, 1, 3, 1, 0, 128, 1, 2, 1, 128, 128, 128,
                                  None, 0, 0, 0, 1, None, 0, 0, 0, 1, 128,
                                  None, 0, 0, 0, 0, 1, 2, 0, 128, 1, 0, None)
    assert st == _lib.PCB_ERR_INVALID
