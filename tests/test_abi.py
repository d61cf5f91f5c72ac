"""CPU tests of the C ABI surface: the library loads, exports every entry point
include/*.h declares, and rejects bad arguments without a GPU."""
import ctypes as C
import glob
import os
import re

import numpy as np
import pytest

from conftest import ROOT


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(dvs_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_functions()
    assert "dvs_open" in names and "dvs_search" in names and len(names) >= 15


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(dvs, name):
    assert hasattr(dvs.lib(), name), f"{name} declared in include/ but not exported"


def test_binding_list_matches_header(dvs):
    from dvstor_b200 import _lib

    assert set(_lib.EXPORTED) <= set(declared_functions())


def test_status_strings(dvs):
    L = dvs.lib()
    assert L.dvs_status_string(0) == b"ok"
    assert L.dvs_status_string(11) == b"capacity exceeded"
    assert L.dvs_status_string(999) == b"unknown status"


def test_null_arguments_are_rejected(dvs):
    L = dvs.lib()
    assert L.dvs_open(None, None) == 1
    assert L.dvs_close(None) == 1
    assert L.dvs_search(None, None, 0, 0, 0, 0, 0, None, None, None) == 1
    assert L.dvs_set_hop_limit(None, 3) == 1
    assert L.dvs_query_prepare(None, None, None, None, None, 1, 4, 4, None) == 1


def test_open_without_device_reports_no_device(dvs, tmp_path):
    if dvs.lib().dvs_device_count() > 0:
        pytest.skip("a device is visible")
    with pytest.raises(dvs.DvsError) as e:
        dvs.Index(str(tmp_path / "x"))
    assert e.value.name == "DVS_ERR_NO_DEVICE"


def test_compute_service_validates_flags(dvs):
    with pytest.raises(ValueError):
        dvs.ComputeService(search_mode="cpu")
    with pytest.raises(ValueError):
        dvs.ComputeService(rabitq_bits=3)
    with pytest.raises(ValueError):
        dvs.ComputeService(beam_width=5, k=10)
    s = dvs.ComputeService(beam_width=64, k=10)
    with pytest.raises(dvs.DvsError):
        s.search_batch(np.zeros((1, 4), np.float32))
