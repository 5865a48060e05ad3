"""The C-ABI library loads without a GPU and exports every entry point of
include/distspmm.h; argument errors come back as status codes, never as a crash."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT
import distspmm_b200 as d
from distspmm_b200 import _lib


def _declared():
    src = open(os.path.join(ROOT, "include", "distspmm.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(dsp_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    names = _declared()
    assert len(names) >= 40
    L = _lib.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert set(names) == set(_lib.PROTOTYPES), set(names) ^ set(_lib.PROTOTYPES)


def test_version_and_device_count_without_gpu():
    L = _lib.lib()
    assert b"sm_100a" in L.dsp_version()
    assert L.dsp_device_count() >= 0


def test_status_codes_on_bad_arguments():
    L = _lib.lib()
    assert L.dsp_partition_bounds(10, 0, 0, None, None) == -1
    assert b"dsp_partition_bounds" in L.dsp_last_error()
    assert L.dsp_alloc_slice(0, 1, None) == -1
    assert L.dsp_comm_select(7, 128, None, None, 0, None, None, (ctypes.c_uint8 * 1)(), None) == -1
    with pytest.raises(d.DspError) as e:
        d.planner.partition_bounds(10, 0, 0)
    assert e.value.code == -1


def test_library_has_no_runtime_cuda_dependency():
    # cudart is linked statically so the library loads on hosts without the CUDA runtime
    import subprocess
    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out
