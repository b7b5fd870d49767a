"""CPU checks of the C ABI library: it loads, exports every symbol the
public header declares, and rejects invalid arguments before touching a
device.  No compute call is made here (there is no GPU on this host)."""
import os
import re
import subprocess

import pytest

from gpu_algos_b200 import capi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "glm_b200.h")


def _declared_functions():
    # expand the header's declaration macros with the C preprocessor
    out = subprocess.run(["gcc", "-E", "-P", "-x", "c", HEADER], check=True, capture_output=True,
                         text=True).stdout
    return sorted(set(re.findall(r"\b(glmb_\w+)\s*\(", out)))


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_loads_and_exports_every_declared_symbol():
    L = capi.lib()
    declared = _declared_functions()
    # basics, per-type entry points, floating-point entry points, the no-allocation
    # entry point, the peer group, sharded gradient (float/double, then the
    # 16-bit types' partial/finalize/sharded) and fit, the multi-GPU context
    assert len(declared) == 4 + 4 * 12 + 9 * 2 + 1 + 6 + 2 + 3 * 2 + 2 + 5 + 2 * 2
    exported = _exported()
    missing = [n for n in declared if n not in exported]
    assert not missing, missing
    for n in declared:
        assert hasattr(L, n)
    assert sorted(capi.exported_symbols()) == declared
    assert capi.version() == 100


def test_no_unexpected_exports():
    # everything the library exports under the glmb_ prefix is declared
    extra = {n for n in _exported() if n.startswith("glmb_")} - set(_declared_functions())
    assert not extra, extra


def test_status_strings():
    assert capi.status_string(0) == "success"
    assert "workspace" in capi.status_string(capi.GLMB_ERR_WORKSPACE)
    assert "invalid" in capi.status_string(capi.GLMB_ERR_INVALID_VALUE)
    assert "sm_100a" in capi.status_string(capi.GLMB_ERR_UNSUPPORTED)
    assert "NCCL" in capi.status_string(capi.GLMB_ERR_COLLECTIVE)
    assert "peer" in capi.status_string(capi.GLMB_ERR_PEER_TIMEOUT)


def test_argument_validation_happens_before_any_device_call():
    L = capi.lib()
    before = capi.launch_count()
    # negative sizes and bad flags are rejected without touching CUDA
    assert L.glmb_gradient_f32(None, None, None, None, None, -1, 1, 1, 1, 0.0, 0.0, 0, None, 0, None) == 1001
    assert L.glmb_gradient_f64(None, None, None, None, None, 4, 1, 1, 8, 0.0, 0.0, 0x100, None, 0, None) == 1001
    # the logistic link is for floating types only
    assert L.glmb_gradient_i32(None, None, None, None, None, 4, 1, 1, 8, 0.0, 0.0, capi.GRAD_LOGISTIC, None, 0,
                               None) == 1001
    assert L.glmb_predict_i32(None, None, None, 3, -2, 1, 1, None) == 1001
    assert L.glmb_prox_step_f32(None, None, -5, 1.0, 0.0, None) == 1001
    assert L.glmb_prox_update_f64(None, None, None, 4, 1, 1, -1.0, 0.0, None) == 1001
    # empty problems are successful no-ops
    assert L.glmb_predict_f32(None, None, None, 8, 0, 1, 5, None) == 0
    assert L.glmb_gradient_u8(None, None, None, None, None, 8, 1, 0, 5, 0.0, 0.0, 0, None, 0, None) == 0
    # the multi-GPU context checks its arguments before any device is touched
    import ctypes
    mg = ctypes.c_void_p()
    devs = (ctypes.c_int * 2)(0, 0)
    assert L.glmb_mg_create(2, devs, 16, 100.0, capi.MG_PEER, ctypes.byref(mg)) == 1001  # a device twice
    assert L.glmb_mg_create(0, devs, 16, 100.0, capi.MG_PEER, ctypes.byref(mg)) == 1001
    assert L.glmb_mg_create(1, devs, 16, 100.0, 7, ctypes.byref(mg)) == 1001
    assert L.glmb_mg_synchronize(None) == 1001 and L.glmb_mg_size(None) == 0
    assert L.glmb_mg_destroy(None) == 0
    assert L.glmb_fit_elastic_net_sharded_f32(None, None, None, None, 4, 1, 1, 8, 0.0, 0.0, 1, 1, 0, None, None, 0,
                                              None) == 1001
    assert capi.launch_count() == before


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(capi, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(capi, "_lib", None)
    with pytest.raises(ImportError):
        capi.lib()
