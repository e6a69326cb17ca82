"""CPU checks of the drop-in boundary: libu15c.so loads, exports exactly
what include/u15c.h declares, and refuses bad arguments before touching a
device. No kernel runs here."""
import ctypes as C
import os
import subprocess

import pytest

import u15b200
from u15b200 import _lib as L


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        pytest.fail(f"{L.LIB_PATH} missing: __graft_entry__.build() builds it")
    return L.lib()


def test_exports_every_declared_symbol(lib):
    declared = set(L.header_symbols())
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " u15c_" in ln}
    assert declared, "no declarations parsed"
    assert declared <= exported, sorted(declared - exported)
    assert exported <= declared, sorted(exported - declared)
    # and the ctypes signature table covers the same surface
    assert declared == set(L.SIGNATURES)


def test_version_and_errors(lib):
    assert b"sm_100a" in lib.u15c_version()
    # refused before any CUDA call: unknown epilogue, bad quant width
    rc = lib.u15c_mot_linear_bf16(None, None, None, 2, None, None, 0, 7, None, None, None, 1, 8, 8)
    assert rc == L.EINVAL and "epilogue" in L.last_error()
    rc = lib.u15c_quant_rows_i8(None, None, None, None, 1, 12)
    assert rc == L.EINVAL
    rc = lib.u15c_split_qk_norm(None, None, None, None, 1, 1, 96, 1e-6)
    assert rc == L.EINVAL and "128" in L.last_error()
    rc = lib.u15c_split_rope(None, None, None, None, 1, 1, 128, 32, 32)
    assert rc == L.EINVAL


def test_sizes_are_host_arithmetic(lib):
    # Sage workspace: q8 + k8 + scales, 256-byte aligned pieces
    n = lib.u15c_sage_workspace_bytes(32, 8, 4096, 4416)
    assert n >= 32 * 4096 * 128 + 8 * 4416 * 128


def test_model_config_validation(lib):
    cfg = L.Config(n_layers=1, hidden=4096, heads=32, kv_heads=8, head_dim=96, inter=12288,
                   n_experts=2, eps=1e-6, theta_t=5e6, theta_hw=1e4)
    h = C.c_void_p()
    rc = lib.u15c_model_create(C.byref(cfg), 0, C.byref(h))
    assert rc == L.EINVAL and "head_dim" in L.last_error()


def test_package_exposes_reference_surface():
    # the MetalOps method names the backbone calls (src/u15-metal-ops.h)
    for name in ("linear", "rms_norm", "split_qk_norm", "split_rope", "build_rope_tables",
                 "swiglu", "sdpa", "sdpa_steel", "sdpa_block_causal", "transpose_thd",
                 "transpose_htd", "transpose_into_cache", "add", "add_row", "silu"):
        assert hasattr(u15b200.CudaOps, name), name
    for name in ("make_cache", "kv_bytes", "scratch_bytes", "forward", "layer_forward",
                 "final_norm", "bind", "finalize"):
        assert hasattr(u15b200.Model, name), name
