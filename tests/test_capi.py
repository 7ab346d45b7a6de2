"""The C-ABI boundary on the CPU box: the library loads, exports every symbol
include/p100/b200.h declares, validates arguments with the reference's
wording before touching a device, refuses to compute without an sm_100 GPU
(no CPU fallback), and the C++ caller (tests/cpp/contract_check.cpp) builds
and gets the reference's exceptions."""
import ctypes as C
import os
import subprocess

import pytest

from conftest import ROOT

import p100_b200 as P


def no_gpu():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        return True


def test_exports_every_declared_symbol(lib):
    syms = P.symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(P.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert set(syms) <= exported


def test_sizes_and_versions(lib):
    assert lib.p100_abi_version() == 3
    assert [lib.p100_block_elems(t) for t in (0, 1, 2, 3, 4, 9)] == [32, 32, 256, 256, 256, -1]
    assert [lib.p100_block_bytes(t) for t in (0, 1, 2, 3, 4, 9)] == [18, 34, 144, 176, 210, -1]
    assert lib.p100_weight_bytes(P.Q4_0, 14336, 4096) == 33030144
    assert lib.p100_weight_bytes(P.Q4_K, 2, 128) == 0
    assert lib.p100_q8_1_bytes(4096, 2) == 2 * 128 * 36
    assert lib.p100_status_name(4) == b"P100_ERR_TIMEOUT"


def test_invalid_arguments_use_reference_wording(lib):
    z = C.c_void_p(16)
    assert lib.p100_qmv(P.Q4_K, z, 4, 128, z, 1, z, None) == P.ERR_INVALID
    assert P.last_error() == "whole weight blocks required"
    assert lib.p100_qmv(7, z, 4, 128, z, 1, z, None) == P.ERR_INVALID
    assert lib.p100_qmv(P.Q4_0, z, 4, 128, z, 17, z, None) == P.ERR_INVALID
    assert lib.p100_q8_1_quantize(z, z, 33, 1, None) == P.ERR_INVALID
    assert P.last_error() == "whole activation blocks required"
    ok, why = P.attn_validate(P.AttnDesc(n_head_q=3, n_head_kv=2))
    assert not ok and why == "n_head_q must be divisible by n_head_kv"
    ok, why = P.attn_validate(P.AttnDesc(softcap=-1.0))
    assert not ok and why == "softcap must be finite and non-negative"
    assert P.attn_validate(P.AttnDesc(seq_q=5, seq_kv=3, causal=True)) == (True, "")
    d = P.AttnDesc(seq_kv=0)
    assert lib.p100_fa_decode(C.byref(d), z, z, z, None, z, None, None, 0, None) == P.ERR_INVALID
    assert P.last_error() == "all dimensions must be positive"
    # quantised K/V conversion: shape and type checks come before any device call
    kv = lib.p100_kv_to_f16
    kv.argtypes = [C.c_int, C.c_void_p] + [C.c_longlong] * 7 + [C.c_void_p, C.c_void_p]
    assert kv(P.KV_F16, z, 128, 4, 1, 1, 4, 16, 16, z, None) == P.ERR_INVALID
    assert kv(P.KV_Q8_0, z, 48, 4, 1, 1, 2, 8, 8, z, None) == P.ERR_INVALID
    assert P.last_error() == "ne00 must be a positive multiple of 32"
    assert kv(P.KV_Q4_0, z, 128, 4, 1, 1, -1, 16, 16, z, None) == P.ERR_INVALID
    assert kv(P.KV_Q8_0, C.c_void_p(17), 128, 4, 1, 1, 4, 16, 16, z, None) == P.ERR_INVALID
    assert P.last_error() == "src must be 2-byte aligned"
    assert kv(P.KV_Q8_0, z, 128, 0, 1, 1, 4, 16, 16, z, None) == P.OK   # nothing to convert
    assert lib.p100_fa_workspace_size(C.byref(d)) == 0
    assert P.last_error() == "all dimensions must be positive"


@pytest.mark.skipif(not no_gpu(), reason="checks the behaviour without a GPU")
def test_no_cpu_fallback(lib):
    z = C.c_void_p(16)
    assert lib.p100_device_check(0) == P.ERR_UNSUPPORTED
    assert lib.p100_qmv(P.Q4_0, z, 4, 4096, z, 1, z, None) == P.ERR_UNSUPPORTED
    assert lib.p100_q8_1_quantize(z, z, 64, 1, None) == P.ERR_UNSUPPORTED
    d = P.AttnDesc(n_head_q=8, n_head_kv=2, seq_kv=100)
    assert lib.p100_fa_decode(C.byref(d), z, z, z, None, z, None, None, 0, None) == P.ERR_UNSUPPORTED


def test_host_fault_injection_tp_init(lib, monkeypatch):
    monkeypatch.setenv("P100_FAULT", "alloc,tp_init")
    h = C.c_void_p()
    buf = (C.c_ubyte * P.TP_ID_BYTES)()
    assert lib.p100_tp_init_rank(buf, 2, 0, 0, C.byref(h)) == P.ERR_NCCL
    assert "injected fault: tp_init" in P.last_error()
    devs = (C.c_int * 2)(0, 1)
    hs = (C.c_void_p * 2)()
    assert lib.p100_tp_create(2, devs, hs) == P.ERR_NCCL
    monkeypatch.setenv("P100_FAULT", "tp_initx")
    assert lib.p100_tp_init_rank(buf, 2, 5, 0, C.byref(h)) == P.ERR_INVALID   # rank 5 of 2


def test_p2p_env_switch(lib, monkeypatch):
    for value, disabled in (("", False), ("0", False), ("1", True), ("false", True), ("00", True)):
        monkeypatch.setenv("P100_DISABLE_P2P", value)
        assert lib.p100_p2p_disabled_by_env() == int(disabled)
    monkeypatch.delenv("P100_DISABLE_P2P")
    assert lib.p100_p2p_disabled_by_env() == 0


def test_cpp_caller_builds_and_gets_reference_errors():
    subprocess.run(["make", "-s", "-C", str(ROOT / "tests" / "cpp")], check=True)
    exe = ROOT / "tests" / "cpp" / "bin" / "contract_check"
    env = dict(os.environ)
    if no_gpu():
        env["CUDA_VISIBLE_DEVICES"] = ""
    r = subprocess.run([str(exe), "errors"], capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS errors" in r.stdout


@pytest.mark.gpu
def test_cpp_caller_gpu_path():
    """The C++ caller (tests/cpp/contract_check.cpp) on the B200: Q8_1
    prepare bit-exact, a Q4_K mat-vec and a split FA decode against the
    oracle, through include/p100/b200.hpp."""
    subprocess.run(["make", "-s", "-C", str(ROOT / "tests" / "cpp")], check=True)
    exe = ROOT / "tests" / "cpp" / "bin" / "contract_check"
    r = subprocess.run([str(exe), "gpu"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout, r.stdout
    assert "PASS" in r.stdout, r.stdout
