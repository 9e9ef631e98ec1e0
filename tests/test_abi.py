"""The C-ABI library loads and exports every entry point include/gdn_b200.h declares.

CPU-only: loading the library and argument validation make no CUDA calls.
"""
import re
from pathlib import Path

import pytest

from flashinfer_bench_tma_thrust_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "gdn_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return re.findall(r"GDN_API\s+[\w\s\*]+?\b(gdn_\w+)\s*\(", text)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "gdn_decode_fwd" in syms and "gdn_prefill_recurrent_fwd" in syms


def test_library_exports_every_declared_symbol(cuda_lib):
    for name in declared_symbols():
        assert hasattr(cuda_lib, name), f"{name} declared in gdn_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in _lib.SIGNATURES"


def test_abi_version_and_status_strings(cuda_lib):
    assert cuda_lib.gdn_abi_version() >= 1
    assert cuda_lib.gdn_status_string(0) == b"ok"
    for code in (-1, -2, -3, -4, -5, -6):
        assert cuda_lib.gdn_status_string(code) != b"unknown status"


NULL = None


def _decode(lib, B=1, HQ=1, HV=2, D=128, dt=(0, 0, 0, 0), ptr=1):
    p = ptr
    return lib.gdn_decode_fwd(p, p, p, NULL, p, dt[0], p, dt[1], p, dt[2], p, dt[3], 0.0, p, p,
                              B, HQ, HV, D, NULL)


def test_decode_validation_without_gpu(cuda_lib):
    lib = cuda_lib
    assert _decode(lib, D=64) == -2
    assert _decode(lib, HQ=3, HV=4) == -2
    assert _decode(lib, dt=(5, 0, 0, 0)) == -3
    assert _decode(lib, B=-1) == -1
    assert _decode(lib, B=0) == 0           # empty batch is a no-op
    assert _decode(lib, ptr=None) == -1     # null tensors rejected before any launch


def test_prefill_validation_without_gpu(cuda_lib):
    lib = cuda_lib
    p = 1

    def call(T=4, N=1, cu_dt=2, D=128):
        return lib.gdn_prefill_recurrent_fwd(p, p, p, None, p, 0, p, 0, p, 0, p, 0, p, cu_dt,
                                             0.0, p, p, T, N, 1, 2, D, None)
    assert call(cu_dt=0) == -3
    assert call(D=256) == -2
    assert call(T=-1) == -1
    assert call(N=0) == 0


def test_prefill_launch_count_validation_without_gpu(cuda_lib):
    """gdn_prefill_chunked_launches checks its sizes before it queries the device; a
    workspace below the two-phase size selects the fused path: one launch."""
    lib = cuda_lib
    assert lib.gdn_prefill_chunked_launches(100, 0, 32, 1 << 30) == 0
    assert lib.gdn_prefill_chunked_launches(-1, 1, 32, 1 << 30) == -1
    assert lib.gdn_prefill_chunked_launches(100, 1, 32, 16) == -5   # workspace too small
    assert lib.gdn_prefill_chunked_launches(4096, 2, 32, 256) == 1  # fused path


@pytest.mark.gpu
def test_prefill_launch_count_rule(monkeypatch):
    """Launches per chunked-prefill call as the library reports them (the bench's
    gpu_launches): 4, plus a scan-order launch above 1024 sequences, plus a second prep
    and scan for split calls (few long sequences leaving SMs idle; values for 148 SMs)."""
    import torch
    from flashinfer_bench_tma_thrust_b200 import prefill as P
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("launch counts below are for a 148-SM B200")
    monkeypatch.delenv("GDN_PREFILL_OVERLAP", raising=False)
    assert P.launches_per_call(4, 4 * 32768, 32) == 6     # long config: split
    assert P.launches_per_call(8, 19679, 32) == 4         # varlen: 256 chains
    assert P.launches_per_call(4, 4 * 1000, 32) == 4      # too short to split
    assert P.launches_per_call(2000, 10**6, 1) == 5       # separate scan order
    monkeypatch.setenv("GDN_PREFILL_OVERLAP", "0")
    assert P.launches_per_call(4, 4 * 32768, 32) == 4
