"""Shared tolerances and comparison helpers for the GPU parity tests.

Tolerances (written here once, used by every parity test):
* output (bf16):  |got - ref| <= OUT_ATOL + OUT_RTOL * |ref|, OUT_ATOL = OUT_RTOL = 1e-2
* new_state (fp32): relative Frobenius error <= STATE_REL_FROB = 1e-3, and the
  reference's own absolute thresholds where its tests state them
  (decode 1e-4, prefill 5e-4: gdn/tests/test_correctness.py:240, :513-514).
"""
import torch

OUT_ATOL = 1e-2
OUT_RTOL = 1e-2
STATE_REL_FROB = 1e-3
DECODE_STATE_ATOL = 1e-4
PREFILL_STATE_ATOL = 5e-4


def to_dev(x, device="cuda"):
    """Move every tensor field of a workloads.*Inputs to `device` (copy of the dataclass)."""
    import dataclasses
    vals = {f.name: getattr(x, f.name) for f in dataclasses.fields(x)}
    vals = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in vals.items()}
    return type(x)(**vals)


def assert_out_close(got, ref, what=""):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    bad = (got - ref).abs() > OUT_ATOL + OUT_RTOL * ref.abs()
    assert not bad.any(), f"{what}: {int(bad.sum())} output elements out of tolerance, " \
        f"max abs err {(got - ref).abs().max().item():.3e}"


def state_errors(got, ref):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    d = got - ref
    return d.abs().max().item(), (d.norm() / ref.norm().clamp_min(1e-30)).item()


def assert_state_close(got, ref, atol, what=""):
    err, rel = state_errors(got, ref)
    assert rel <= STATE_REL_FROB and err <= atol, f"{what}: state max-abs {err:.3e} " \
        f"(atol {atol}), rel-frob {rel:.3e} (tol {STATE_REL_FROB})"
