"""Shared helpers for the GPU tests: the CUDA backend registered as
tensor.CUDA(0) in the oracle's restated tensor package, so the same op
sequence runs on both devices (as tensor/device_mps_test.go does for MPS)."""
import numpy as np

from oracle import gotensor_ref as T

_backend = None


def cuda_backend():
    global _backend
    if _backend is None:
        from gotensor.backend import CudaBackend
        _backend = CudaBackend(0)
        T.register_backend(T.CUDA_TYPE, lambda index: _backend if index == 0 else CudaBackend(index))
    return _backend


def cpu_backend():
    return T.backend_for(T.CPU)


def assert_close(got, want, tol, what=""):
    got, want = np.asarray(got, dtype=np.float64), np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    with np.errstate(invalid="ignore"):
        ok = np.abs(got - want) <= tol * np.maximum(1.0, np.abs(want))
    bad = ~(ok | (got == want) | (np.isnan(got) & np.isnan(want)))
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.size} differ; first at {i}: got {got.flat[i]!r}, "
                             f"want {want.flat[i]!r} (tol {tol})")


def assert_bits(got, want, what=""):
    got, want = np.asarray(got), np.asarray(want)
    assert got.dtype == want.dtype and got.shape == want.shape, (what, got.dtype, want.dtype, got.shape, want.shape)
    if got.size == 0:
        return
    same = (got.view(np.uint8).reshape(got.size, -1) == want.view(np.uint8).reshape(want.size, -1)).all(axis=1)
    same |= np.isnan(got.astype(np.float64)) & np.isnan(want.astype(np.float64))
    if not same.all():
        i = int(np.argmin(same))
        raise AssertionError(f"{what}: {int((~same).sum())} of {same.size} differ bitwise; first at {i}: "
                             f"got {got.flat[i]!r}, want {want.flat[i]!r}")
