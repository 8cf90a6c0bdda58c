"""Shared helpers for the parity tests (tolerances written out here)."""
import numpy as np

# Tolerances of the parity contract (fp32 kernels against the oracle):
IMAGE_ATOL = 1e-4          # rendered colour / alpha, absolute
GRAD_RTOL = 1e-3           # parameter gradients, relative (per-tensor L2 and per element)
GRAD_FLOOR = 1e-4          # per-element absolute floor, as a fraction of the tensor's max |ref|
ADAM_RTOL = 1e-6           # Adam-updated parameters, relative


def assert_image_close(got, ref, atol=IMAGE_ATOL, what="image"):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    err = np.abs(got - ref).max() if got.size else 0.0
    assert err <= atol, f"{what}: max abs error {err:.3g} > {atol}"
    return err


def assert_grad_close(got, ref, rtol=GRAD_RTOL, floor=GRAD_FLOOR, what="grad"):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    nref = np.linalg.norm(ref)
    if nref == 0:
        assert np.abs(got).max() <= 1e-12, what
        return 0.0
    rel = np.linalg.norm(got - ref) / nref
    assert rel <= rtol, f"{what}: relative L2 error {rel:.3g} > {rtol}"
    atol = floor * np.abs(ref).max()
    bad = np.abs(got - ref) > rtol * np.abs(ref) + atol
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements out of tolerance; worst "
                           f"{np.abs(got - ref)[bad].max():.3g} at ref {ref[bad][np.argmax(np.abs(got - ref)[bad])]:.3g}")
    return rel


def assert_adam_close(got, ref, rtol=ADAM_RTOL, what="adam"):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=1e-30, err_msg=what)


def assert_adam_update_close(got, ref, before, rtol=ADAM_RTOL, what="adam"):
    """Adam-updated parameters whose step was formed with the hardware
    approximate square root and reciprocal: within ``rtol`` of the parameter
    plus ``rtol`` of the step the oracle took (|before - ref|), so that a
    parameter the step moves close to zero is judged against the step."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    before = np.asarray(before, np.float64)
    tol = rtol * (np.abs(ref) + np.abs(before - ref))
    err = np.abs(got - ref)
    bad = ~(err <= tol)
    assert not bad.any(), (f"{what}: {int(bad.sum())} elements out of tolerance; worst excess "
                           f"{(err - tol)[bad].max():.3g}")

