"""Shared helpers of the parity tests: seeded inputs and the north-star tolerance."""
import numpy as np

# North-star tolerance for attention outputs (fp16 KV, fp32 accumulate), against the oracle fed
# the same fp16-rounded K/V: |got - ref| <= ATOL + RTOL * |ref| elementwise.
ATOL = 2e-3
RTOL = 1e-2


def normal(rng, *shape):
    return rng.standard_normal(shape).astype(np.float32)


def f16_round(a):
    """f32 -> fp16 (round to nearest even) -> f32, what the cache stores."""
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def assert_close(got, ref, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float32).ravel()
    ref = np.asarray(ref, np.float32).ravel()
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), (f"{what}: {int(bad.sum())}/{ref.size} outside tolerance, max abs err "
                           f"{err.max():.3g} at {int(err.argmax())}")


def bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))
