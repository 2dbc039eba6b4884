"""Helpers shared by the CPU and GPU tests."""

import hashlib

import numpy as np


def inputs_digest(arrays: dict) -> str:
    """Same digest as tests/golden/make_golden.py (detects generator drift)."""
    h = hashlib.sha256()
    for k in sorted(arrays):
        a = np.ascontiguousarray(arrays[k])
        h.update(k.encode())
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def regenerate(pkg, name: str, expected_sha: str | None = None):
    s = pkg.workloads.spec(name)
    x = pkg.workloads.host_inputs(s)
    if expected_sha is not None:
        got = inputs_digest({k: v for k, v in x.items() if isinstance(v, np.ndarray)})
        assert got == expected_sha, f"{name}: regenerated inputs differ from the golden inputs"
    return x, s


def model_shaped_inputs(pkg, expected_sha: str):
    return regenerate(pkg, "model_shaped", expected_sha)


def rel_err(actual, expected) -> float:
    """Normwise relative error max|a - e| / max|e|."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    return float(np.max(np.abs(a - e)) / max(np.max(np.abs(e)), 1e-30))


def assert_close(actual, expected, atol, rtol, label=""):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, f"{label}: shape {a.shape} != {e.shape}"
    bad = np.abs(a - e) > atol + rtol * np.abs(e)
    assert not bad.any(), (f"{label}: {int(bad.sum())} mismatches; max abs err "
                           f"{np.max(np.abs(a - e)):.3g}")
