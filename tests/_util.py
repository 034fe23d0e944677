"""Shared helpers of the parity tests: seeded inputs and the tolerance rule."""
from __future__ import annotations

import numpy as np

# North-star tolerance for every float output (loss, logits, activations,
# gradients): |x - ref| <= ATOL + RTOL * |ref|, ref = the fp32 CPU reference.
RTOL = 1e-4
ATOL = 1e-5


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal(r, shape, std=1.0):
    return (r.standard_normal(shape) * std).astype(np.float32)


def close_report(x, ref32, ref64=None, rtol=RTOL, atol=ATOL):
    """Elementwise tolerance check with float64 adjudication.

    An element passes if |x - ref32| <= atol + rtol*|ref32|.  An element that
    misses passes anyway when ``ref64`` is given and x is about as close to
    the float64 value as the fp32 reference itself is: the miss is then the
    reference's own rounding, which is the rule of the reference's
    tools/parity/precision_probe.py:91-96.  "About as close" is
    |x - f64| <= |ref32 - f64| + atol + rtol*|f64| + 3 * rms(ref32 - f64);
    the last term is the fp32 reference's typical error over the whole
    tensor, so two independent roundings of a cancelling sum are not
    compared element by element.
    Returns (ok, details dict).
    """
    x = np.asarray(x, np.float64)
    r = np.asarray(ref32, np.float64)
    err = np.abs(x - r)
    bad = err > atol + rtol * np.abs(r)
    n_bad_raw = int(bad.sum())
    if n_bad_raw and ref64 is not None:
        t = np.asarray(ref64, np.float64)
        own = np.abs(r - t)
        mine = np.abs(x - t)
        slack = 3.0 * float(np.sqrt(np.mean(own * own))) if own.size else 0.0
        bad = bad & (mine > own + atol + rtol * np.abs(t) + slack)
    info = {
        "max_abs": float(err.max()) if err.size else 0.0,
        "max_rel": float((err / (np.abs(r) + 1e-30)).max()) if err.size else 0.0,
        "n": int(err.size),
        "n_outside_tol": n_bad_raw,
        "n_fail_after_fp64": int(bad.sum()),
    }
    return not bad.any(), info


def assert_close(x, ref32, ref64=None, rtol=RTOL, atol=ATOL, what=""):
    ok, info = close_report(x, ref32, ref64, rtol, atol)
    assert ok, f"{what}: {info}"
    return info


def rel_l2(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(x - ref) / max(np.linalg.norm(ref), 1e-300))


def gpt_init(shapes, r, std=0.02, ln_noise=0.0):
    """Reference initialisation (see neuralsuite_b200.model.init_params) for a
    shape list from param_shapes()."""
    from neuralsuite_b200.model import GPTConfig, init_params

    V, C = shapes[0]
    block = shapes[1][0]
    L = (len(shapes) - 4) // 12
    return init_params(GPTConfig(V, block, L, 1, C), r, std, ln_noise)
