"""Circle's population depth law: the maximum-entropy distribution on ``[minimum, maximum]`` with a
given mean, ``p(d) ~ exp(tilt * d)``.  The tilt is found by bisection (the mean is increasing in the
tilt); the law is a fixed prior, never a per-sequence quota.
Behaviour: ``nexttransformer/models/native/depth.py:7-33``.
"""
from functools import lru_cache
import math


def _tilted(depths, centre, tilt):
    z = [tilt * (d - centre) for d in depths]
    top = max(z)
    w = [math.exp(v - top) for v in z]
    s = sum(w)
    return [v / s for v in w]


@lru_cache(maxsize=64)
def depth_reference(minimum, maximum, mean):
    """(probabilities of depths minimum..maximum, survival P(D >= s) for s = 1..maximum)."""
    if not minimum < mean < maximum:
        raise ValueError("Circle target must be strictly inside its depth range")
    depths = list(range(minimum, maximum + 1))
    lo, hi = -64.0, 64.0
    for _ in range(90):
        mid = 0.5 * (lo + hi)
        p = _tilted(depths, mean, mid)
        if sum(d * q for d, q in zip(depths, p)) < mean:
            lo = mid
        else:
            hi = mid
    probs = _tilted(depths, mean, 0.5 * (lo + hi))
    survival = tuple(1.0 if s <= minimum else sum(probs[s - minimum:]) for s in range(1, maximum + 1))
    return tuple(probs), survival
