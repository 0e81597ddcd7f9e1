"""Pure-Python split-KV merge oracles (small cases only).

Test infrastructure, not product code.

* ``lse_merge`` follows the v7 / general merge kernels
  (``operators/mha/kernels/mha_paged_decode_ascend_v7.py:346-370``,
  ``mha_paged_decode_ascend_cube_general.py:253-278``): partials are normalised outputs with
  a natural-log LSE; a partial whose LSE is at or below ``-1e29`` (the ``-1e30`` empty-split
  sentinel, v7.py:312) carries weight zero; the denominator is clamped at ``1e-30``.
* ``raw_state_merge`` follows the raw (A, max, sum) format of
  ``mha_paged_decode_ascend_fused.py:553-556`` / ``mha_simd_merge.py:59-80`` and the
  reference's own oracle test ``tests/mha/test_raw_partial_state.py:7-26``: a state with
  ``sum <= 0`` is invalid and ignored.
"""
import math

EMPTY_LSE = -1.0e30
VALID_LSE = -1.0e29


def lse_merge(partials):
    """Merge ``[(output_vector, lse), ...]`` into one output vector (list of floats)."""
    if not partials:
        raise ValueError("at least one partial required")
    dim = len(partials[0][0])
    acc = [0.0] * dim
    maximum = EMPTY_LSE
    total = 0.0
    for values, lse in partials:
        peak = max(maximum, lse)
        old = math.exp(maximum - peak)
        new = math.exp(lse - peak) if lse > VALID_LSE else 0.0
        acc = [a * old + x * new for a, x in zip(acc, values)]
        total = total * old + new
        maximum = peak
    return [a / max(total, 1e-30) for a in acc]


def raw_state_merge(states):
    """Merge ``[(accumulator_vector, max, sum), ...]`` unnormalised states."""
    valid = [(a, m, s) for a, m, s in states if s > 0]
    if not valid:
        return [0.0] * len(states[0][0])
    peak = max(m for _, m, _ in valid)
    factors = [math.exp(m - peak) for _, m, _ in valid]
    denominator = sum(f * s for f, (_, _, s) in zip(factors, valid))
    dim = len(valid[0][0])
    return [sum(f * a[d] for f, (a, _, _) in zip(factors, valid)) / denominator for d in range(dim)]
