"""SWIFT skip patterns (CPU): a contiguous middle block of round(ratio * L)
layers, the first two and last two kept, candidates at different starts with
the centred one first; the calibrator names the best-accepting pattern."""
from swarmllm_b200.engine.swift import SkipCalibrator, skip_patterns


def test_skip_patterns():
    ps = skip_patterns(20, 0.45)
    assert 2 <= len(ps) <= 5
    for m in ps:
        assert sum(m) == 9 and not any(m[:2]) and not any(m[-2:])
        idx = [i for i, s in enumerate(m) if s]
        assert idx == list(range(idx[0], idx[0] + 9))      # one contiguous block
    starts = [m.index(True) for m in ps]
    assert starts[0] == 2 + (20 - 4 - 9) // 2 and len(set(starts)) == len(starts)
    assert skip_patterns(4, 0.5) == [[False] * 4]           # too small to skip
    assert sum(skip_patterns(10, 0.99)[0]) == 6              # outer layers always kept


def test_calibrator():
    c = SkipCalibrator(skip_patterns(12, 0.4))
    c.record(0, 3, 10)
    c.record(1, 7, 10)
    assert c.best() == 1
