"""The per-SM speed table on the host (paged_attention.SmSpeeds): timing records
of large calls move the weights toward the measured speeds, records of another
call or with a CTA off its own SM are ignored, and the table stops learning
after SmSpeeds.SAMPLES records.  No GPU: the records are built here."""

from __future__ import annotations

import numpy as np

from llm_serving_runtime_b200.paged_attention import _TIMING_DTYPE, SmSpeeds


def _records(n, tag, speeds, weights, total=1_000_000, smids=None):
    rec = np.zeros(n, dtype=_TIMING_DTYPE)
    cost = np.maximum(1, (total * weights / weights.sum()).astype(np.int64))
    rec["cost"] = cost
    rec["t0"] = 1_000
    rec["t1"] = 1_000 + (cost / speeds).astype(np.int64)  # ns: cost units at each SM's speed
    rec["smid"] = np.arange(n) if smids is None else smids
    rec["tag"] = tag
    return rec.view(np.uint8)


def test_weights_follow_the_measured_speeds_then_stay():
    n = 148
    rng = np.random.default_rng(0)
    true = 1.0 + 0.1 * rng.standard_normal(n)
    t = SmSpeeds(n)
    assert t.learning and np.allclose(t.weights.numpy(), 1.0)
    for i in range(SmSpeeds.SAMPLES):
        tag = t.new_tag()
        assert t.absorb(tag, _records(n, tag, true, t.weights.numpy().astype(np.float64)))
    assert not t.learning
    w = t.weights.numpy()
    assert abs(w.mean() - 1.0) < 1e-5
    assert np.corrcoef(w, true)[0, 1] > 0.999
    # the slowest SM gets the smallest share
    assert int(np.argmin(w)) == int(np.argmin(true))


def test_foreign_or_displaced_records_are_ignored():
    n = 8
    t = SmSpeeds(n)
    ones = np.ones(n)
    tag = t.new_tag()
    assert not t.absorb(tag + 1, _records(n, tag, ones * 2, ones))  # another call's records
    # after a miss the next calls are not sampled for a while
    assert [t.want_sample() for _ in range(3)] == [False, False, True]
    smids = np.arange(n)
    smids[3] = 2  # two CTAs on one SM: no per-SM speed can be read off
    assert not t.absorb(tag, _records(n, tag, ones, ones, smids=smids))
    assert t.samples == 0 and np.allclose(t.weights.numpy(), 1.0)


def test_speeds_are_clamped_and_normalised():
    n = 4
    t = SmSpeeds(n)
    tag = t.new_tag()
    assert t.absorb(tag, _records(n, tag, np.array([10.0, 1.0, 1.0, 1.0]), np.ones(n)))
    w = t.weights.numpy()
    assert abs(w.mean() - 1.0) < 1e-5 and w.max() / w.min() < 1.6 / 0.6 + 1e-3


def test_devices_with_too_many_sms_keep_equal_shares():
    t = SmSpeeds(4096)
    assert t.n == 0 and not t.learning
