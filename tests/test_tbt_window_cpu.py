"""Token-weighted time-between-tokens window used by the avg_tbt_slo check."""
from deltaserve_vllm_b200.engine.ft.tbt_window import DecodeGapWindow


def test_token_weighted_mean_and_owed_gaps():
    w = DecodeGapWindow(window_s=10.0, idle_gap_s=1.0)
    w.note_step(0.00, 0, False)            # first step: no gap yet
    w.note_step(0.02, 4, True)             # 4 tokens waited 20 ms
    w.note_step(0.05, 0, True)             # no decode while running: 30 ms owed
    w.note_step(0.06, 2, True)             # 2 tokens waited 10 + 30 ms
    assert abs(w.mean(0.06) - (4 * 0.02 + 2 * 0.04) / 6) < 1e-12
    # a hypothetical next step of 15 ms with 3 decode rows
    assert abs(w.mean_with(0.06, 3, 0.015) - (4 * 0.02 + 2 * 0.04 + 3 * 0.015) / 9) < 1e-12


def test_idle_gap_and_window_expiry():
    w = DecodeGapWindow(window_s=1.0, idle_gap_s=0.5)
    w.note_step(0.0, 0, False)
    w.note_step(0.1, 2, True)
    w.note_step(0.2, 0, False)             # nothing running: nothing owed
    w.note_step(0.25, 1, True)
    assert abs(w.mean(0.25) - (2 * 0.1 + 0.05) / 3) < 1e-12
    w.note_step(5.0, 8, True)              # after an idle gap: not a token gap
    assert w.mean(5.0) is None             # the old steps left the 1 s window
    assert w.mean_with(5.0, 0, 0.01) == 0.0


def test_ring_overwrites_oldest():
    w = DecodeGapWindow(window_s=1e9, idle_gap_s=1.0, capacity=4)
    t = 0.0
    w.note_step(t, 0, False)
    for k in range(10):
        t += 0.01 * (k + 1)
        w.note_step(t, 1, True)
    # only the last 4 records remain: gaps 0.07, 0.08, 0.09, 0.10
    assert abs(w.mean(t) - 0.085) < 1e-12
