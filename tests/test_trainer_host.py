"""Learning-rate schedule and loss-scale state machine of the step driver
against train.py's formulas (train.py:31, 500, 617-624, 661-677), on the CPU."""
import math

from usaf_b200.trainer import LossScaler, lr_at


def test_lr_schedule():
    peak = 2e-4
    # 100 steps: warm-up max(1, int(100 * 0.05)) = 5 steps
    assert lr_at(1, 100, peak) == peak * 1 / 5
    assert lr_at(5, 100, peak) == peak
    lr_min = peak / 10
    for step in (6, 40, 77, 100):
        cos_lr = 0.5 * (1 + math.cos(math.pi * (step - 5) / (100 - 5)))
        assert lr_at(step, 100, peak) == lr_min + (peak - lr_min) * cos_lr
    assert abs(lr_at(100, 100, peak) - lr_min) < 1e-12
    # fewer than 20 steps: one warm-up step
    assert lr_at(1, 10, peak) == peak
    assert lr_at(2, 10, peak) < peak


def test_loss_scale_skip_and_growth():
    s = LossScaler()
    assert s.scale == 4096.0
    for expect in (2048.0, 1024.0, 512.0):
        s.update(False)
        assert s.scale == expect
    s = LossScaler(init=128.0)
    s.update(False)
    s.update(False)
    assert s.scale == 64.0          # floor
    s = LossScaler(init=1000.0, scale_up_every=3)
    s.update(True); s.update(True)
    assert s.scale == 1000.0
    s.update(True)
    assert s.scale == 2000.0
    s.update(False)                 # a skip halves but keeps the streak count
    assert s.scale == 1000.0 and s.good_streak == 3 and s.n_skipped == 1
    s.update(True); s.update(True)
    assert s.good_streak == 5 and s.scale == 1000.0
    s.update(True)
    assert s.scale == 2000.0
    s = LossScaler(init=65536.0, scale_up_every=1)
    s.update(True)
    assert s.scale == 65536.0       # cap
    st = s.state_dict()
    t = LossScaler()
    t.load_state_dict(st)
    assert t.scale == s.scale and t.good_streak == s.good_streak
