"""Learning-rate schedules: warmup endpoints, decay endpoints and shapes, floors, and the
device-scalar scheduler's state round trip."""
import math

import pytest
import torch

from pan2_b200.optim.lr import HostLambdaLR, make_lr_lambda


def test_warmup_then_cosine_to_floor():
    f = make_lr_lambda("cosine_decay", warmup_steps=5, decay_steps=11, max_steps=100,
                       warmup_start_ratio=0.2, decay_floor_ratio=0.05)
    assert f(0) == pytest.approx(0.2) and f(4) == pytest.approx(1.0)
    assert f(2) == pytest.approx(0.2 * 0.5 + 0.5)
    assert f(5) == pytest.approx(1.0)                       # decay starts at full rate
    assert f(10) == pytest.approx(0.05 + 0.95 * 0.5 * (1 + math.cos(math.pi * 0.5)))
    assert f(15) == pytest.approx(0.05) and f(1000) == pytest.approx(0.05)  # floor, held
    vals = [f(s) for s in range(5, 16)]
    assert all(a >= b for a, b in zip(vals, vals[1:]))


def test_linear_and_constant_schedules():
    lin = make_lr_lambda("linear_decay", 0, None, 11, 0.0, 0.1)  # decay over max_steps - warmup
    assert lin(0) == pytest.approx(1.0) and lin(10) == pytest.approx(0.1) and lin(5) == pytest.approx(0.55)
    const = make_lr_lambda("constant_with_warmup", 3, None, 50, 0.0, 0.3)
    assert const(0) == 0.0 and const(2) == 1.0 and const(40) == 1.0
    with pytest.raises(ValueError):
        make_lr_lambda("step", 1, None, 10, 0.0, 0.0)


def test_device_scalar_scheduler_state_round_trip():
    f = make_lr_lambda("cosine_decay", 2, 8, 20, 0.0, 0.1)
    t = torch.zeros(1)
    s = HostLambdaLR(1e-3, f, t)
    for _ in range(6):
        s.step()
    assert t.item() == pytest.approx(1e-3 * f(6))
    t2 = torch.zeros(1)
    s2 = HostLambdaLR(1e-3, f, t2)
    s2.load_state_dict(s.state_dict())
    assert t2.item() == pytest.approx(t.item()) and s2.get_last_lr() == s.get_last_lr()
