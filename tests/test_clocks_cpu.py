"""The benchmark's nvidia-smi clock sampler: parsing, GPU selection, the "under load" median and
the throttle reasons (a stand-in process replaces nvidia-smi)."""
from pan2_b200.utils.clocks import ClockSampler

ROWS = (
    "0, GPU-aaa, 1500, 1965, 900.5, 0x4, Not Active, Not Active, Not Active, Active\n"
    "0, GPU-aaa, 1600, 1965, 950.0, 0x4, Not Active, Not Active, Not Active, Active\n"
    "1, GPU-bbb, 1965, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active\n"
    "2, GPU-ccc, 700, 1965, 990.0, 0x40, Not Active, Active, Not Active, Not Active\n"
    "garbage line\n"
)


class _Proc:
    def terminate(self):
        pass

    def kill(self):
        pass

    def communicate(self, timeout=None):
        return ROWS, None


def _stop(gpus=None):
    s = ClockSampler()
    s.proc = _Proc()
    return s.stop(gpus=gpus)


def test_selected_gpus_under_load():
    r = _stop(gpus=[0, 1])
    assert r["samples"] == 3 and r["sm_max_mhz"] == 1965.0
    # samples drawing at least half the peak power: GPU 0's two rows
    assert r["sm_mhz"] == 1550.0 and r["reasons"] == ["sw_power_cap"]


def test_reasons_of_every_sampled_gpu():
    r = _stop(gpus=[2])
    assert r["reasons"] == ["hw_thermal_slowdown"] and r["sm_mhz"] == 700.0


def test_no_sampler_process():
    assert ClockSampler().stop()["samples"] == 0
