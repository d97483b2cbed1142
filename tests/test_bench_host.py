"""Host logic of bench.py (no GPU): the workloads of the BASELINE configs,
the byte counts the rooflines divide by, the by-tensor balance across ranks,
the ncu traffic figure each config quotes, and the clock sampler, which is
driven here by a stand-in NVML module (it only reads clocks)."""
import collections
import sys
import time
import types

import bench


def _total(config):
    return sum(bench.numel(s) for _, s in bench.CONFIGS[config]["shapes"]())


def test_workload_sizes():
    # Llama-3-8B (291 tensors), Llama-3-70B, GPT-2 block
    # and 124M (wte tied to the head), the 2^30 + 37 flat tensor
    assert len(bench.CONFIGS["llama3-8b"]["shapes"]()) == 291
    assert _total("llama3-8b") == 8_030_261_248
    assert _total("llama3-70b") == 70_553_706_496
    assert _total("gpt2-block") == 7_087_872
    assert _total("gpt2-124m") == 124_439_808
    assert _total("flat-vonly") == (1 << 30) + 37


def test_algorithmic_bytes_per_param():
    n = 1 << 24
    kw8, kw70 = bench.CONFIGS["llama3-8b"]["kw"], bench.CONFIGS["llama3-70b"]["kw"]
    # pass 1 and the single-touch step, fp32 4-bit + CoState and bf16 3-bit + CoState
    assert bench.pass1_bytes(n, kw8, 4) / n == 14.2421875
    assert bench.step_bytes(n, kw8, 4) / n == 14.421875
    assert bench.pass1_bytes(n, kw70, 2) / n == 8.2421875
    assert bench.step_bytes(n, kw70, 2) / n == 8.421875
    # a tensor below min_m_compress_elements keeps fp32 exp_avg; its shard of a
    # split tensor decides by the whole tensor
    assert bench.kind_of(4095, kw8) == (False, True)
    assert bench.kind_of(4095, kw8, n_policy=1 << 20) == (True, True)


def test_by_tensor_balance():
    shapes = bench.CONFIGS["llama3-8b"]["shapes"]()
    for world in (2, 4, 8):
        owner = bench.lpt_assign(shapes, world)
        load = collections.Counter()
        for i, (_, s) in enumerate(shapes):
            load[owner[i]] += bench.numel(s)
        assert len(load) == world
        assert max(load.values()) / (sum(load.values()) / world) < 1.01


def test_traffic_figure_per_kernel_kind():
    fp32 = bench.profiled_traffic("llama3-8b")
    bf16 = bench.profiled_traffic("llama3-70b")
    assert 13.5 < fp32 < 14.5 and 8.0 < bf16 < 8.6
    assert bench.profiled_traffic("gpt2-124m") == fp32
    assert bench.profiled_traffic("flat-vonly") is None  # no capture of that kernel kind


def test_clock_sampler_reads_nvml(monkeypatch):
    fake = types.ModuleType("pynvml")
    fake.NVML_CLOCK_SM = 1
    clocks = iter([1965, 1840, 1830] + [1835] * 1000)
    fake.nvmlInit = lambda: None
    fake.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    fake.nvmlDeviceGetClockInfo = lambda h, kind: next(clocks)
    fake.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: 0x4 | 0x1  # power cap, idle
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    c = bench.Clocks(0)
    c.start()
    time.sleep(0.05)
    out = c.stop()
    assert out["source"] == "nvml" and out["samples"] >= 2
    assert out["sm_max_mhz"] == 1965 and 1830 <= out["sm_mhz"] <= 1965
    assert out["reasons"] == ["sw_power_cap"]  # the idle bit is not a slowdown reason


def test_clock_sampler_flags_slowdowns(monkeypatch):
    fake = types.ModuleType("pynvml")
    fake.NVML_CLOCK_SM = 1
    fake.nvmlInit = lambda: None
    fake.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    fake.nvmlDeviceGetClockInfo = lambda h, kind: 1500
    fake.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    fake.nvmlDeviceGetCurrentClocksEventReasons = lambda h: 0x8 | 0x40 | 0x20
    monkeypatch.setitem(sys.modules, "pynvml", fake)
    c = bench.Clocks(0)
    c.start()
    out = c.stop()
    assert out["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]
    assert out["sm_mhz"] == 1500
