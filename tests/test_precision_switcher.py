"""DynamicPrecisionSwitcher: the reference's own test cases
(DynamicMultiPrecisionWireTests.cs:365-470) and the static selector."""
import pytest

from glacier.inference.distributed_b200 import DynamicPrecisionSwitcher, WirePrecisionMode as W


@pytest.mark.parametrize("batch", [32, 64, 128, 512, 2048])
def test_prefill_batch_at_least_32_selects_int8(batch):
    assert DynamicPrecisionSwitcher().select_precision(batch, 0, False) == W.INT8_Symmetric


@pytest.mark.parametrize("batch", [1, 8, 16, 31])
def test_prefill_batch_below_32_selects_fp16(batch):
    assert DynamicPrecisionSwitcher().select_precision(batch, 0, False) == W.FP16


def test_decode_selects_fp16_under_normal_latency():
    s = DynamicPrecisionSwitcher()
    s.update_measured_latency(0.45)
    assert s.select_precision(1, 50, True) == W.FP16


def test_deep_context_decode_keeps_fp16_under_congestion():
    s = DynamicPrecisionSwitcher()
    s.update_measured_latency(3.0)
    assert s.select_precision(1, 17000, True) == W.FP16
    assert s.select_precision(1, 16384, True) == W.INT8_Symmetric  # the boundary itself is not deep


def test_congestion_backs_off_to_int8():
    s = DynamicPrecisionSwitcher()
    s.update_measured_latency(3.5)
    assert s.select_precision(16, 100, False) == W.INT8_Symmetric
    assert s.select_precision(1, 100, True) == W.INT8_Symmetric


def test_ema_latency_convergence_and_first_sample():
    s = DynamicPrecisionSwitcher()
    assert s.current_ema_latency_ms == 0.5
    s.update_measured_latency(2.0)
    assert s.current_ema_latency_ms == 2.0  # the first sample sets it directly
    s.update_measured_latency(-1.0)  # ignored
    assert s.current_ema_latency_ms == 2.0
    for _ in range(20):
        s.update_measured_latency(1.0)
    assert abs(s.current_ema_latency_ms - 1.0) < 0.05


def test_forced_override_always_respected():
    s = DynamicPrecisionSwitcher(W.FP32)
    assert s.select_precision(512, 0, False) == W.FP32
    assert s.select_precision(1, 0, True) == W.FP32
    s.forced_precision = W.FP8_E4M3
    assert s.select_precision(1, 0, True) == W.FP8_E4M3


def test_switch_count_and_reset():
    s = DynamicPrecisionSwitcher()
    s.update_measured_latency(5.0)
    s.select_precision(64, 0, False)
    assert s.total_switches > 0
    s.reset()
    assert s.current_ema_latency_ms == 0.5
    assert s.total_switches == 0
    assert s.last_selected_precision == W.FP16


def test_override_rtt_and_static_selector():
    s = DynamicPrecisionSwitcher()
    assert s.select_precision(4, 0, False, override_rtt_ms=3.0) == W.INT8_Symmetric
    f = DynamicPrecisionSwitcher.select_optimal_wire_precision
    assert f(1, True, 9.0) == W.FP16
    assert f(8, False, 3.0) == W.INT8_Symmetric
    assert f(31, False, 0.1) == W.FP16 and f(32, False, 0.1) == W.INT8_Symmetric
    assert f(512, False, 0.1, W.FP32) == W.FP32
