"""MetricAccumulator / DistributedMetricAccumulator (reference: mvp_engine/utils/metrics.py:16-295)."""

import pytest
import torch


def test_local_reducers():
    from mvp_engine.utils.metrics import MetricAccumulator

    acc = MetricAccumulator()
    for name, red in (("s", "sum"), ("m", "mean"), ("x", "max"), ("l", "last")):
        acc.register(name, red)
    with pytest.raises(ValueError):
        acc.register("s", "sum")
    for v in (1.0, torch.tensor(5.0), 3, None):
        acc.update(s=v, m=v, x=v, l=v)
    assert acc.finalize() == {"s": 9.0, "m": 3.0, "x": 5.0, "l": 3.0}
    assert float(acc.get("s")) == 9.0
    with pytest.raises(KeyError):
        acc.update(nope=1.0)
    acc.reset()
    assert acc.finalize() == {}
    acc.update(m=True)
    assert acc.finalize() == {"m": 1.0}
    acc.update(s=torch.ones(2))
    with pytest.raises(ValueError):
        acc.finalize()


def test_distributed_metric_single_process():
    from mvp_engine.utils.metrics import DistributedMetricAccumulator

    acc = DistributedMetricAccumulator(torch.device("cpu"))
    acc.register("loss", accumulate="avg", reduce="avg")
    acc.register("tokens", accumulate="add", reduce="sum")
    acc.register("peak", accumulate="max", reduce="max")
    acc.register("lr", accumulate="last", reduce="none")
    with pytest.raises(ValueError):
        acc.register("bad", accumulate="median")
    acc.update(loss=2.0, tokens=10, peak=3.0, lr=1e-3)
    acc.update(loss=4.0, tokens=6, peak=1.0, lr=2e-3)
    assert acc.loss.local_value == 3.0 and acc.tokens.local_value == 16.0
    with pytest.raises(RuntimeError):
        _ = acc.loss.global_value
    acc.reduce_all()
    assert acc.loss.global_value == 3.0 and acc.peak.global_value == 3.0
    assert abs(acc.lr.global_value - 2e-3) < 1e-9
    acc.reset()
    with pytest.raises(RuntimeError):
        _ = acc.loss.local_value
    with pytest.raises(AttributeError):
        _ = acc.missing


def _ranks(rank, world, port):
    import torch.distributed as dist

    from mvp_engine.testing.utils import distributed_env
    from mvp_engine.utils.metrics import DistributedMetricAccumulator

    with distributed_env(rank=rank, world_size=world, local_rank=rank, master_port=port):
        dist.init_process_group("gloo")
        acc = DistributedMetricAccumulator(torch.device("cpu"))
        acc.register("loss", accumulate="mean", reduce="mean")
        acc.register("tokens", accumulate="sum", reduce="sum")
        acc.register("peak", accumulate="max", reduce="max")
        acc.register("mine", accumulate="last", reduce="none")
        for k in range(rank + 1):  # rank r makes r + 1 updates
            acc.update(loss=float(rank * 10 + k), tokens=100, peak=float(rank), mine=float(rank))
        acc.reduce_all()
        return {n: getattr(acc, n).global_value for n in ("loss", "tokens", "peak", "mine")}


def test_distributed_metric_gloo_world2():
    from mvp_engine.testing import spawn_workers

    r0, r1 = spawn_workers(_ranks, 2, timeout=120)
    # rank 0: loss mean 0, 100 tokens; rank 1: loss mean 10.5, 200 tokens
    for r in (r0, r1):
        assert r["loss"] == pytest.approx(5.25) and r["tokens"] == 300.0 and r["peak"] == 1.0
    assert r0["mine"] == 0.0 and r1["mine"] == 1.0


def test_mfu_kit_formula_and_peaks(monkeypatch):
    from mvp_engine.kit import MFUKit

    kit = MFUKit()
    assert kit.normalize_device_name("NVIDIA B200") == "NVIDIA B200"
    assert kit.normalize_device_name("NVIDIA H100 80GB HBM3") == "NVIDIA H100 SXM"
    assert kit.normalize_device_name("Some GPU") == "Some GPU" and kit.normalize_device_name(" ") is None
    assert kit.resolve_peak_tflops(device_type="cpu", precision="bf16", configured_device_name="b200") == \
        ("NVIDIA B200", 2250.0)
    assert kit.resolve_peak_tflops(device_type="cpu", precision="bf16") == (None, None)
    kit.accumulate_microbatch(model_flops=1.0e15)
    kit.accumulate_microbatch(model_flops=1.25e15)
    log = kit.build_log(device_type="cpu", precision="bf16", step_time_seconds=2.0, configured_device_name="B200")
    assert log == {"perf/mfu": pytest.approx(2.25e15 / 2.0 / 2250e12)}
    assert kit.accumulated_model_flops == 0.0  # the window was consumed
    assert kit.build_log(model_flops_per_step=1e12, device_type="cpu", precision="int3", step_time_seconds=1.0,
                         configured_device_name="B200") == {}
    monkeypatch.setenv("MVP_PEAK_TFLOPS", "1000")
    assert kit.build_log(model_flops_per_step=1e15, device_type="cpu", precision="bf16",
                         step_time_seconds=1.0) == {"perf/mfu": pytest.approx(1.0)}
    with pytest.raises(ValueError):
        kit.calculate_mfu(model_flops_per_step=1.0, step_time_seconds=0.0, device_peak_tflops=1.0, world_size=1)
