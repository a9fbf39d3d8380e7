"""bench.py host logic on the CPU: the clock sampler against a fake NVML module,
the clock summary and the JSON contract's throttle-reason names."""
import os
import sys
import time
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _fake_nvml(reasons_seq, uuid="GPU-1234"):
    """NVML stand-in: one GPU with the given UUID; clock-event reasons come from
    `reasons_seq` in order (the last value repeats). Every call is recorded."""
    calls = []
    state = {"i": 0}
    m = types.SimpleNamespace(NVML_CLOCK_SM=1, calls=calls)

    def rec(name, fn):
        def f(*a):
            calls.append(name)
            return fn(*a)
        setattr(m, name, f)

    def by_uuid(u):
        if u != uuid:
            raise RuntimeError("not found")
        return "h0"

    def reasons(h):
        v = reasons_seq[min(state["i"], len(reasons_seq) - 1)]
        state["i"] += 1
        return v

    rec("nvmlInit", lambda: None)
    rec("nvmlShutdown", lambda: None)
    rec("nvmlDeviceGetHandleByUUID", by_uuid)
    rec("nvmlDeviceGetHandleByPciBusId", lambda b: (_ for _ in ()).throw(RuntimeError("no bus")))
    rec("nvmlDeviceGetClockInfo", lambda h, c: 1890)
    rec("nvmlDeviceGetMaxClockInfo", lambda h, c: 1965)
    rec("nvmlDeviceGetPowerUsage", lambda h: 812_000)
    rec("nvmlDeviceGetCurrentClocksEventReasons", reasons)
    return m


def test_nvml_sampler_collects_rows_during_a_short_region():
    nvml = _fake_nvml([0x0, 0x4])
    s = bench.ClockSampler(3, uuid="GPU-1234", nvml=nvml)
    s.start()
    time.sleep(0.15)
    out = s.stop()
    assert out["source"] == "nvml"
    rows = out["rows"]
    assert len(rows) >= 3  # start + periodic + stop samples
    assert all(r[0] == "3" and r[1] == "1890" and r[2] == "1965" for r in rows)
    summary = bench.summarize_clocks(rows)
    assert summary["sm_mhz"] == 1890.0 and summary["sm_max_mhz"] == 1965.0
    assert summary["reasons"] == ["sw_power_cap"] and summary["samples"] == len(rows)
    # read-only queries only: nothing that sets clocks, limits or modes
    assert not [c for c in nvml.calls if "Set" in c or "Reset" in c]


def test_sampler_maps_each_reason_bit():
    nvml = _fake_nvml([0x8 | 0x40 | 0x20])
    s = bench.ClockSampler(0, uuid="GPU-1234", nvml=nvml)
    s.start()
    out = s.stop()
    summary = bench.summarize_clocks(out["rows"])
    assert summary["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_sampler_falls_back_when_the_gpu_is_not_found():
    nvml = _fake_nvml([0], uuid="GPU-other")
    s = bench.ClockSampler(0, uuid="GPU-1234", bus_id="00000000:18:00.0", nvml=nvml)
    assert not s._open_nvml()


def test_summary_of_no_samples_is_explicit():
    assert bench.summarize_clocks([]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}


def test_workload_layouts_fit_their_models():
    import types as _t

    from heiretsu_b200.config import GPTConfig
    from heiretsu_b200.models.fused import fused_supported
    from heiretsu_b200.trainer import build_argparser

    for name, w in bench.WORKLOADS.items():
        for n in (1, 2, 4, 8):
            dp, ep, tp, pp = layout = w.layout(n)
            assert dp * ep * tp * pp == n, (name, n)
            m = w.model
            assert m["n_head"] % tp == 0 and m["n_embed"] % tp == 0 and pp <= m["n_layer"]
            if ep > 1:
                assert m["num_experts"] % ep == 0
            args = build_argparser().parse_args(bench.train_flags(w, layout))
            assert (args.dp, args.ep, args.tp, args.pp) == layout
            assert args.batch_size == w.micro and args.grad_accum_steps == w.accum
            assert args.num_experts == m.get("num_experts", args.num_experts)
            cfg = GPTConfig(**w.model_kwargs(), dropout=0.0)
            ok, why = fused_supported(cfg, _t.SimpleNamespace(dp=dp, ep=ep, tp=tp, pp=pp))
            assert ok, (name, n, why)
    assert bench.parallelism_name(bench.WORKLOADS["gpt2s_dp"].layout(8)) == "dp8"
    assert bench.parallelism_name(bench.WORKLOADS["moe_dp2_ep2_tp2"].layout(8)) == "dp2_ep2_tp2"


def test_reference_config_accepts_every_workload():
    import pytest

    from oracle import load_reference, ref_dir

    if ref_dir() is None:
        pytest.skip("reference implementation not found")
    ref = load_reference()
    for w in bench.WORKLOADS.values():
        cfg = ref.gpt_model.GPTConfig(**w.model_kwargs(), dropout=0.0)
        assert cfg.n_layer == w.model["n_layer"] and cfg.num_experts == w.model.get("num_experts", 0)


def test_scalar_reader_returns_every_value_in_order():
    import torch

    from heiretsu_b200.trainer import ScalarReader

    r = ScalarReader(depth=2)
    out = []
    for i in range(5):
        r.push(torch.tensor(float(i)))
        if len(r) > 1:
            out.append(r.pop())
    while len(r):
        out.append(r.pop())
    assert out == [0.0, 1.0, 2.0, 3.0, 4.0]
    r.push(torch.tensor(1.0))
    r.push(torch.tensor(2.0))
    import pytest
    with pytest.raises(RuntimeError):
        r.push(torch.tensor(3.0))


def test_cpu_sanity_config_both_arms():
    """bench.py --config cpu_sanity: both implementations print the JSON line, train the same
    model on the same batches and reach the same loss (fp32, one process)."""
    import json
    import subprocess

    from oracle import have_reference

    out = {}
    for impl in ("ours", "reference"):
        r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--config", "cpu_sanity", "--impl", impl,
                            "--steps", "2", "--warmup", "1"], capture_output=True, text=True, timeout=600,
                           env=dict(os.environ, OMP_NUM_THREADS="2"))
        assert r.returncode == 0, r.stderr[-3000:]
        out[impl] = json.loads(r.stdout.strip().splitlines()[-1])
    o = out["ours"]
    assert o["unit"] == "tokens/s" and o["value"] > 0 and o["dtype"] == "fp32" and o["n_gpus"] == 0
    assert o["config"]["seq_len"] == 256 and o["config"]["global_batch"] == 8
    ref = out["reference"]
    if "unavailable" in ref:
        assert not have_reference()
        return
    assert abs(o["final_loss"] - ref["final_loss"]) < 1e-4
