"""The measurement arithmetic of bench.py, on the CPU: FLOP per token, the roofline of the dominant
kernel (live in-step duration preferred over the alone-timing) and the peak source."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # the module only defines functions; main() runs under __main__
    return mod


def test_flop_per_token_of_the_26m_model(bench):
    # 6 * (L * (4 d^2 + 2 d F) + V d) + 6 * L * S * d for V 6400, d 512, L 6, F 2048, S 2048
    assert bench.flop_per_token(6400, 512, 6, 2048, 2048) == 170_655_744


def _breakdown():
    return {
        "attention_bwd": {"ms": 0.32, "per_step": 6, "work": 137.4e9, "kind": "tensor"},
        "gemm_fwd_ff1": {"ms": 0.064, "per_step": 6, "work": 68.7e9, "kind": "tensor"},
        "adamw": {"ms": 0.11, "per_step": 1, "work": 765e6, "kind": "hbm"},
    }


def test_roofline_prefers_the_in_step_duration(bench):
    pk = {"hbm_gbs": 6455.6, "bf16_tflops": 1656.9, "source": "measured"}
    r = bench.roofline_of(_breakdown(), pk, {"attention_bwd": 0.35, "attention_fwd": 0.15})
    assert r["kernel"] == "attention_bwd" and r["bound"] == "tensor" and r["unit"] == "TFLOP/s"
    assert r["ms_per_launch"] == 0.35 and r["ms_per_launch_alone"] == 0.32
    assert r["achieved"] == pytest.approx(137.4e9 / 0.35e-3 / 1e12, rel=1e-3)
    assert r["frac"] == pytest.approx(r["achieved"] / 1656.9, rel=1e-3)
    assert "event nodes" in r["timing"]
    total = 0.32 * 6 + 0.064 * 6 + 0.11
    assert r["share_of_kernel_time"] == pytest.approx(0.32 * 6 / total, abs=1e-4)


def test_roofline_falls_back_to_the_alone_timing(bench):
    pk = {"hbm_gbs": 6455.6, "bf16_tflops": 1656.9, "source": "measured"}
    r = bench.roofline_of(_breakdown(), pk, None)
    assert r["ms_per_launch"] == 0.32 and "alone" in r["timing"]
    assert r["achieved"] == pytest.approx(137.4e9 / 0.32e-3 / 1e12, rel=1e-3)


def test_peaks_come_from_the_measured_file(bench):
    p = bench.peaks()
    if os.path.exists(os.path.join(ROOT, "MEASURED_PEAKS.json")):
        assert p["source"] == "measured" and p["bf16_tflops"] > 1000 and p["hbm_gbs"] > 5000
    else:
        assert p["source"] == "fallback"


def test_result_line_is_alone_on_stdout():
    """Output that a native library writes to file descriptor 1 after claim_stdout() lands on
    standard error; standard output holds the result line only."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import os, bench; bench.claim_stdout(); os.write(1, b'NCCL version x\\n'); print('chatter'); "
            "bench.emit({'metric': 'm', 'value': 1.0})")
    r = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.splitlines() == ['{"metric": "m", "value": 1.0}']
    assert "NCCL version x" in r.stderr and "chatter" in r.stderr
