"""The benchmark CLI keeps the reference's flags (benchmarks/benchmark_forward.py:24-53)."""

import pytest

from flash_attention_2_lab_b200 import benchmark_forward


def test_cli_accepts_reference_flags():
    with pytest.raises(SystemExit) as e:
        benchmark_forward.main(["--help"])
    assert e.value.code == 0


@pytest.mark.gpu
def test_cli_runs_small_case(capsys):
    benchmark_forward.main(["--batch", "1", "--heads", "4", "--query-length", "256", "--causal",
                            "--dtype", "float16", "--samples", "3", "--iterations", "3",
                            "--warmup", "3", "--kernels", "sm100", "sdpa"])
    out = capsys.readouterr().out
    assert "sm100" in out and "TFLOPS" in out and "sdpa / sm100" in out


@pytest.mark.gpu
def test_cli_sustained_mode(capsys):
    benchmark_forward.main(["--batch", "1", "--heads", "8", "--query-length", "1024",
                            "--kernels", "sm100", "--sustained", "1"])
    out = capsys.readouterr().out
    assert "sustained" in out and "TFLOPS/GHz" in out


@pytest.mark.gpu
def test_cli_backward_mode(capsys):
    benchmark_forward.main(["--batch", "1", "--heads", "4", "--query-length", "512", "--causal",
                            "--samples", "2", "--iterations", "2", "--warmup", "2",
                            "--kernels", "sm100", "sdpa", "--backward"])
    out = capsys.readouterr().out
    assert "(backward)" in out and "sm100" in out


@pytest.mark.gpu
def test_cli_backward_sustained_mode(capsys):
    benchmark_forward.main(["--batch", "1", "--heads", "4", "--query-length", "1024",
                            "--kernels", "sm100", "--backward", "--sustained", "1"])
    out = capsys.readouterr().out
    assert "sustained" in out and "(backward)" in out and "TFLOPS/GHz" in out
