"""The C++ host harnesses (benchmark_b200/harness) mirror the reference's
bench CLIs: 0.attention/main.cu (exit codes 0 ok, 1 failure, 2 bad
arguments, 77 no usable GPU) and 5.GEMM/gemm256_tma_tcgen05_bench.cu.
CPU tests check argument handling; GPU tests run their validation modes."""
import csv
import subprocess
from pathlib import Path

import pytest

BIN = Path(__file__).resolve().parents[1] / "benchmark_b200" / "bin"
ATTN = BIN / "attention_bench"
GEMM = BIN / "gemm_bench"
CUBLAS = BIN / "cublas_bench"
PROBE = BIN / "peak_probe"


def _run(exe, *args, timeout=600):
    if not exe.exists():
        pytest.fail(f"{exe.name} is not built (python -m benchmark_b200.build)")
    return subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("exe", [ATTN, GEMM, CUBLAS, PROBE])
def test_help_exits_zero(exe):
    r = _run(exe, "--help")
    assert r.returncode == 0 and "--" in r.stdout


@pytest.mark.parametrize("args", [["--bogus"], ["--d", "96"], ["--iters", "0"],
                                  ["--blocks", "-1"], ["--pattern", "zebra"]])
def test_attention_bad_arguments_exit_two(args):
    assert _run(ATTN, *args).returncode == 2


@pytest.mark.parametrize("args", [["--bogus"], ["--sizes", "100"], ["--impl", "x"],
                                  ["--validate-pattern", "zebra"], ["--b-layout", "diag"]])
def test_gemm_bad_arguments_exit_two(args):
    assert _run(GEMM, *args).returncode == 2


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["--validate-suite", "--scalar-validate-suite"])
def test_attention_validate_suite(mode):
    r = _run(ATTN, mode)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.gpu
def test_attention_benchmark_csv(tmp_path):
    out = tmp_path / "attn.csv"
    r = _run(ATTN, "--blocks", "8", "--k-tiles", "4", "--warmup", "1", "--iters", "2",
             "--csv", str(out))
    assert r.returncode == 0, r.stderr
    rows = list(csv.reader(out.open()))
    assert len(rows) == 2
    # run.py reads the tail of each row: TFLOP/s, status, cuda_error, notes.
    assert rows[1][-3] == "ok" and float(rows[1][-4]) > 0


@pytest.mark.gpu
@pytest.mark.parametrize("impl", ["tcgen05", "cublas"])
@pytest.mark.parametrize("layout", ["col", "row"])
@pytest.mark.parametrize("pattern,size", [("pattern", "256"), ("ones", "512"),
                                          ("pattern", "1024")])
def test_gemm_validate(impl, layout, pattern, size):
    r = _run(GEMM, "--validate", "--validate-size", size, "--validate-pattern", pattern,
             "--impl", impl, "--b-layout", layout)
    assert r.returncode == 0 and "status=ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_gemm_benchmark_csv(tmp_path):
    out = tmp_path / "gemm.csv"
    r = _run(GEMM, "--sizes", "1024,2048", "--warmup", "1", "--iters", "2", "--csv", str(out))
    assert r.returncode == 0, r.stdout + r.stderr
    rows = list(csv.DictReader(out.open()))
    assert [int(x["size"]) for x in rows] == [1024, 2048]
    assert all(x["status"] == "ok" and float(x["event_TFLOPS"]) > 0 for x in rows)


@pytest.mark.parametrize("args", [["--mode", "int8"], ["--m", "0"], ["--repeat", "0"],
                                  ["--bogus"]])
def test_cublas_bad_arguments_exit_two(args):
    assert _run(CUBLAS, *args).returncode == 2


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["fp16", "bf16", "tf32", "fp32"])
def test_cublas_bench_modes_run(mode):
    r = _run(CUBLAS, "--m", "1024", "--n", "512", "--k", "768", "--repeat", "3", "--warmup", "1",
             "--mode", mode)
    assert r.returncode == 0, r.stdout + r.stderr
    csv_line = [ln for ln in r.stdout.splitlines() if ln.startswith("csv,")]
    assert len(csv_line) == 1 and csv_line[0].split(",")[1] == mode
    assert float(csv_line[0].split(",")[8]) > 0


def test_peak_probe_bad_arguments_exit_two():
    assert _run(PROBE, "--probe", "fp8").returncode == 2
    assert _run(PROBE, "--iters", "1").returncode == 2


@pytest.mark.gpu
def test_peak_probe_all_runs_with_plausible_rates():
    r = _run(PROBE, "--probe", "all", "--iters", "2048")
    assert r.returncode == 0, r.stdout + r.stderr
    vals = {}
    for ln in r.stdout.splitlines():
        if ln.startswith("probe="):
            kv = dict(x.split("=", 1) for x in ln.split() if "=" in x)
            vals[kv["probe"]] = float(kv["value"])
    base = {"mma_m128_n256_ss_1acc", "mma_m128_n128_ss_1acc", "mma_m128_n128_ts_1acc",
            "mma_m128_n128_ss_2acc", "mma_m128_n128_ts_2acc", "mma_m128_n128_ss_ts_2acc"}
    assert set(vals) == base | {b + "_ones" for b in base} | {
        "mma_pair_m256_n128_ss", "mma_pair_m256_n256_ss",
        "issue_m128_n128_ss_same_operands", "issue_m128_n128_ss_distinct_operands",
        "issue_m128_n128_ss_same_operands_zeros", "issue_m128_n128_ss_distinct_operands_zeros",
        "tmem_ld_32x32b_x32", "tmem_st_32x32b_x32", "mufu_ex2_f32", "hbm_copy_1GiB"} | {
        "tile_issue_d128_" + m for m in ("mma_only", "commits", "commits_waits",
                                         "two_issuers_commits_waits", "two_issuers_mma_only")} | {
        "softmax_" + m for m in ("ex2", "ex2_cvt", "cvt", "ex2_intpack", "pair_cvt",
                                 "pair_intpack", "ex2_bf16x2", "ex2_f16x2", "pair_cvt_1warp")}
    assert vals["mma_m128_n256_ss_1acc"] > 500  # TFLOP/s
    assert vals["hbm_copy_1GiB"] > 1000        # GB/s
    assert all(v > 0 for v in vals.values())
