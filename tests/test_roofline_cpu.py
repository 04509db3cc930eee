"""The ncu CSV parser / roofline classifier (vla-kernels_b200/roofline.py) on
committed samples of real ncu exports (tests/golden/make_ncu_samples.py): the
wide --page raw form of an attention capture (B=512, 2 launches) and a launch
list in the long form. The classifier keeps the reference's thresholds
(bench/roofline.py:31-41)."""
import os

import pytest

import roofline

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
RAW = os.path.join(GOLDEN, "ncu_raw_sample.csv")
LAUNCHES = os.path.join(GOLDEN, "ncu_launches_sample.csv")


def test_wide_form_units_and_values():
    k = roofline.parse(RAW)
    assert len(k) == 2
    (kid, name), m = next(iter(k.items()))
    assert kid == "0" and "gqa_attention_sm100" in name
    assert m["duration_ns"] == pytest.approx(108992.0)
    assert m["dram_read_bytes"] == pytest.approx(240.137984e6)
    assert m["dram_write_bytes"] == pytest.approx(33.712896e6)
    assert m["tensor_pct"] == pytest.approx(24.633326)
    assert m["registers"] == 128


def test_roofline_figures_against_measured_peak():
    m = next(iter(roofline.parse(RAW).values()))
    algorithmic = 512 * 564480  # C3/C5 bytes per batch element x B
    r = roofline.roofline(m, {"hbm_gbs": 6540.8}, algorithmic)
    assert r["dram_bytes"] == pytest.approx(273.85088e6)
    assert r["dram_gbs"] == pytest.approx(273.85088e6 / 108992.0)
    assert r["frac_hbm"] == pytest.approx(r["dram_gbs"] / 6540.8)
    assert r["traffic_over_algorithmic"] == pytest.approx(273.85088e6 / algorithmic)
    assert r["class"] == "balanced"  # SM 37 %, memory 31 %: between the thresholds


def test_kernel_traffic_median_per_launch():
    t = roofline.kernel_traffic(RAW, "gqa_attention")
    assert t == pytest.approx((273.85088e6 + 273.472768e6) / 2)
    assert roofline.kernel_traffic(RAW, "no_such_kernel") is None


def test_launch_list_shares():
    rows = roofline.launch_shares(roofline.parse(LAUNCHES))
    assert rows[0]["kernel"].find("gqa_attention_sm100") >= 0
    assert rows[0]["launches"] == 12
    assert sum(r["share"] for r in rows) == pytest.approx(1.0)
    assert rows[0]["us_per_launch"] == pytest.approx(rows[0]["total_ms"] * 1e3 / 12)


@pytest.mark.parametrize("sm,mem,want", [(70, 30, "compute-bound"), (30, 70, "bandwidth-bound"),
                                         (10, 15, "latency/occupancy-bound"), (40, 50, "balanced"),
                                         (None, 50, "unknown"), (65, 65, "compute-bound")])
def test_classify_matches_reference_rule(sm, mem, want):
    assert roofline.classify(sm, mem) == want


def test_cli_prints_both_forms(capsys):
    assert roofline.main([RAW, "--algorithmic-bytes", str(512 * 564480)]) == 0
    out = capsys.readouterr().out
    assert "gqa_attention_sm100" in out and "balanced" in out
    assert roofline.main([LAUNCHES]) == 0
    assert "share" in capsys.readouterr().out


def test_short_kernel_names():
    assert roofline.short("void unnamed>::gqa_attention_sm100<0, 0, 1>(unnamed>::Params)", 60) == \
        "gqa_attention_sm100<0, 0, 1>"
    assert roofline.short("void unnamed>::gqa_attention_sm100<0, 0, 1>(unnamed>::Params)", 60,
                          templates=False) == "gqa_attention_sm100"
    torch_name = ("void at::native::vectorized_elementwise_kernel<4, at::native::FillFunctor<float>, "
                  "std::array<char *, 1>>(int, at::native::FillFunctor<float>, std::array<char *, 1>)")
    assert roofline.short(torch_name, 200, templates=False) == "vectorized_elementwise_kernel"
    assert roofline.short(torch_name, 29) == "vectorized_elementwise_kernel"
    assert roofline.short("gemm", 10) == "gemm"
