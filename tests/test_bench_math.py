"""bench.py's measurement arithmetic, checked on the CPU.

The GPU numbers in the JSON line rest on a few host-side pieces: the seeded
input rows (every world size must see the same rows, or the N > 1 parity leg
and the scaling lines compare different inputs), the DRAM traffic estimate of
the GEMM roofline (algorithmic bytes per shape times the ratio an ncu capture
measured, profiles/ncu_traffic.json), the roofline fraction and its peak, and
the head-group setting the config reports (it must be the one the model runs).
"""
import json
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200"))

import bench  # noqa: E402


@pytest.mark.parametrize("world", [2, 3, 8])
def test_seeded_rows_do_not_depend_on_the_split(world):
    S, dim = 3 * bench.ROW_CHUNK + 517, 16
    full = bench.seeded_rows(0, S, dim, seed=11)
    base, rem = divmod(S, world)
    start = 0
    for r in range(world):
        n = base + (r < rem)
        part = bench.seeded_rows(start, start + n, dim, seed=11)
        assert torch.equal(part.view(torch.int16), full[start:start + n].view(torch.int16)), (world, r)
        start += n
    assert start == S


def _algorithmic(M, N, K):
    # int8 A and B, bf16 output, fp32 row scales, fp32 column scales + bf16 bias
    return M * K + N * K + 2 * M * N + 4 * M + 6 * N


def test_gemm_traffic_scales_the_profiled_ratios():
    with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
        rec = json.load(f)
    ratio = {tuple(e["nk"]): e["ratio"] for e in rec["shapes"]}
    M = 128000
    shapes = [(M, 15360, 5120), (M, 5120, 5120), (M, 13824, 5120), (M, 5120, 13824)]
    traffic, used = bench.gemm_dram_traffic(shapes)
    want = sum(ratio[(N, K)] * _algorithmic(M, N, K) for M, N, K in shapes) / len(shapes)
    assert traffic == pytest.approx(want, rel=1e-12)
    assert used == [round(ratio[(N, K)], 3) for _, N, K in shapes]
    # every recorded ratio came from a capture: DRAM bytes over the shape's algorithmic bytes
    for e in rec["shapes"]:
        assert e["ratio"] == pytest.approx((e["dram_read"] + e["dram_write"]) / e["algorithmic_bytes"], rel=1e-3)


def test_gemm_traffic_falls_back_to_the_default_ratio():
    with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
        default = json.load(f)["default"]["ratio"]
    traffic, used = bench.gemm_dram_traffic([(4096, 2048, 1024)])
    assert used == [round(default, 3)]
    assert traffic == pytest.approx(default * _algorithmic(4096, 2048, 1024), rel=1e-12)


@pytest.mark.parametrize("in_step", [False, True])
def test_gemm_roofline_fraction(in_step):
    pk = {"hbm_gbs": 6450.0, "bf16_tflops": 1665.0, "bf16_tflops_sustained": 1386.0}
    work, ms = 2.0 * 128000 * 5120 * 5120 * 4, 8.0
    r = bench.gemm_roofline({"gemm": {"work": work, "ms": ms, "calls": 4}}, pk, "measured", in_step=in_step)
    achieved = work / (ms * 1e-3) / 1e12
    peak = 2.0 * (pk["bf16_tflops_sustained"] if in_step else pk["bf16_tflops"])
    assert r["bound"] == "tensor" and r["unit"] == "TOPS"
    assert r["achieved"] == pytest.approx(achieved, abs=0.05)
    assert r["peak"] == pytest.approx(peak, abs=0.05)
    assert r["frac"] == pytest.approx(achieved / peak, abs=1e-4)
    assert ("sustained" if in_step else "burst") in r["peak_source"]
    assert bench.gemm_roofline({}, pk, "measured") is None


def test_peaks_fall_back_when_the_measured_file_is_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(bench, "PEAKS_FILE", str(tmp_path / "absent.json"))
    pk, src = bench.peaks()
    assert src == "fallback" and pk == bench.FALLBACK_PEAKS
    f = tmp_path / "peaks.json"
    f.write_text(json.dumps({"hbm_gbs": 1.0, "bf16_tflops": 2.0, "bf16_tflops_sustained": 3.0}))
    monkeypatch.setattr(bench, "PEAKS_FILE", str(f))
    pk, src = bench.peaks()
    assert src == "measured" and pk["bf16_tflops"] == 2.0


@pytest.mark.parametrize("env,world", [({}, 2), ({"H3B_SP_OVERLAP_GROUPS": "5"}, 8),
                                       ({"MINIMAX_SP_OVERLAP_CHUNKS": "4"}, 2),
                                       ({"MINIMAX_SP_OVERLAP_CHUNKS": "3"}, 2),
                                       ({"MINIMAX_SP_OVERLAP_CHUNKS_W4": "4"}, 4),
                                       ({"H3B_SP_OVERLAP_GROUPS": "1"}, 4)])
def test_reported_overlap_groups_are_the_models(monkeypatch, env, world):
    from h3b import sp
    for k in ("H3B_SP_OVERLAP_GROUPS", "MINIMAX_SP_OVERLAP_CHUNKS", "MINIMAX_SP_OVERLAP_CHUNKS_W4"):
        monkeypatch.delenv(k, raising=False)
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    from types import SimpleNamespace
    cfg = SimpleNamespace(heads=40)  # the benchmark block's head count
    hp = cfg.heads // world
    n = sp.overlap_groups(hp, world)
    # the model overlaps only with more than one group that divides the rank's heads
    assert bench.overlap_groups(cfg, world) == (n if n > 1 and hp % n == 0 else 0)
