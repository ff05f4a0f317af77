"""framework/profile.py: the ncu CSV summaries (hand-made fixtures in ncu's CSV shape) and the
capture commands; no GPU needed."""
import os

import pytest

from framework import profile

FIX = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fixtures")


def _read(name):
    with open(os.path.join(FIX, name)) as f:
        return f.read()


def test_launch_list_summary():
    s = profile.summarize_launches(_read("ncu_launches_sample.csv"))
    assert [k for k, *_ in s] == ["kern_b(float *)", "kern_a(int)"]
    (kb, nb, tb, mb, shb), (ka, na, ta, ma, sha) = s
    assert (nb, na) == (1, 2)
    assert tb == pytest.approx(9.0) and ta == pytest.approx(8.0) and ma == pytest.approx(4.0)
    assert shb + sha == pytest.approx(1.0)
    assert "kern_a(int)" in profile.format_launches(s)


def test_raw_summary_units_and_stalls():
    (r,) = profile.summarize_raw(_read("ncu_raw_sample.csv"))
    assert r["duration_us"] == pytest.approx(12.5)
    assert r["dram_read"] == pytest.approx(100.5e6) and r["dram_write"] == pytest.approx(512e3)
    assert r["tensor_pct"] == pytest.approx(17.25)
    assert r["stalls"][0] == ("long_scoreboard", 3.5)
    text = profile.format_raw([r])
    assert "traffic 101.01 MB" in text and "long_scoreboard 3.50" in text


def test_ncu_commands_keep_clock_control_none():
    cmds = profile.ncu_commands("rbf", None)
    assert all("--clock-control none" in c for c in cmds if c.startswith("python"))
    assert any("--page raw --csv" in c for c in cmds)


def test_ncu_section_captures_name_one_kernel_each():
    cmds = [c for c in profile.ncu_commands("rbf", None) if "--section" in c]
    assert len(cmds) == 2
    for c, k in zip(cmds, ("rbf_fwd_tc_kernel", "rbf_bwd_tc_kernel")):
        assert f"-k regex:{k}" in c and " -c 3 " in c


def test_cli_summaries(capsys):
    assert profile.main(["--launches", os.path.join(FIX, "ncu_launches_sample.csv")]) == 0
    assert "kern_b" in capsys.readouterr().out
    assert profile.main(["--raw", os.path.join(FIX, "ncu_raw_sample.csv")]) == 0
    assert "tensor pipe %" in capsys.readouterr().out


@pytest.mark.gpu
def test_profile_candidate_sees_the_library_kernels(cuda_device):
    table, cuda_us, wall_us = profile.profile_candidate("rbf", mode="both", iters=3)
    assert "rbf_fwd_tc_kernel" in table
    assert "rbf_bwd_tc_kernel" in table
    assert 0 < cuda_us and 0 < wall_us


def test_timeline_formatting():
    import numpy as np
    from framework.timeline import ROLES, format_timeline
    buf = np.zeros((8, 1024), np.uint64)
    n = np.zeros(8, np.int32)
    t0 = 5_000_000
    buf[0][0] = (10 << 56) | t0
    buf[0][1] = (11 << 56) | (t0 + 640)
    buf[4][0] = (30 << 56) | (t0 + 1500)
    n[0], n[4] = 2, 1
    lines = format_timeline(buf, n)
    assert lines == ["PROD 10@0.00 11@0.64", "C0 30@1.50"]
    assert format_timeline(np.zeros((8, 4), np.uint64), np.zeros(8, np.int32)) == []
    assert len(ROLES) == 8


def test_span_summary_reads_the_per_cta_records():
    """format_spans: start / release / last strip / end per CTA (48-bit globaltimer ns; SM id
    above the end stamp, tile count above the last-strip stamp) -> quantiles and tiles per CTA."""
    import numpy as np
    from framework.timeline import format_spans
    sp = np.zeros((1024, 4), np.uint64)
    base = 1_000_000
    for c in range(4):
        start = base + 100 * c
        sp[c, 0] = start
        sp[c, 2] = start + 50
        tiles = 2 if c < 3 else 3
        sp[c, 3] = (start + 4000 * tiles) | (tiles << 48)
        sp[c, 1] = (start + 4000 * tiles + 200) | (7 << 48)
    lines = format_spans(sp, 4)
    text = "\n".join(lines)
    assert "tiles per CTA: 2 x3, 3 x1" in text
    assert lines[0].startswith("start") and "max    0.30" in lines[0]
    assert "last strip->end  p50 0.20  max 0.20" in text
    assert "3 tiles: end p50 12.50" in text
