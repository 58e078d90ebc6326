"""kernels/bench/profile.py (CPU only): the ncu command lines keep the pool's capture rules, and a
launch-list CSV turns into the per-kernel table of the profile summaries."""

import pytest

from kernels.bench import profile

CSV = '''==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","python","h","void dk::<unnamed>::w4a16_gemv_kernel<1, 1, 0>(CUtensorMap, CUtensorMap, CUtensorMap, dk::<unnamed>::GemvParams)","1","7","(288, 1, 1)","(48, 6, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","6000"
"1","1","python","h","void dk::<unnamed>::decode_attention_kernel<6, 128>(CUtensorMap, CUtensorMap, dk::<unnamed>::AttnParams)","1","7","(160, 1, 1)","(32, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","9000"
"2","1","python","h","void dk::<unnamed>::w4a16_gemv_kernel<1, 1, 0>(CUtensorMap, CUtensorMap, CUtensorMap, dk::<unnamed>::GemvParams)","1","7","(288, 1, 1)","(48, 6, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","3"
==PROF== Disconnected from process 1
'''


def test_launch_summary(tmp_path):
    f = tmp_path / "launches.csv"
    f.write_text(CSV)
    s = profile.launch_summary(str(f))
    assert [e["kernel"] for e in s] == ["dk::<unnamed>::w4a16_gemv_kernel<1, 1, 0>",
                                       "dk::<unnamed>::decode_attention_kernel<6, 128>"]
    assert s[0]["launches"] == 2 and s[0]["total_us"] == pytest.approx(9.0) and s[0]["mean_us"] == pytest.approx(4.5)
    assert s[0]["share"] == pytest.approx(0.5) and s[1]["share"] == pytest.approx(0.5)
    md = profile.markdown(s, top=1)
    assert "| dk::<unnamed>::w4a16_gemv_kernel<1, 1, 0> | 2 | 9.0 | 50.0% |" in md
    assert "(1 more kernels) | 1 | 9.0 | 50.0%" in md and "| **total** | 3 | 18.0 | |" in md


def test_commands_keep_the_capture_rules():
    cmd = profile.ncu_command("launches", ["decode", "ours", "2"], "l.csv", skip=5, count=100)
    assert cmd[:4] == ["ncu", "--metrics", "gpu__time_duration.sum", "--clock-control"] and "none" in cmd
    assert cmd[cmd.index("-s") + 1] == "5" and cmd[cmd.index("-c") + 1] == "100"
    full = profile.ncu_command("kernel", ["gemv", "151936", "1536"], "p", kernel="w4a16_gemv", skip=2, count=1)
    assert full[full.index("--clock-control") + 1] == "none" and "--set" in full
    assert full[full.index("-k") + 1] == "regex:w4a16_gemv" and full[full.index("-c") + 1] == "1"
    assert full.index("-s") < full.index("-c")
    with pytest.raises(ValueError):
        profile.ncu_command("kernel", ["gemv", "1536", "1536"], "p")  # no kernel filter
    with pytest.raises(ValueError):
        profile.ncu_command("kernel", ["gemv", "1536", "1536"], "p", kernel="x", count=10)  # too many launches
    with pytest.raises(ValueError):
        profile.ncu_command("sanitize", ["gemv"], "p")
