"""CPU: the profiles pipeline (ncu_report.py).

* the committed summaries under profiles/ are exactly what the generator
  makes from the archived data beside them (the stale check of the
  reference's analysis/report/make_report.py:596-633), and every sanity
  anchor holds on that data;
* raw-page parsing normalises ncu's auto-scaled units (the reference's
  analysis/ncu/extract.py:55-70 does the same for bytes and time);
* each anchor refuses data that contradicts itself.
"""

import json
import os
import shutil

import pytest

import ncu_report

RAW = '''"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","gpu__time_duration.sum","dram__bytes_read.sum","dram__bytes_write.sum","dram__bytes.sum.per_second","l1tex__t_sectors_pipe_lsu_mem_global_op_ld.sum","l1tex__t_requests_pipe_lsu_mem_global_op_ld.sum","sm__warps_active.avg.pct_of_peak_sustained_active","sm__maximum_warps_per_active_cycle_pct","launch__occupancy_limit_registers","launch__occupancy_limit_shared_mem","launch__occupancy_limit_warps","launch__shared_mem_per_block_dynamic","smsp__average_warps_issue_stalled_long_scoreboard_per_issue_active.ratio","smsp__average_warps_issue_stalled_selected_per_issue_active.ratio","smsp__average_warps_issue_stalled_wait_per_issue_active.ratio"
"","","","","","","","","","","","us","Mbyte","Kbyte","Tbyte/s","sector","","%","%","block","block","block","Kbyte/block","inst","inst","inst"
"0","1","python","h","void gqa_decode_scan_kernel<9>(ScanParams)","1","7","(288, 1, 1)","(148, 1, 1)","0","10.0","100.000000","600.000000","4000.000000","6.040000","500","100","14.0","14.0625","1.000000","1.000000","7.000000","198.216000","6.5","1.0","2.0"
'''

LAUNCHES = '''==PROF== Connected to process 1
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","1","p","h","void gqa::gqa_decode_scan_kernel<9>(gqa::ScanParams)","1","7","(288, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","170.5"
"1","1","p","h","void gqa::gqa_decode_scan_kernel<9>(gqa::ScanParams)","1","7","(288, 1, 1)","(148, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","us","169.5"
"2","1","p","h","void fill(float *)","1","7","(256, 1, 1)","(512, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","ns","60000"
'''


def _bench_line(**over):
    d = {"metric": "m", "value": 6306.75, "unit": "GB/s", "n_gpus": 1, "steps": 100,
         "warmup": 5, "ms_per_step": 0.17025, "pct_of_sol": 96.26,
         "config": {"workload": "config2_rep", "kv_bytes_per_step": 1 << 30},
         "e2e": {"value": 6200.0, "ms_per_step": (1 << 30) / 6200.0e6},
         "roofline": {"achieved": 6306.75, "peak": 6551.7, "frac": 0.9626},
         "clocks": {"sm_mhz": 1900, "reasons": ["sw_power_cap"]}}
    d.update(over)
    return d


def test_committed_profiles_are_current():
    stale = ncu_report.generate(check=True)
    assert stale == [], f"regenerate with ncu_report.py generate: {stale}"


def test_every_gqa_kernel_has_a_capture():
    caps, _, _ = ncu_report.load_all()
    kernels = {m["kernel"].split("<")[0].split("::")[-1] for _, (_, secs) in caps.items()
               for _, m in secs}
    for k in ("gqa_decode_scan_kernel", "gqa_decode_fixed_merge_kernel",
              "gqa_decode_shard_merge_kernel", "gqa_decode_simt_kernel",
              "gqa_decode_plan_kernel", "gqa_decode_block_table_to_csr_kernel",
              "mla_decode_kernel"):
        assert k in kernels, k
    for _, (_, secs) in caps.items():
        for _, m in secs:
            assert m["dram_gbs"] is not None and m["achieved_occupancy_pct"] is not None
            assert m["lsu_load_sectors_per_request"] is not None or \
                "block_table_to_csr" in m["kernel"]


def test_raw_page_units(tmp_path):
    p = tmp_path / "raw.csv"
    p.write_text(RAW)
    rows, units = ncu_report.read_raw_page(str(p))
    m = ncu_report.launch_metrics(rows[0], units)
    assert m["kernel"] == "gqa_decode_scan_kernel<9>"
    assert m["duration_us"] == 100.0
    assert m["dram_read_bytes"] == 600e6 and m["dram_write_bytes"] == 4e6
    assert m["dram_gbs"] == pytest.approx(6040.0)
    assert m["ncu_dram_gbs"] == pytest.approx(6040.0)
    assert m["lsu_load_sectors_per_request"] == 5.0
    assert m["smem_dynamic_bytes"] == pytest.approx(198216.0)
    assert m["occupancy_limiter"] == "registers+shared_mem (1 blocks/SM)"
    assert m["stall_1"] == "long_scoreboard=6.50" and m["stall_2"] == "wait=2.00"
    ncu_report.check_capture("raw", {}, [("launch.0", m)])


def test_archive_round_trip_and_traffic_anchor(tmp_path):
    p = tmp_path / "raw.csv"
    p.write_text(RAW)
    path = ncu_report.extract(str(p), "cap", "ncu ...", algorithmic_bytes=600_000_000,
                              algorithmic_kernel="gqa_decode_scan", out_dir=str(tmp_path))
    header, secs = ncu_report.read_archive(path)
    assert header["algorithmic_bytes"] == 600_000_000
    assert secs[0][1]["dram_bytes"] == 604_000_000
    ncu_report.check_capture("cap", header, secs)
    assert ncu_report.traffic_ratio("cap", str(tmp_path)) == pytest.approx(604 / 600)
    # a kernel that moved half its data did not do the work
    header["algorithmic_bytes"] = 1_208_000_000
    with pytest.raises(ncu_report.SanityError):
        ncu_report.check_capture("cap", header, secs)
    # a unit mix-up shows as bytes / duration disagreeing with ncu's own rate
    secs[0][1]["ncu_dram_gbs"] = 60.4
    header["algorithmic_bytes"] = 600_000_000
    with pytest.raises(ncu_report.SanityError):
        ncu_report.check_capture("cap", header, secs)


def test_launch_list(tmp_path):
    p = tmp_path / "launches.csv"
    p.write_text(LAUNCHES)
    per = ncu_report.read_launch_list(str(p))
    assert per["gqa::gqa_decode_scan_kernel<9>"] == [2, 340.0]
    assert per["fill"] == [1, 60.0]
    path = ncu_report.launches(str(p), "l", "ncu ...", top="gqa_decode_scan", out_dir=str(tmp_path))
    header, secs = ncu_report.read_archive(path)
    assert secs[0][1]["share_pct"] == pytest.approx(85.0)
    ncu_report.check_launch_list("l", header, secs)
    header["expect_top"] = "fill"
    with pytest.raises(ncu_report.SanityError):
        ncu_report.check_launch_list("l", header, secs)


def _lines(*ds):
    return [("python bench.py", d) for d in ds]


def test_bench_anchors():
    ncu_report.check_bench("b", _lines(_bench_line()))
    with pytest.raises(ncu_report.SanityError):  # value not kv bytes / time
        ncu_report.check_bench("b", _lines(_bench_line(value=7000.0)))
    with pytest.raises(ncu_report.SanityError):  # fraction not achieved / peak
        ncu_report.check_bench("b", _lines(_bench_line(
            roofline={"achieved": 6306.75, "peak": 6551.7, "frac": 0.99})))
    with pytest.raises(ncu_report.SanityError):  # a throttled run is rejected
        ncu_report.check_bench("b", _lines(_bench_line(
            clocks={"sm_mhz": 900, "reasons": ["hw_slowdown"]})))
    with pytest.raises(ncu_report.SanityError):  # fewer than 3 warm-up steps
        ncu_report.check_bench("b", _lines(_bench_line(warmup=1)))


def test_generate_fills_and_detects_stale_blocks(tmp_path):
    d = tmp_path / "profiles"
    d.mkdir()
    raw = tmp_path / "raw.csv"
    raw.write_text(RAW)
    ncu_report.extract(str(raw), "cap", "ncu ...", out_dir=str(d))
    log = tmp_path / "bench.log"
    log.write_text("warning: something\n" + json.dumps(_bench_line()) + "\n")
    ncu_report.bench([(str(log), "python bench.py")], "run", out_dir=str(d))
    note, lines = ncu_report.read_bench(str(d / "run.bench.txt"))
    assert lines == [("python bench.py", _bench_line())]
    (d / "k.md").write_text("# k\n<!-- GEN:ncu:cap -->\nold\n<!-- /GEN:ncu:cap -->\n"
                            "<!-- GEN:bench:run -->\n<!-- /GEN:bench:run -->\n"
                            "<!-- GEN:kernels -->\n<!-- /GEN:kernels -->\n")
    assert ncu_report.generate(check=True, profiles=str(d)) == ["k.md"]
    assert ncu_report.generate(profiles=str(d)) == ["k.md"]
    text = (d / "k.md").read_text()
    assert "`gqa_decode_scan_kernel<9>`" in text and "old" not in text
    assert "Source: profiles/run.bench.txt" in text
    assert ncu_report.generate(check=True, profiles=str(d)) == []
    # a marker naming data that does not exist is an error, not an empty block
    shutil.copy(d / "k.md", d / "k2.md")
    with open(d / "k2.md", "a") as f:
        f.write("<!-- GEN:ncu:missing -->\n<!-- /GEN:ncu:missing -->\n")
    with pytest.raises(SystemExit):
        ncu_report.generate(check=True, profiles=str(d))
    os.remove(d / "k2.md")
