#!/usr/bin/env python
"""Profiles pipeline: ncu captures and bench lines -> the committed summaries.

B200 counterpart of the reference's analysis/ncu/extract.py (an ncu report
reduced to the few metrics the write-up quotes: DRAM throughput,
sectors/request, achieved occupancy, occupancy limiter, top-3 stalls, L2 hit
rate, DRAM/L2 bytes) and analysis/report/make_report.py (every published
number generated between ``<!-- GEN:name -->`` markers from archived data;
sanity anchors re-derived from that data refuse to publish when they are off,
make_report.py:170-217; ``--check`` fails when a committed block is stale,
make_report.py:596-633).

Archived data lives beside the summaries under ``profiles/`` as small text
files, each carrying the command that produced it:

  <stem>.ncu.txt       key metrics of every launch in one ncu capture
  <stem>.launches.txt  per-kernel launches / total time / share of a
                       ``--metrics gpu__time_duration.sum`` launch list
  <stem>.bench.txt     bench.py JSON lines

Subcommands (run from anywhere; paths are taken as given):

  ncu_report.py extract CAPTURE --name STEM --command CMD
                [--algorithmic-bytes N --algorithmic-kernel REGEX] [--note TEXT]
      CAPTURE is a .ncu-rep (exported with ``ncu -i CAPTURE --page raw --csv``)
      or an already exported raw-page CSV.
  ncu_report.py launches CSV --name STEM --command CMD [--top REGEX]
      CSV is the ``--csv --log-file`` output of a launch-list capture.
  ncu_report.py bench --name STEM --entry LOG CMD [--entry LOG CMD ...] [--note TEXT]
      Each LOG holds bench.py output written by CMD; its JSON lines are
      archived under that command.
  ncu_report.py generate [--check]
      Regenerates every GEN block of profiles/*.md after the sanity anchors
      pass; ``--check`` changes nothing and exits 1 when a block is stale.
"""

import argparse
import configparser
import csv
import io
import json
import os
import re
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
PROFILES = os.path.join(REPO, "profiles")


class SanityError(SystemExit):
    """A sanity anchor failed: the archived data contradicts itself."""

    def __init__(self, what):
        super().__init__(f"SANITY ANCHOR FAILED: {what} - refusing to publish")
        self.what = what


# ---------------------------------------------------------------- raw page

# ncu prints decimal SI prefixes; everything is normalised to bytes, us, GHz,
# GB/s.
_BYTES = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "Tbyte": 1e12}
_US = {"ns": 1e-3, "nsecond": 1e-3, "us": 1.0, "usecond": 1.0, "ms": 1e3, "msecond": 1e3,
       "s": 1e6, "second": 1e6}
_GHZ = {"hz": 1e-9, "Khz": 1e-6, "Mhz": 1e-3, "Ghz": 1.0}
_GBS = {"byte/s": 1e-9, "Kbyte/s": 1e-6, "Mbyte/s": 1e-3, "Gbyte/s": 1.0, "Tbyte/s": 1e3}
_PER_BLOCK = {"byte/block": 1.0, "Kbyte/block": 1e3, "Mbyte/block": 1e6}
_PER_CYCLE = {"byte/cycle": 1.0, "Kbyte/cycle": 1e3, "Mbyte/cycle": 1e6}


def _num(s):
    try:
        return float(str(s).replace(",", ""))
    except ValueError:
        return None


def _scaled(row, units, name, table, what):
    v = _num(row.get(name, ""))
    if v is None:
        return None
    u = units.get(name, "")
    if u not in table:
        raise SystemExit(f"metric {name}: unknown {what} unit {u!r}")
    return v * table[u]


def read_raw_page(path):
    """(rows, units) of an ncu raw page: one {column: text} dict per launch."""
    if path.endswith(".ncu-rep"):
        r = subprocess.run(["ncu", "-i", path, "--page", "raw", "--csv"], capture_output=True,
                           text=True, check=True)
        text = r.stdout
    else:
        with open(path, newline="") as f:
            text = f.read()
    rows = [r for r in csv.reader(io.StringIO(text)) if r]
    # ncu may print notes before the table; the header row starts with "ID"
    start = next((i for i, r in enumerate(rows) if r[0] == "ID"), None)
    if start is None or len(rows) < start + 3:
        raise SystemExit(f"{path}: not an ncu raw-page CSV (header, units, >= 1 launch)")
    names, unit_row = rows[start], rows[start + 1]
    units = dict(zip(names, unit_row))
    return [dict(zip(names, r)) for r in rows[start + 2:]], units


def short_kernel_name(name):
    """'void gqa_decode_scan_kernel<9>(ScanParams)' -> 'gqa_decode_scan_kernel<9>'."""
    n = name.strip()
    if n.startswith("void "):
        n = n[5:]
    depth = 0
    for i, c in enumerate(n):
        if c == "<":
            depth += 1
        elif c == ">":
            depth -= 1
        elif c == "(" and depth == 0:
            return n[:i]
    return n


_STALL = re.compile(r"^smsp__average_warps_issue_stalled_(.+)_per_issue_active\.ratio$")
_LIMIT = "launch__occupancy_limit_"


def launch_metrics(row, units):
    """The summary metrics of one launch (None where the capture lacks one)."""
    m = {"kernel": short_kernel_name(row.get("Kernel Name", "")),
         "grid": row.get("Grid Size", ""), "block": row.get("Block Size", "")}
    m["duration_us"] = _scaled(row, units, "gpu__time_duration.sum", _US, "time")
    m["dram_read_bytes"] = _scaled(row, units, "dram__bytes_read.sum", _BYTES, "byte")
    m["dram_write_bytes"] = _scaled(row, units, "dram__bytes_write.sum", _BYTES, "byte")
    if m["dram_read_bytes"] is not None and m["dram_write_bytes"] is not None:
        m["dram_bytes"] = m["dram_read_bytes"] + m["dram_write_bytes"]
    else:
        m["dram_bytes"] = _scaled(row, units, "dram__bytes.sum", _BYTES, "byte")
    if m["dram_bytes"] is not None and m["duration_us"]:
        m["dram_gbs"] = m["dram_bytes"] / (m["duration_us"] * 1e3)
    else:
        m["dram_gbs"] = None
    m["ncu_dram_gbs"] = _scaled(row, units, "dram__bytes.sum.per_second", _GBS, "rate")
    m["dram_pct_of_peak"] = _num(row.get("gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
                                         ""))
    per_cycle = _scaled(row, units, "dram__bytes.sum.peak_sustained", _PER_CYCLE, "byte/cycle")
    dram_ghz = _scaled(row, units, "dram__cycles_elapsed.avg.per_second", _GHZ, "frequency")
    m["dram_peak_gbs"] = per_cycle * dram_ghz if per_cycle and dram_ghz else None
    ratio = _num(row.get("l1tex__average_t_sectors_per_request_pipe_lsu_mem_global_op_ld.ratio",
                         ""))
    if ratio is None:
        sec = _num(row.get("l1tex__t_sectors_pipe_lsu_mem_global_op_ld.sum", ""))
        req = _num(row.get("l1tex__t_requests_pipe_lsu_mem_global_op_ld.sum", ""))
        ratio = sec / req if sec is not None and req else None
    m["lsu_load_sectors_per_request"] = ratio
    m["achieved_occupancy_pct"] = _num(row.get("sm__warps_active.avg.pct_of_peak_sustained_active",
                                               ""))
    m["theoretical_occupancy_pct"] = _num(row.get("sm__maximum_warps_per_active_cycle_pct", ""))
    limits = [(_num(v), k[len(_LIMIT):]) for k, v in row.items() if k.startswith(_LIMIT)]
    limits = [(v, k) for v, k in limits if v is not None]
    if limits:
        lo = min(v for v, _ in limits)
        m["occupancy_limiter"] = "+".join(sorted(k for v, k in limits if v == lo)) + \
            f" ({lo:g} blocks/SM)"
    else:
        m["occupancy_limiter"] = None
    m["l2_hit_pct"] = _num(row.get("lts__t_sector_hit_rate.pct", ""))
    m["tensor_pipe_pct"] = _num(row.get("sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
                                        ""))
    m["registers_per_thread"] = _num(row.get("launch__registers_per_thread", ""))
    m["smem_dynamic_bytes"] = _scaled(row, units, "launch__shared_mem_per_block_dynamic",
                                      _PER_BLOCK, "per-block")
    m["sm_clock_ghz"] = _scaled(row, units, "sm__cycles_elapsed.avg.per_second", _GHZ, "frequency")
    m["dram_clock_ghz"] = dram_ghz
    stalls = []
    for k, v in row.items():
        s = _STALL.match(k)
        if s and s.group(1) != "selected" and _num(v) is not None:
            stalls.append((_num(v), s.group(1)))
    stalls.sort(reverse=True)
    for i in range(3):
        m[f"stall_{i + 1}"] = f"{stalls[i][1]}={stalls[i][0]:.2f}" if i < len(stalls) else None
    return m


# ---------------------------------------------------------------- archive

def _fmt(v):
    if v is None:
        return "n/a"
    if isinstance(v, float):
        return str(int(v)) if v.is_integer() and abs(v) < 1e15 else repr(v)
    return str(v)


def _parser():
    cp = configparser.ConfigParser(interpolation=None)
    cp.optionxform = str
    return cp


def write_archive(path, header, sections):
    cp = _parser()
    cp["capture"] = {k: _fmt(v) for k, v in header.items() if v is not None}
    for name, d in sections:
        cp[name] = {k: _fmt(v) for k, v in d.items()}
    buf = io.StringIO()
    cp.write(buf)
    with open(path, "w") as f:
        f.write(buf.getvalue().rstrip() + "\n")


def _typed(v):
    if v == "n/a":
        return None
    x = _num(v)
    return v if x is None else x


def read_archive(path):
    """(header dict, [(section name, dict)]) with numbers parsed."""
    cp = _parser()
    with open(path) as f:
        cp.read_file(f)
    header = {k: _typed(v) for k, v in cp["capture"].items()} if "capture" in cp else {}
    secs = [(s, {k: _typed(v) for k, v in cp[s].items()}) for s in cp.sections()
            if s != "capture"]
    return header, secs


def extract(capture, name, command, algorithmic_bytes=None, algorithmic_kernel=None,
            note=None, out_dir=PROFILES):
    rows, units = read_raw_page(capture)
    sections = [(f"launch.{i}", launch_metrics(r, units)) for i, r in enumerate(rows)]
    header = {"command": command, "source": os.path.basename(capture), "note": note,
              "algorithmic_bytes": algorithmic_bytes, "algorithmic_kernel": algorithmic_kernel}
    path = os.path.join(out_dir, f"{name}.ncu.txt")
    write_archive(path, header, sections)
    return path


def read_launch_list(path):
    """{kernel: [launches, total us]} from a long-format ncu --csv log."""
    with open(path, newline="") as f:
        lines = [ln for ln in f if ln.startswith('"')]
    per = {}
    for r in csv.DictReader(io.StringIO("".join(lines))):
        if r.get("Metric Name") != "gpu__time_duration.sum":
            continue
        v = _num(r["Metric Value"])
        u = r.get("Metric Unit", "")
        if v is None or u not in _US:
            raise SystemExit(f"{path}: bad duration {r['Metric Value']!r} {u!r}")
        k = short_kernel_name(r["Kernel Name"])[:100]
        e = per.setdefault(k, [0, 0.0])
        e[0] += 1
        e[1] += v * _US[u]
    if not per:
        raise SystemExit(f"{path}: no gpu__time_duration.sum rows")
    return per


def launches(csv_path, name, command, top=None, out_dir=PROFILES):
    per = read_launch_list(csv_path)
    total = sum(t for _, t in per.values())
    sections = []
    for k, (n, t) in sorted(per.items(), key=lambda kv: -kv[1][1]):
        sections.append((f"kernel.{len(sections)}",
                         {"kernel": k, "launches": n, "total_us": round(t, 3),
                          "share_pct": round(100.0 * t / total, 3)}))
    header = {"command": command, "source": os.path.basename(csv_path), "expect_top": top}
    path = os.path.join(out_dir, f"{name}.launches.txt")
    write_archive(path, header, sections)
    return path


def bench_lines(log_path):
    out = []
    with open(log_path) as f:
        for ln in f:
            ln = ln.strip()
            if ln.startswith("{") and ln.endswith("}"):
                try:
                    out.append(json.loads(ln))
                except json.JSONDecodeError:
                    pass
    return out


_KEEP = {
    None: ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
           "median_us_per_step", "pct_of_sol", "higher_is_better", "scaling", "vs_baseline",
           "dtype", "gpu_launches", "unavailable", "stages_us"),
    "config": ("workload", "api", "kernel", "num_splits", "exchange", "parallelism",
               "global_batch", "kv_bytes_per_step", "bytes_per_step", "per_step_sample_requests"),
    "e2e": ("value", "unit", "ms_per_step", "h2d_bytes_per_step", "d2h_bytes_per_step",
            "serial_ms_per_step", "serial_value"),
    "roofline": ("bound", "achieved", "peak", "unit", "frac", "traffic", "kernel"),
    "clocks": ("sm_mhz", "sm_max_mhz", "reasons", "samples"),
    "cpu_baseline": ("value", "unit", "cores", "kind"),
    "reference_py": ("value", "unit", "cores", "kind", "ms_per_full_step_extrapolated", "sample"),
}


def slim(d):
    """The fields of a bench.py line the summaries and anchors use."""
    out = {k: d[k] for k in _KEEP[None] if k in d}
    for sub, keys in _KEEP.items():
        if sub is not None and isinstance(d.get(sub), dict):
            out[sub] = {k: d[sub][k] for k in keys if k in d[sub]}
    return out


def bench(entries, name, note=None, out_dir=PROFILES):
    """Archive the JSON lines of several bench.py runs: entries is a list of
    (log path, the command that wrote it)."""
    path = os.path.join(out_dir, f"{name}.bench.txt")
    with open(path, "w") as f:
        if note:
            f.write(f"# note: {note}\n")
        for log_path, command in entries:
            lines = bench_lines(log_path)
            if not lines:
                raise SystemExit(f"{log_path}: no bench.py JSON line")
            f.write(f"# command: {command}\n")
            for d in lines:
                f.write(json.dumps(slim(d), sort_keys=True) + "\n")
    return path


def read_bench(path):
    """(note, [(command, line dict)])."""
    note, command, out = None, None, []
    with open(path) as f:
        for ln in f:
            if ln.startswith("# note:"):
                note = ln.split(":", 1)[1].strip()
            elif ln.startswith("# command:"):
                command = ln.split(":", 1)[1].strip()
            elif ln.strip():
                out.append((command, json.loads(ln)))
    return note, out


# ---------------------------------------------------------------- anchors

def _close(a, b, rel):
    return a is not None and b is not None and abs(a - b) <= rel * max(abs(a), abs(b), 1e-30)


REJECT_REASONS = {"hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"}


def check_capture(stem, header, secs):
    """Anchors of one ncu capture."""
    for sname, m in secs:
        where = f"{stem} {sname} ({m.get('kernel')})"
        if m.get("dram_gbs") is not None and m.get("ncu_dram_gbs") is not None:
            if not _close(m["dram_gbs"], m["ncu_dram_gbs"], 0.03):
                raise SanityError(f"{where}: DRAM bytes / duration = {m['dram_gbs']:.1f} GB/s but "
                                  f"ncu reports {m['ncu_dram_gbs']:.1f} GB/s (unit mix-up?)")
        ach, th = m.get("achieved_occupancy_pct"), m.get("theoretical_occupancy_pct")
        if ach is not None and th is not None and ach > th + 1.0:
            raise SanityError(f"{where}: achieved occupancy {ach}% above theoretical {th}%")
        if m.get("dram_pct_of_peak") is not None and not 0 <= m["dram_pct_of_peak"] <= 100.5:
            raise SanityError(f"{where}: DRAM throughput {m['dram_pct_of_peak']}% of peak")
    alg = header.get("algorithmic_bytes")
    if alg:
        pat = re.compile(str(header.get("algorithmic_kernel") or "."))
        hits = [m for _, m in secs if pat.search(m.get("kernel", ""))]
        if not hits:
            raise SanityError(f"{stem}: no launch matches {pat.pattern!r}")
        for m in hits:
            t = m.get("dram_bytes")
            if t is None:
                raise SanityError(f"{stem}: {m['kernel']} has no DRAM byte counters")
            # the kernel must have moved its data (less means it skipped work)
            # and not re-read it (more than 5 % over means wasted traffic the
            # summary has to explain)
            if not 0.98 * alg <= t <= 1.05 * alg:
                raise SanityError(f"{stem}: {m['kernel']} moved {t:.0f} DRAM bytes for "
                                  f"{alg:.0f} algorithmic bytes ({t / alg:.3f}x)")


def check_launch_list(stem, header, secs):
    share = sum(d["share_pct"] for _, d in secs)
    if abs(share - 100.0) > 0.1:
        raise SanityError(f"{stem}: shares add up to {share:.3f}%")
    top = header.get("expect_top")
    if top and not re.search(str(top), str(secs[0][1]["kernel"])):
        raise SanityError(f"{stem}: top kernel is {secs[0][1]['kernel']}, expected {top}")


def check_bench(stem, lines):
    for i, d in enumerate(d for _, d in lines):
        where = f"{stem} line {i + 1}"
        if d.get("impl") == "reference" or "unavailable" in d:
            continue
        if d.get("warmup", 0) < 3:
            raise SanityError(f"{where}: {d.get('warmup')} warm-up steps (3 required)")
        cfg = d.get("config", {})
        kv = cfg.get("kv_bytes_per_step") or cfg.get("bytes_per_step")
        ms = d.get("ms_per_step")
        if kv and ms and not _close(d["value"], kv / (ms * 1e-3) / 1e9, 0.005):
            raise SanityError(f"{where}: value {d['value']} GB/s but bytes per step / "
                              f"ms_per_step = {kv / (ms * 1e-3) / 1e9:.2f}")
        e2e = d.get("e2e") or {}
        if kv and e2e.get("ms_per_step") and \
                not _close(e2e["value"], kv / (e2e["ms_per_step"] * 1e-3) / 1e9, 0.005):
            raise SanityError(f"{where}: e2e value {e2e['value']} disagrees with its ms_per_step")
        rl = d.get("roofline") or {}
        if rl.get("peak") and rl.get("achieved") is not None and rl.get("frac") is not None:
            if abs(rl["frac"] - rl["achieved"] / rl["peak"]) > 1e-3:
                raise SanityError(f"{where}: roofline frac {rl['frac']} != achieved / peak")
        if rl.get("peak") and d.get("pct_of_sol") is not None:
            want = 100.0 * d["value"] / (rl["peak"] * d.get("n_gpus", 1))
            if abs(d["pct_of_sol"] - want) > 0.05:
                raise SanityError(f"{where}: pct_of_sol {d['pct_of_sol']} != {want:.2f}")
        reasons = set((d.get("clocks") or {}).get("reasons") or [])
        if reasons & REJECT_REASONS:
            raise SanityError(f"{where}: clocks show {sorted(reasons & REJECT_REASONS)}; "
                              "the run is rejected and must be taken again")


# ---------------------------------------------------------------- blocks

def _g(v, fmt="{:.1f}"):
    return "n/a" if v is None else fmt.format(v)


def block_ncu(stem, header, secs):
    rows = ["| kernel | grid x block | us | DRAM bytes (r + w) | DRAM GB/s | DRAM % of peak | "
            "LSU sectors/req | occupancy achieved / theor. | limiter | regs | L2 hit | "
            "tensor pipe | top stalls |",
            "|---|---|---|---|---|---|---|---|---|---|---|---|---|"]
    for _, m in secs:
        stalls = ", ".join(s for s in (m.get("stall_1"), m.get("stall_2"), m.get("stall_3")) if s)
        rows.append(
            f"| `{m['kernel']}` | {m.get('grid')} x {m.get('block')} | "
            f"{_g(m.get('duration_us'), '{:.2f}')} | "
            f"{_g(m.get('dram_read_bytes'), '{:.4g}')} + {_g(m.get('dram_write_bytes'), '{:.4g}')} | "
            f"{_g(m.get('dram_gbs'), '{:.0f}')} | {_g(m.get('dram_pct_of_peak'))} | "
            f"{_g(m.get('lsu_load_sectors_per_request'), '{:.2f}')} | "
            f"{_g(m.get('achieved_occupancy_pct'))} / {_g(m.get('theoretical_occupancy_pct'))} % | "
            f"{m.get('occupancy_limiter') or 'n/a'} | {_g(m.get('registers_per_thread'), '{:.0f}')} | "
            f"{_g(m.get('l2_hit_pct'))} % | {_g(m.get('tensor_pipe_pct'))} % | {stalls or 'n/a'} |")
    extra = []
    if header.get("algorithmic_bytes"):
        extra.append(f"Algorithmic bytes per launch of `{header.get('algorithmic_kernel')}`: "
                     f"{header['algorithmic_bytes']:.0f}.")
    if header.get("note"):
        extra.append(str(header["note"]))
    clocks = [(m.get("sm_clock_ghz"), m.get("dram_clock_ghz")) for _, m in secs]
    if clocks and clocks[0][0]:
        extra.append(f"SM / DRAM clock during the capture: {clocks[0][0]:.2f} / "
                     f"{clocks[0][1]:.2f} GHz; ncu DRAM peak "
                     f"{_g(secs[0][1].get('dram_peak_gbs'), '{:.0f}')} GB/s.")
    return "\n".join(rows + [""] + extra + ["", f"Command: `{header.get('command')}`",
                                            f"Source: profiles/{stem}.ncu.txt"])


def block_launches(stem, header, secs):
    rows = ["| kernel | launches | total us | share |", "|---|---|---|---|"]
    for _, d in secs:
        rows.append(f"| `{d['kernel'][:90]}` | {d['launches']:.0f} | {d['total_us']:.1f} | "
                    f"{d['share_pct']:.1f} % |")
    return "\n".join(rows + ["", f"Command: `{header.get('command')}`",
                             f"Source: profiles/{stem}.launches.txt"])


def block_bench(stem, note, lines):
    rows = ["| # | workload | api / kernel | N | ms / step | median us | GB/s | % of SoL | e2e GB/s | "
            "roofline frac | SM MHz (reasons) |",
            "|---|---|---|---|---|---|---|---|---|---|---|"]
    commands = []
    for command, d in lines:
        if command not in commands:
            commands.append(command)
        ci = commands.index(command) + 1
        c = d.get("config", {})
        if d.get("impl") == "reference":
            rows.append(f"| {ci} | {c.get('workload')} | reference (CPU, C port) | "
                        f"{d.get('n_gpus')} | {d.get('ms_per_step')} | "
                        f"{d.get('median_us_per_step')} | {d.get('value')} | | | | "
                        f"{(d.get('cpu_baseline') or {}).get('cores')} host threads |")
            rp = d.get("reference_py")
            if rp:
                # the reference's own python/reference.py on a sample of the
                # same step, extrapolated to the whole step
                rows.append(f"| {ci} | {c.get('workload')} | reference.py (CPU, unmodified) | "
                            f"{d.get('n_gpus')} | {rp.get('ms_per_full_step_extrapolated')} | | "
                            f"{rp.get('value')} | | | | {rp.get('cores')} host threads |")
            continue
        kern = c.get("api", "block_table") if c.get("kernel", "auto") == "auto" else c.get("kernel")
        if c.get("kernel") == "v2":
            kern += f" ns={c.get('num_splits')}"
        if c.get("exchange"):
            kern += f" / {c['exchange']}"
        clk = d.get("clocks") or {}
        rows.append(f"| {ci} | {c.get('workload')} | {kern} | {d.get('n_gpus')} | "
                    f"{d.get('ms_per_step')} | {d.get('median_us_per_step')} | {d.get('value')} | "
                    f"{d.get('pct_of_sol')} | {(d.get('e2e') or {}).get('value')} | "
                    f"{(d.get('roofline') or {}).get('frac')} | "
                    f"{clk.get('sm_mhz')} ({', '.join(clk.get('reasons') or []) or 'none'}) |")
    out = rows + [""]
    if note:
        out += [note, ""]
    out += ["Commands:", ""] + [f"{i + 1}. `{c}`" for i, c in enumerate(commands)]
    return "\n".join(out + ["", f"Source: profiles/{stem}.bench.txt"])


def block_kernels(captures):
    """One row per kernel over all captures: the quantities every kernel's
    summary must give (DRAM throughput, sectors/request, achieved occupancy)."""
    rows = ["| kernel | capture | us | DRAM GB/s | DRAM % of peak | LSU sectors/req | "
            "achieved occupancy | limiter |", "|---|---|---|---|---|---|---|---|"]
    seen = set()
    for stem, (header, secs) in sorted(captures.items()):
        for _, m in secs:
            key = (m["kernel"], stem)
            if key in seen or not any(t in m["kernel"] for t in ("gqa_decode", "mla_", "dsa_")):
                continue
            seen.add(key)
            rows.append(f"| `{m['kernel']}` | {stem} | {_g(m.get('duration_us'), '{:.2f}')} | "
                        f"{_g(m.get('dram_gbs'), '{:.0f}')} | {_g(m.get('dram_pct_of_peak'))} | "
                        f"{_g(m.get('lsu_load_sectors_per_request'), '{:.2f}')} | "
                        f"{_g(m.get('achieved_occupancy_pct'))} % | "
                        f"{m.get('occupancy_limiter') or 'n/a'} |")
    return "\n".join(rows + ["", "Source: profiles/*.ncu.txt"])


# ---------------------------------------------------------------- generate

MARKER = re.compile(r"(<!-- GEN:([a-z]+):?([A-Za-z0-9_.\-]*) -->)(.*?)(<!-- /GEN:\2:?\3 -->)",
                    re.S)


def load_all(profiles=PROFILES):
    caps, lists, benches = {}, {}, {}
    for fn in sorted(os.listdir(profiles)):
        p = os.path.join(profiles, fn)
        if fn.endswith(".ncu.txt"):
            caps[fn[:-len(".ncu.txt")]] = read_archive(p)
        elif fn.endswith(".launches.txt"):
            lists[fn[:-len(".launches.txt")]] = read_archive(p)
        elif fn.endswith(".bench.txt"):
            benches[fn[:-len(".bench.txt")]] = read_bench(p)
    return caps, lists, benches


def sanity(caps, lists, benches):
    for stem, (h, s) in caps.items():
        check_capture(stem, h, s)
    for stem, (h, s) in lists.items():
        check_launch_list(stem, h, s)
    for stem, (_, lines) in benches.items():
        check_bench(stem, lines)


def render(kind, stem, caps, lists, benches):
    if kind == "ncu":
        if stem not in caps:
            raise SystemExit(f"GEN:ncu:{stem}: no profiles/{stem}.ncu.txt")
        return block_ncu(stem, *caps[stem])
    if kind == "launches":
        if stem not in lists:
            raise SystemExit(f"GEN:launches:{stem}: no profiles/{stem}.launches.txt")
        return block_launches(stem, *lists[stem])
    if kind == "bench":
        if stem not in benches:
            raise SystemExit(f"GEN:bench:{stem}: no profiles/{stem}.bench.txt")
        return block_bench(stem, *benches[stem])
    if kind == "kernels":
        return block_kernels(caps)
    raise SystemExit(f"unknown generated block kind {kind!r}")


def regenerate(text, caps, lists, benches):
    def sub(m):
        body = render(m.group(2), m.group(3), caps, lists, benches)
        return f"{m.group(1)}\n{body.rstrip()}\n{m.group(5)}"
    return MARKER.sub(sub, text)


def generate(check=False, profiles=PROFILES):
    """Regenerate (or, with check, compare) every GEN block; returns the list
    of stale files."""
    caps, lists, benches = load_all(profiles)
    sanity(caps, lists, benches)
    stale = []
    for fn in sorted(os.listdir(profiles)):
        if not fn.endswith(".md"):
            continue
        p = os.path.join(profiles, fn)
        with open(p) as f:
            text = f.read()
        new = regenerate(text, caps, lists, benches)
        if new != text:
            stale.append(fn)
            if not check:
                with open(p, "w") as f:
                    f.write(new)
    return stale


# ---------------------------------------------------------------- queries

def traffic_ratio(stem, profiles=PROFILES):
    """DRAM bytes / algorithmic bytes of the capture's algorithmic kernel
    (first matching launch), or None when the archive is absent."""
    p = os.path.join(profiles, f"{stem}.ncu.txt")
    if not os.path.exists(p):
        return None
    header, secs = read_archive(p)
    alg = header.get("algorithmic_bytes")
    pat = re.compile(str(header.get("algorithmic_kernel") or "."))
    for _, m in secs:
        if alg and pat.search(m.get("kernel", "")) and m.get("dram_bytes"):
            return m["dram_bytes"] / alg
    return None


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("extract")
    e.add_argument("capture")
    e.add_argument("--name", required=True)
    e.add_argument("--command", required=True)
    e.add_argument("--algorithmic-bytes", type=int, default=None)
    e.add_argument("--algorithmic-kernel", default=None)
    e.add_argument("--note", default=None)
    ll = sub.add_parser("launches")
    ll.add_argument("csv")
    ll.add_argument("--name", required=True)
    ll.add_argument("--command", required=True)
    ll.add_argument("--top", default=None)
    b = sub.add_parser("bench")
    b.add_argument("--name", required=True)
    b.add_argument("--entry", nargs=2, action="append", required=True, metavar=("LOG", "COMMAND"))
    b.add_argument("--note", default=None)
    g = sub.add_parser("generate")
    g.add_argument("--check", action="store_true")
    a = ap.parse_args(argv)
    if a.cmd == "extract":
        print(extract(a.capture, a.name, a.command, a.algorithmic_bytes, a.algorithmic_kernel,
                      a.note))
    elif a.cmd == "launches":
        print(launches(a.csv, a.name, a.command, a.top))
    elif a.cmd == "bench":
        print(bench([tuple(e) for e in a.entry], a.name, a.note))
    else:
        stale = generate(check=a.check)
        if a.check and stale:
            print("stale generated blocks in: " + ", ".join(stale), file=sys.stderr)
            return 1
        print("up to date" if not stale else "regenerated: " + ", ".join(stale))
    return 0


if __name__ == "__main__":
    sys.exit(main())
