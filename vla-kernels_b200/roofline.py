#!/usr/bin/env python3
"""Nsight Compute CSV -> per-kernel roofline figures on B200.

The reference classifies kernels from an ``ncu --csv`` export with Speed-of-
Light thresholds (bench/roofline.py:19-62). This module keeps that classifier
(same thresholds, 60 / 20 % of peak) and adds what the B200 evidence needs:
DRAM bytes per launch, achieved DRAM bandwidth against the measured HBM copy
peak (MEASURED_PEAKS.json), the tensor-pipe share, the launch-list shares, and
the traffic check against a kernel's algorithmic bytes.

Two CSV forms are read:
  long  ``ncu --csv ...`` or ``ncu -i REP --page details --csv``: one row per
        (launch, metric) with "Metric Name" / "Metric Unit" / "Metric Value"
        (also the launch list of ``--metrics gpu__time_duration.sum``);
  wide  ``ncu -i REP --page raw --csv``: one row per launch, metric names as
        columns and a row of units under the header.

  python vla-kernels_b200/roofline.py FILE.csv [--peaks MEASURED_PEAKS.json]
         [--kernel REGEX] [--algorithmic-bytes N] [--hi 60] [--lo 20]
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import re
import statistics
import sys

# metric (raw name or Speed-of-Light section name) -> canonical key
METRICS = {
    "gpu__time_duration.sum": "duration_ns",
    "Duration": "duration_ns",
    "dram__bytes_read.sum": "dram_read_bytes",
    "dram__bytes_write.sum": "dram_write_bytes",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": "dram_pct",
    "DRAM Throughput": "dram_pct",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed": "sm_pct",
    "Compute (SM) Throughput": "sm_pct",
    "gpu__compute_memory_throughput.avg.pct_of_peak_sustained_elapsed": "mem_pct",
    "Memory Throughput": "mem_pct",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": "tensor_pct",
    "sm__inst_executed_pipe_xu.avg.pct_of_peak_sustained_active": "xu_pct",
    "smsp__issue_active.avg.pct_of_peak_sustained_active": "issue_pct",
    "sm__warps_active.avg.pct_of_peak_sustained_active": "warps_active_pct",
    "Achieved Occupancy": "warps_active_pct",
    "lts__t_sector_hit_rate.pct": "l2_hit",
    "L2 Hit Rate": "l2_hit",
    "L1/TEX Hit Rate": "l1_hit",
    "launch__registers_per_thread": "registers",
    "Registers Per Thread": "registers",
    "l1tex__t_bytes_pipe_lsu_mem_local_op_ld.sum": "local_ld_bytes",
    "l1tex__t_bytes_pipe_lsu_mem_local_op_st.sum": "local_st_bytes",
}

# unit -> factor to the canonical unit (bytes, nanoseconds, percent, count)
_SCALE = {
    "byte": 1.0, "kbyte": 1e3, "mbyte": 1e6, "gbyte": 1e9, "tbyte": 1e12,
    "kibyte": 1024.0, "mibyte": 1024.0 ** 2, "gibyte": 1024.0 ** 3,
    "nsecond": 1.0, "ns": 1.0, "usecond": 1e3, "us": 1e3, "msecond": 1e6, "ms": 1e6,
    "second": 1e9, "s": 1e9,
}


def _value(raw: str, unit: str) -> float | None:
    raw = (raw or "").replace(",", "").strip()
    try:
        v = float(raw)
    except ValueError:
        return None
    return v * _SCALE.get((unit or "").strip().lower(), 1.0)


def _clean_lines(path: str) -> str:
    with open(path, newline="") as f:
        # ncu's preamble (==PROF== / ==WARNING== lines) precedes the header
        return "".join(ln for ln in f if not ln.startswith(("==", "\x00")))


def parse(path: str) -> dict:
    """{(launch id, kernel name): {canonical key: value}} in launch order,
    from either CSV form. Values are in bytes, nanoseconds, percent or
    counts."""
    text = _clean_lines(path)
    rows = list(csv.reader(io.StringIO(text)))
    if not rows:
        return {}
    hdr = rows[0]
    kernels: dict = {}
    if "Metric Name" in hdr:  # long form
        ix = {h: i for i, h in enumerate(hdr)}
        for r in rows[1:]:
            if len(r) < len(hdr):
                continue
            key = METRICS.get(r[ix["Metric Name"]].strip())
            if key is None:
                continue
            v = _value(r[ix["Metric Value"]], r[ix["Metric Unit"]] if "Metric Unit" in ix else "")
            if v is not None:
                kernels.setdefault((r[ix["ID"]], r[ix["Kernel Name"]].strip()), {})[key] = v
        return kernels
    # wide form: header, units, then one row per launch
    units = rows[1] if len(rows) > 1 else [""] * len(hdr)
    ix = {h: i for i, h in enumerate(hdr)}
    for r in rows[2:]:
        if len(r) < len(hdr):
            continue
        m = {}
        for name, key in METRICS.items():
            i = ix.get(name)
            if i is None:
                continue
            v = _value(r[i], units[i])
            if v is not None:
                m[key] = v
        kernels[(r[ix.get("ID", 0)], r[ix.get("Kernel Name", 1)].strip())] = m
    return kernels


def classify(sm, mem, hi: float = 60.0, lo: float = 20.0) -> str:
    """The reference's Speed-of-Light classes (bench/roofline.py:31-41)."""
    if sm is None or mem is None:
        return "unknown"
    if sm >= hi and sm >= mem:
        return "compute-bound"
    if mem >= hi and mem > sm:
        return "bandwidth-bound"
    if sm < lo and mem < lo:
        return "latency/occupancy-bound"
    return "balanced"


def load_peaks(path: str | None = None) -> tuple[dict, str]:
    """MEASURED_PEAKS.json (hbm_gbs, bf16_tflops); the pool's earlier
    measurement (6650 GB/s, 1590 TFLOP/s) when it is absent."""
    if path is None:
        path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def roofline(m: dict, peaks: dict, algorithmic_bytes: float | None = None) -> dict:
    """Roofline figures of one launch: DRAM bytes (read + write), achieved DRAM
    GB/s and its fraction of the measured HBM copy peak, tensor-pipe share, the
    SOL class, and traffic over algorithmic bytes when those are given."""
    out: dict = {}
    rd, wr = m.get("dram_read_bytes"), m.get("dram_write_bytes")
    if rd is not None and wr is not None:
        out["dram_bytes"] = rd + wr
        dur = m.get("duration_ns")
        if dur:
            gbs = (rd + wr) / dur  # bytes per ns = GB/s
            out["dram_gbs"] = gbs
            out["frac_hbm"] = gbs / peaks["hbm_gbs"]
        if algorithmic_bytes:
            out["traffic_over_algorithmic"] = (rd + wr) / algorithmic_bytes
    for k in ("dram_pct", "tensor_pct", "xu_pct", "issue_pct", "warps_active_pct", "registers",
              "local_ld_bytes", "local_st_bytes"):
        if k in m:
            out[k] = m[k]
    out["class"] = classify(m.get("sm_pct"), m.get("mem_pct"))
    return out


def launch_shares(kernels: dict) -> list[dict]:
    """Per kernel name: launches, total device time and share of the total,
    from a launch list (gpu__time_duration.sum per launch), largest first."""
    agg: dict = {}
    for (_, name), m in kernels.items():
        d = m.get("duration_ns")
        if d is None:
            continue
        a = agg.setdefault(name, [0, 0.0])
        a[0] += 1
        a[1] += d
    total = sum(v[1] for v in agg.values()) or 1.0
    out = [{"kernel": k, "launches": v[0], "total_ms": v[1] / 1e6, "share": v[1] / total,
            "us_per_launch": v[1] / v[0] / 1e3} for k, v in agg.items()]
    return sorted(out, key=lambda r: -r["total_ms"])


def kernel_traffic(path: str, kernel_regex: str) -> float | None:
    """Median DRAM bytes (read + write) per launch of the kernels matching
    kernel_regex in an ncu CSV, or None."""
    pat = re.compile(kernel_regex)
    vals = [m["dram_read_bytes"] + m["dram_write_bytes"] for (_, name), m in parse(path).items()
            if pat.search(name) and "dram_read_bytes" in m and "dram_write_bytes" in m]
    return statistics.median(vals) if vals else None


def _strip_group(n: str, open_ch: str, close_ch: str) -> str:
    """n without a trailing bracketed group (its matching bracket found by
    scanning back from the end)."""
    n = n.rstrip()
    if not n.endswith(close_ch):
        return n
    depth = 0
    for i in range(len(n) - 1, -1, -1):
        depth += n[i] == close_ch
        depth -= n[i] == open_ch
        if depth == 0:
            return n[:i]
    return n


def short(name: str, width: int, templates: bool = True) -> str:
    """A kernel's name without return type, namespaces or parameter list, and
    without its template arguments unless `templates`:
    "void ns::k<float, 4>(int)" -> "k<float, 4>" (or "k")."""
    n = _strip_group(name, "(", ")")
    if not templates:
        n = _strip_group(n, "<", ">")
    depth, cut = 0, 0  # the last "::" outside template brackets
    for i, ch in enumerate(n):
        depth += ch == "<"
        depth -= ch == ">" and depth > 0
        if depth == 0 and n.startswith("::", i):
            cut = i + 2
    n = n[cut:].strip()
    if n.startswith("void "):
        n = n[5:]
    return (n or name)[:width]


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("csv")
    ap.add_argument("--peaks", default=None)
    ap.add_argument("--kernel", default=None, help="only kernels whose name matches this regex")
    ap.add_argument("--algorithmic-bytes", type=float, default=None)
    ap.add_argument("--hi", type=float, default=60.0)
    ap.add_argument("--lo", type=float, default=20.0)
    a = ap.parse_args(argv)
    kernels = parse(a.csv)
    if not kernels:
        sys.exit("no kernel metrics found: expected an ncu --csv export (long or --page raw)")
    if a.kernel:
        pat = re.compile(a.kernel)
        kernels = {k: v for k, v in kernels.items() if pat.search(k[1])}
    peaks, src = load_peaks(a.peaks)
    only_time = all(set(m) <= {"duration_ns"} for m in kernels.values())
    if only_time:
        print(f"{'kernel':48} {'launches':>8} {'total_ms':>9} {'share':>7} {'us/launch':>10}")
        for r in launch_shares(kernels):
            print(f"{short(r['kernel'], 48):48} {r['launches']:8d} {r['total_ms']:9.3f} "
                  f"{100 * r['share']:6.1f}% {r['us_per_launch']:10.2f}")
        return 0
    print(f"peaks: HBM {peaks['hbm_gbs']} GB/s ({src})")
    hdr = (f"{'kernel':36} {'id':>3} {'dur_us':>8} {'DRAM_MB':>9} {'GB/s':>7} {'fHBM':>6} "
           f"{'DRAM%':>6} {'tens%':>6} {'issue%':>6}  class")
    print(hdr)
    print("-" * len(hdr))
    for (kid, name), m in kernels.items():
        r = roofline(m, peaks, a.algorithmic_bytes)
        f = lambda k, fmt: format(r[k], fmt) if k in r else "-"  # noqa: E731
        dur = m.get("duration_ns")
        print(f"{short(name, 36):36} {kid:>3} {dur / 1e3 if dur else 0:8.2f} "
              f"{r['dram_bytes'] / 1e6 if 'dram_bytes' in r else 0:9.2f} {f('dram_gbs', '7.0f'):>7} "
              f"{f('frac_hbm', '6.3f'):>6} {f('dram_pct', '6.1f'):>6} {f('tensor_pct', '6.1f'):>6} "
              f"{f('issue_pct', '6.1f'):>6}  {r['class']}")
    return 0


if __name__ == "__main__":
    try:
        sys.exit(main())
    except BrokenPipeError:  # output piped into head and the like
        sys.exit(0)
