"""Cut small ncu CSV samples for the roofline parser tests from real exports.

  python tests/golden/make_ncu_samples.py RAW.csv LAUNCHES.csv

RAW.csv is ``ncu -i REP --page raw --csv`` of an attention capture; the
sample keeps the ID / Kernel Name columns and the metrics the parser reads
(header, units row and every launch). LAUNCHES.csv is a launch list
(``ncu --metrics gpu__time_duration.sum --csv --log-file ...``); the sample
keeps its preamble, header, the first 4 launches and the first 12 launches
each of the attention and softmax kernels.
"""
import csv
import io
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "vla-kernels_b200"))
import roofline  # noqa: E402


def main(raw_path: str, launches_path: str):
    rows = list(csv.reader(io.StringIO(roofline._clean_lines(raw_path))))
    keep = [i for i, h in enumerate(rows[0]) if h in ("ID", "Kernel Name") or h in roofline.METRICS]
    with open(os.path.join(HERE, "ncu_raw_sample.csv"), "w", newline="") as f:
        w = csv.writer(f, quoting=csv.QUOTE_ALL)
        for r in rows:
            w.writerow([r[i] for i in keep])
    lines = open(launches_path).read().splitlines(keepends=True)
    pre = [ln for ln in lines if ln.startswith("==")]
    body = [ln for ln in lines if not ln.startswith("==")]
    pick = body[1:5] + [ln for ln in body if "gqa_attention" in ln][:12] + \
        [ln for ln in body if "softmax" in ln][:12]
    with open(os.path.join(HERE, "ncu_launches_sample.csv"), "w") as f:
        f.writelines(pre[:3] + body[:1] + pick)


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2])
