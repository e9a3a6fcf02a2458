"""Extract the reference's recorded mel-probe statistics.

Run where the reference tree is checked out, with its path as the only
argument: python tests/golden/make_mel_probe_stats.py <reference checkout>.
The reference's mel probe (tests/test_mel_cpu.cpp) compares its serial DFT
mel (the production path) with a double-precision FFT transform of the same
windowed samples on six signals, and cpu-lab/mel-kernel-v1.jsonl records, per
signal, how many of the 240,000 mel values differ in their float bits and the
largest and RMS differences.  This script copies the FFT rows (opt 4096, one
thread) into tests/golden/mel_probe_fft_stats.json, so the test that
reproduces them never reads the reference at run time.
"""
import json
import os
import sys


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_mel_probe_stats.py <reference checkout>")
    src = os.path.join(sys.argv[1], "cpu-lab", "mel-kernel-v1.jsonl")
    rows = {}
    for line in open(src):
        d = json.loads(line)
        if d.get("opt") == 4096 and d.get("threads") == 1:
            rows[d["signal"]] = {k: d[k] for k in ("floatBitDifferences", "maxAbsError", "rmsError")}
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mel_probe_fft_stats.json")
    with open(out, "w") as f:
        json.dump({"source": "cpu-lab/mel-kernel-v1.jsonl (opt 4096, threads 1)", "signals": rows}, f, indent=1)
    print(f"wrote {out}: {sorted(rows)}")


if __name__ == "__main__":
    main()
