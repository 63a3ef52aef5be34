#!/usr/bin/env python3
"""Regenerate the golden fixtures in tests/golden/ from the reference sources.

The reference (Anemll/fp8-mlp-metal41-bench) is Swift + Metal and cannot run
on Linux, and it ships no golden-vector files.  What it does ship are constant
tables inside its sources and published run output.  This script reads those
as TEXT (it executes nothing from the reference) and writes them as JSON:

  reference_tables.json
    e2m1_to_e4m3_lut   fp8_mlp.metal:305-309 (kE2M1ToE4M3)
    e2m1_magnitudes    main.swift:45         (e2m1ToFloat's mag table)
    e2m1_code_cycle    main.swift:51         (e2m1Code)
    ue8m0_code_cycle   main.swift:81         (ue8m0Code)
    tiles              main.swift:142-143
    suite_shapes       main.swift:156-160
    dtypes             main.swift:85-95 (raw values)
  reference_outputs.json
    tables             every published result table (README.md, the M5 Max
                       autotune log), each as its header, rule and raw lines
    log_lines          the header / autotune / running lines of the log
    profiles           the two published profile JSON files, verbatim

Run:  python tests/golden/make_golden.py /path/to/reference
The committed JSON is what the tests read; the reference tree is not needed
at test time.
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _read(ref, rel):
    with open(os.path.join(ref, rel), encoding="utf-8") as f:
        return f.read()


def _array_after(text, anchor, open_ch="[", close_ch="]"):
    i = text.index(anchor)
    j = text.index(open_ch, i) + len(open_ch)
    k = text.index(close_ch, j)
    return text[j:k], text[:i].count("\n") + 1


def tables(ref):
    metal = _read(ref, "fp8_mlp.metal")
    swift = _read(ref, "main.swift")
    body, lut_line = _array_after(metal, "kE2M1ToE4M3[16]", "{", "}")
    lut = [int(t, 16) for t in re.findall(r"0x[0-9A-Fa-f]+", body)]
    mag_body, mag_line = _array_after(swift, "let mag: [Float] =", "= [", "]")
    mags = [float(t) for t in mag_body.split(",")]
    e2_body, e2_line = _array_after(swift, "func e2m1Code", "[0x", "]")
    e2 = [int(t, 16) for t in re.findall(r"0x[0-9A-Fa-f]+", "0x" + e2_body)]
    ue_i = swift.index("func ue8m0Code")
    ue_body = swift[swift.index("= [", ue_i) + 3:swift.index("]", swift.index("= [", ue_i))]
    ue = [int(t) for t in ue_body.split(",")]
    tiles = [f"{a}x{b}" for a, b in re.findall(r"Tile\(bm: (\d+), bn: (\d+)\)",
                                               swift[swift.index("let tiles = ["):swift.index("// Best measured")])]
    suite = [dict(name=n, N=int(a), K=int(b), M=int(c), iters=int(d)) for n, a, b, c, d in re.findall(
        r'ShapeCase\(name: "(\w+)", N: (\d+), K: (\d+), M: (\d+), iters: (\d+)\)', swift)]
    dts = []
    enum = swift[swift.index("enum DType"):swift.index("var kernel")]
    for line in enum.splitlines():
        m = re.match(r'\s*case (\w+)(?: = "([^"]+)")?', line)
        if m:
            dts.append(m.group(2) or m.group(1))
    return {
        "source": "Anemll/fp8-mlp-metal41-bench (read as text by tests/golden/make_golden.py)",
        "e2m1_to_e4m3_lut": {"where": f"fp8_mlp.metal:{lut_line}", "values": lut},
        "e2m1_magnitudes": {"where": f"main.swift:{mag_line}", "values": mags},
        "e2m1_code_cycle": {"where": f"main.swift:{e2_line}", "values": e2},
        "ue8m0_code_cycle": {"where": "main.swift:80-83", "values": ue},
        "tiles": {"where": "main.swift:142-143", "values": tiles},
        "suite_shapes": {"where": "main.swift:156-160", "values": suite},
        "dtypes": {"where": "main.swift:85-95", "values": dts},
    }


_ROW = re.compile(r"^(square|thin|fat|custom)\s+\d+\s+\d+\s+\d+\s+\S+\s+\S+\s+[\d.]+\s+[\d.]+\s+\S+\s+\S+$")


def _tables_in(text, where):
    out = []
    lines = text.splitlines()
    for i, line in enumerate(lines):
        if line.startswith("shape ") and "median_ms" in line and i + 1 < len(lines) \
                and set(lines[i + 1]) == {"-"}:
            rows = []
            j = i + 2
            while j < len(lines) and _ROW.match(lines[j]):
                rows.append(lines[j])
                j += 1
            out.append({"where": f"{where}:{i + 1}-{j}", "header": line,
                        "rule": lines[i + 1], "rows": rows})
    return out


def outputs(ref):
    readme = _read(ref, "README.md")
    log = _read(ref, "result_m5max_autotune.txt")
    tabs = _tables_in(readme, "README.md") + _tables_in(log, "result_m5max_autotune.txt")
    keep = [l for l in log.splitlines() if l.split(":")[0] in
            ("device", "timing", "dtypes", "shapes", "architecture", "tiles", "wrote profile")
            or l.startswith("autotune ") or l.startswith("running ") or l == "ok"]
    profs = {}
    pdir = os.path.join(ref, "profiles")
    for name in sorted(os.listdir(pdir)):
        if name.endswith(".json"):
            profs[name] = _read(ref, os.path.join("profiles", name))
    return {"source": "Anemll/fp8-mlp-metal41-bench published output (read as text)",
            "tables": tabs, "log_lines": keep, "profiles": profs}


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the reference checkout>")
    ref = sys.argv[1]
    for name, obj in (("reference_tables.json", tables(ref)),
                      ("reference_outputs.json", outputs(ref))):
        path = os.path.join(HERE, name)
        with open(path, "w", encoding="utf-8") as f:
            json.dump(obj, f, indent=1, sort_keys=True)
            f.write("\n")
        print("wrote", path)


if __name__ == "__main__":
    main()
