"""Generate tests/golden/reference_absmax.json by running the REFERENCE on a B200.

Runs the reference kernel (tests/side_aware.cu of QuickRunCUDA, compiled from
its sources into oracle/_ref/ by oracle/Makefile) and records C[0]:
  * through the reference harness itself (oracle/_ref/QuickRunCUDA, built from
    QuickRunCUDA.cpp) on its own `-r` fill (mt19937_64 per 1 Mi-dword chunk,
    QuickRunCUDA.cpp:432-457), with the cubin passed via --reuse-cubin;
  * through this repository's harness on the seeded uniform inputs of the
    benchmark configurations (the reference harness cannot produce them);
  * with DEBUG_STORE_999_IN_A, the reference's known-answer hook.
The JSON is committed; test_oracle.py checks the CPU oracle reproduces every
recorded output from the same inputs.  Needs a GPU; usage:
    python tests/golden/make_reference_goldens.py [--out tests/golden/reference_absmax.json]
"""
from __future__ import annotations

import argparse
import json
import shutil
import subprocess
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REF = ROOT / "oracle" / "_ref"
HARNESS = ROOT / "quickruncuda_b200" / "bin" / "qrc_harness"

REF_RANDOM_CASES = [  # (seed, mask, n): the reference harness' own -r data
    (1234, 0x3FFFFFFF, 1 << 20),
    (1, 0xBF7FFFFF, 1 << 24),
    (2, 0xFFFFFFFF, 1 << 24),
    (3, 0x3F8FFFFF, 12_345_678),
    (4, 0x3FFFFFFF, 100_000_000),
    (5, 0xBFFFFFFF, 1_000_000_000),
]
UNIFORM_CASES = [  # (seed, outlier or 0, n): the synthetic inputs, reference kernel under our harness
    (0, 7.5, 1_048_576),
    (1, 7.5, 1_000_000_000),
    (11, 0.0, 4 << 20),
    (12, 2.5, 3 * (1 << 20) + 4),
]


def run(cmd, cwd):
    r = subprocess.run([str(c) for c in cmd], cwd=cwd, capture_output=True, text=True, timeout=900)
    if r.returncode != 0:
        raise RuntimeError(f"{cmd}\n{r.stdout[-2000:]}\n{r.stderr[-2000:]}")
    return r.stdout


def c0(path: Path) -> int:
    return int(np.fromfile(path, dtype=np.uint32)[0])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ROOT / "tests" / "golden" / "reference_absmax.json"))
    args = ap.parse_args()
    cases = []
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        shutil.copy(REF / "side_aware_ref.cubin", td / "output.cubin")
        for seed, mask, n in REF_RANDOM_CASES:
            out = td / "c.bin"
            cmd = [REF / "QuickRunCUDA", "--reuse-cubin", "-i", "-p", "-t", "1024", "-A", max(n, 1 << 21),
                   "-0", n, "-C", 1, "-T", 3, "-r", "--randomSeed", seed, "--randomMask", hex(mask),
                   "--dump-c", out]
            run(cmd, td)
            cases.append({"name": f"refharness_r_s{seed}_m{mask:08x}_n{n}", "harness": "reference",
                          "fill": "ref_random", "seed": seed, "mask": mask, "n": n, "c0_bits": c0(out),
                          "argv": "QuickRunCUDA --reuse-cubin -i -p -t 1024 -A %d -0 %d -C 1 -T 3 -r "
                                  "--randomSeed %d --randomMask %s --dump-c c.bin" % (max(n, 1 << 21), n, seed, hex(mask))})
            print(cases[-1]["name"], hex(cases[-1]["c0_bits"]), flush=True)
        for seed, outlier, n in UNIFORM_CASES:
            out = td / "c.bin"
            fill = f"uniform:{seed}" + (f":{outlier}" if outlier else "")
            run([HARNESS, "--cubin", REF / "side_aware_ref.cubin", "-i", "-p", "-t", "1024",
                 "-A", max(n, 1 << 21), "-0", n, "-C", 1, "-T", 3, "--fill-a", fill, "--dump-c", out], td)
            cases.append({"name": f"ourharness_uniform_s{seed}_o{outlier}_n{n}", "harness": "qrc_harness",
                          "fill": "uniform", "seed": seed, "outlier": outlier, "n": n, "c0_bits": c0(out)})
            print(cases[-1]["name"], hex(cases[-1]["c0_bits"]), flush=True)
        out = td / "c.bin"
        n = 1 << 22
        run([HARNESS, "--cubin", REF / "side_aware_ref_999.cubin", "-i", "-p", "-t", "1024", "-A", n, "-0", n,
             "-C", 1, "-T", 2, "--fill-a", "uniform:2", "--dump-c", out], td)
        cases.append({"name": "known_answer_999", "harness": "qrc_harness", "fill": "known_999", "n": n,
                      "c0_bits": c0(out)})
    doc = {"description": "C[0] of the reference kernel tests/side_aware.cu (built from source, -DNDEBUG) on a B200",
           "generator": "tests/golden/make_reference_goldens.py", "cases": cases}
    Path(args.out).write_text(json.dumps(doc, indent=1) + "\n")
    print("wrote", args.out)


if __name__ == "__main__":
    main()
