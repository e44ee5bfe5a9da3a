"""Regenerates tests/golden/golden.npz from the reference's own code.

Builds the reference compiler from its sources (oracle/Makefile.ref, outputs
in oracle/_ref/), emits the reference CPU units for oracle/models/*.ns,
compiles tests/golden/gen_golden.cpp against one emitted unit plus the
shared input generator, runs it, and packs every array it writes into one
compressed archive. Needs the reference sources: set NS_REFERENCE to the reference
checkout. It runs on a build host, never on the GPU box.

    python tests/golden/gen_golden.py
"""
import glob
import os
import subprocess
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF = os.environ.get("NS_REFERENCE")
FLAGS = ["-O3", "-march=x86-64-v3"]


def run(cmd, **kw):
    print("+", " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=ROOT, **kw)


def main():
    if not REF or not os.path.isdir(os.path.join(REF, "src")):
        sys.exit("set NS_REFERENCE to the reference source tree")
    run(["make", "-s", "-f", "oracle/Makefile.ref", f"REF={REF}", "-j8"])
    ref_dir = os.path.join(ROOT, "oracle", "_ref")
    with tempfile.TemporaryDirectory() as tmp:
        rnd = os.path.join(tmp, "nsrand.o")
        run(["gcc", *FLAGS, "-ffp-contract=off", "-fPIC", "-c", "oracle/nsrand.c", "-o", rnd])
        exe = os.path.join(tmp, "gen_golden")
        run(["g++", "-std=c++17", *FLAGS, f'-DREF_TU="{ref_dir}/tmlp.cpp"', f'-DREF_DIR="{ref_dir}"',
             "tests/golden/gen_golden.cpp", rnd, "-o", exe, "-ldl"])
        out = os.path.join(tmp, "out")
        os.makedirs(out)
        run([exe, out])
        arrays = {os.path.basename(f)[:-4]: np.load(f) for f in sorted(glob.glob(os.path.join(out, "*.npy")))}
    dst = os.path.join(ROOT, "tests", "golden", "golden.npz")
    np.savez_compressed(dst, **arrays)
    print(f"wrote {len(arrays)} arrays to {dst} ({os.path.getsize(dst)} bytes)")


if __name__ == "__main__":
    sys.exit(main())
