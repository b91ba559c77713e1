"""Regenerate the golden scan vectors in tests/golden/*.bin.

Compiles tests/golden/make_golden.cpp against the reference's own
Sources/CPURef/selective_scan_cpu.cpp (read in place from the reference
checkout; env MAMBA_REF overrides its location), writes the binary into
oracle/_ref/, runs it, and writes one .bin file per case next to this script.
Run it only where the reference checkout exists:

    python tests/golden/make_golden.py
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.build_oracle import reference_root  # noqa: E402


def main():
    cpu_dir = os.path.join(reference_root(), "Sources", "CPURef")
    ref_src = os.path.join(cpu_dir, "selective_scan_cpu.cpp")
    if not os.path.exists(ref_src):
        sys.exit("reference sources not found at %s" % cpu_dir)
    out_dir = os.path.join(ROOT, "oracle", "_ref")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "make_golden")
    subprocess.run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", cpu_dir,
                    os.path.join(HERE, "make_golden.cpp"), ref_src, "-o", exe], check=True)
    subprocess.run([exe, HERE], check=True)


if __name__ == "__main__":
    main()
