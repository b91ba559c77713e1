"""Build recipe for the CPU oracle (test infrastructure only).

Outputs:
  oracle/_build/liboracle.so   the C restatement (oracle/scan_ref.c)
  oracle/_ref/libref_scan.so   the reference's own Sources/CPURef/
                               selective_scan_cpu.cpp plus oracle/ref_shim.cpp,
                               compiled in place from the reference tree
                               (only when that tree is present; the prebuilt
                               library is what travels to GPU machines).

The reference tree is $MAMBA_REF, or by default a checkout named `reference`
next to this repository's root directory.

Both builds use -ffp-contract=off so the compiler never fuses a multiply and
an add, which keeps the restatement bit-identical to the reference build.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF_OUT = os.path.join(HERE, "_ref")
REPO = os.path.dirname(HERE)


def reference_root():
    """Location of the reference checkout: $MAMBA_REF when set, else a
    directory named `reference` beside this repository's root."""
    return os.environ.get("MAMBA_REF") or os.path.join(os.path.dirname(REPO), "reference")


def _run(cmd):
    subprocess.run(cmd, check=True)


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build_restatement(force=False):
    os.makedirs(BUILD, exist_ok=True)
    src = os.path.join(HERE, "scan_ref.c")
    out = os.path.join(BUILD, "liboracle.so")
    if force or _stale(out, [src]):
        _run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fopenmp", "-fPIC",
              "-shared", src, "-o", out, "-lm"])
    return out


def build_reference(force=False):
    """Compile the reference's CPU oracle from its own sources, if present."""
    ref = reference_root()
    cpu_dir = os.path.join(ref, "Sources", "CPURef")
    ref_src = os.path.join(cpu_dir, "selective_scan_cpu.cpp")
    out = os.path.join(REF_OUT, "libref_scan.so")
    if not os.path.exists(ref_src):
        if os.environ.get("MAMBA_REF"):
            raise FileNotFoundError("MAMBA_REF=%s has no Sources/CPURef/selective_scan_cpu.cpp" % ref)
        # No checkout here (e.g. a GPU machine): use the prebuilt library if
        # it travelled with the tree.
        return out if os.path.exists(out) else None
    os.makedirs(REF_OUT, exist_ok=True)
    shim = os.path.join(HERE, "ref_shim.cpp")
    if force or _stale(out, [ref_src, shim]):
        _run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fPIC", "-shared",
              "-pthread", "-I", cpu_dir, ref_src, shim, "-o", out])
    return out


def build_all(force=False):
    a = build_restatement(force)
    b = build_reference(force)
    return a, b


if __name__ == "__main__":
    print(build_all(force="--force" in sys.argv))
