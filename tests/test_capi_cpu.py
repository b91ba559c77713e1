"""CPU tests of the C ABI boundary (no kernel launches).

* libmamba_b200.so loads and exports every function include/mamba.h declares.
* The header compiles as C, and the struct layouts the ctypes binding uses
  equal the C compiler's (sizeof / offsetof probe).
* Error convention of the reference C API (Sources/Mamba/MambaRuntime.cpp:
  134-179): NULL handles give -1 / NULL, never a crash.
"""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import mamba_b200 as mb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mamba.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(mamba_\w+)\s*\(", text)
    return sorted(set(names))


def test_header_declares_reference_api():
    names = set(declared_functions())
    reference_api = {"mamba_create", "mamba_destroy", "mamba_load_weights", "mamba_forward",
                     "mamba_create_state", "mamba_reset_state", "mamba_step",
                     "mamba_destroy_state"}
    assert reference_api <= names


def test_library_exports_every_declared_symbol():
    L = mb.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", mb.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mamba_\w+)", out))
    for name in declared_functions():
        assert name in exported, name
        assert hasattr(L, name)
    assert set(mb._PROTOTYPES) == set(declared_functions())


PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "mamba.h"
int main(void) {
  printf("%zu %zu %zu %zu\n", sizeof(MambaConfig), offsetof(MambaConfig, n_layer),
         offsetof(MambaConfig, dtype), sizeof(MambaScanArgs));
  printf("%zu %zu %zu %zu\n", offsetof(MambaScanArgs, batch), offsetof(MambaScanArgs, chunk_len),
         offsetof(MambaScanArgs, x_stride), offsetof(MambaScanArgs, y_stride));
  return 0;
}
"""


def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), str(src),
                    "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    a = list(map(int, lines[0].split()))
    b = list(map(int, lines[1].split()))
    # Reference MambaConfig: 24 bytes, n_layer @16, dtype @20.
    assert a[:3] == [24, 16, 20]
    assert a[0] == ctypes.sizeof(mb.MambaConfig)
    assert a[3] == ctypes.sizeof(mb.MambaScanArgs)
    assert b == [mb.MambaScanArgs.batch.offset, mb.MambaScanArgs.chunk_len.offset,
                 mb.MambaScanArgs.x_stride.offset, mb.MambaScanArgs.y_stride.offset]


def test_c_example_compiles(tmp_path):
    """examples/simple_forward.c (the reference's commented-out usage,
    Examples/simple_forward.c:10-39, made real) compiles and links as C."""
    exe = tmp_path / "simple_forward"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER),
                    os.path.join(ROOT, "examples", "simple_forward.c"), "-o", str(exe),
                    "-L", os.path.dirname(mb.LIB_PATH), "-lmamba_b200",
                    "-Wl,-rpath," + os.path.dirname(mb.LIB_PATH), "-lm"], check=True)
    assert exe.exists()


def test_null_handles_return_errors():
    L = mb.lib()
    assert L.mamba_create(None) is None
    assert "null config" in mb.last_error()
    assert L.mamba_load_weights(None, None, 0) == -1
    assert L.mamba_forward(None, None, None, 1, 1) == -1
    assert L.mamba_create_state(None, 1) is None
    assert L.mamba_step(None, None, None, None) == -1
    L.mamba_destroy(None)
    L.mamba_destroy_state(None)
    L.mamba_reset_state(None)
    assert L.mamba_state_batch(None) == -1
    assert L.mamba_selective_scan(None, None, 0, None) == -1
    assert L.mamba_forward_device(None, None, None, 1, 1, None) == -1


def test_bad_configs_rejected():
    L = mb.lib()
    for bad in [mb.MambaConfig(0, 16, 4, 2, 1, 1), mb.MambaConfig(64, 17, 4, 2, 1, 1),
                mb.MambaConfig(64, 16, 9, 2, 1, 1), mb.MambaConfig(64, 16, 4, 2, 0, 1),
                mb.MambaConfig(64, 16, 4, 2, 1, 7)]:
        assert L.mamba_create(ctypes.byref(bad)) is None
        assert L.mamba_weights_blob_size(ctypes.byref(bad)) == 0


def test_scan_args_validation_without_gpu():
    """Argument checks run before any device work."""
    a = mb.MambaScanArgs()
    a.batch, a.seqlen, a.dim, a.dstate = 1, 4, 8, 17
    assert mb.lib().mamba_selective_scan(ctypes.byref(a), None, 0, None) == -1
    assert "dstate" in mb.last_error()


def test_blob_size_and_dt_rank():
    L = mb.lib()
    for (M, N, K, E, nl) in [(768, 16, 4, 2, 1), (2048, 16, 4, 2, 3), (2560, 16, 4, 2, 2),
                             (100, 5, 3, 3, 2)]:
        cfg = mb.MambaConfig(M, N, K, E, nl, 1)
        assert L.mamba_dt_rank(ctypes.byref(cfg)) == -(-M // 16)
        rng = np.random.default_rng(0)
        blob = mb.make_weight_blob(cfg, [mb.random_layer_weights(cfg, rng) for _ in range(nl)]) \
            if M <= 768 else None
        expect = 64 + 4 * nl * sum(int(np.prod(s)) for s in mb.layer_shapes(cfg).values())
        assert L.mamba_weights_blob_size(ctypes.byref(cfg)) == expect
        if blob is not None:
            assert len(blob) == expect
    # dt_rank values of the standard configs: 768->48, 2048->128, 2560->160
    assert [mb.MambaConfig(m, 16, 4, 2, 1, 1).dt_rank for m in (768, 2048, 2560)] == [48, 128, 160]


def test_create_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    cfg = mb.MambaConfig(64, 16, 4, 2, 1, 1)
    assert mb.lib().mamba_create(ctypes.byref(cfg)) is None
    assert mb.last_error() != ""


_LOG_PROBE = """
import ctypes, mamba_b200 as mb
cfg = mb.MambaConfig(0, 16, 4, 2, 1, mb.F16)  # d_model 0: rejected before any CUDA call
assert mb.lib().mamba_create(ctypes.byref(cfg)) is None
print(mb.last_error())
"""


@pytest.mark.parametrize("level", [None, "1"])
def test_mamba_log_levels(level):
    """MAMBA_LOG >= 1 copies every error onto stderr as one line prefixed
    'mamba-b200:' (the reference's 'mamba-metal:' one-liners); unset, the
    library writes nothing."""
    env = dict(os.environ)
    env.pop("MAMBA_LOG", None)
    if level:
        env["MAMBA_LOG"] = level
    env["PYTHONPATH"] = os.path.join(ROOT, "mamba-metal_b200") + os.pathsep + env.get("PYTHONPATH", "")
    r = subprocess.run(["python", "-c", _LOG_PROBE], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr
    assert "mamba_create" in r.stdout
    lines = [l for l in r.stderr.splitlines() if l.startswith("mamba-b200:")]
    if level:
        assert len(lines) == 1 and "error: mamba_create:" in lines[0]
    else:
        assert lines == []
