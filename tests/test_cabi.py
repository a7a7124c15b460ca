"""CPU: the C-ABI library loads, exports exactly what include/kbb200.h
declares, and rejects bad arguments on the host before touching a GPU."""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "kbb200.h"


def declared_functions() -> list[str]:
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(kb_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "kb_gelu_tanh_f32" in names and "kb_gemv_f32" in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    from kbb200 import _lib

    lib = C.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_binding_table_matches_header():
    from kbb200 import _lib

    assert sorted(_lib.SIGNATURES) == declared_functions()
    # parameter counts agree with the header prototypes
    src = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", src)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), name


def test_only_c_abi_symbols_are_public():
    import subprocess

    from kbb200 import _lib

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True).stdout
    syms = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert {s for s in syms if s.startswith("kb_")} == set(declared_functions())


def test_version_and_status_strings():
    from kbb200 import LIB

    assert LIB.kb_version() >= 100
    assert LIB.kb_status_string(0) == b"ok"
    assert LIB.kb_status_string(3) == b"workspace too small"
    assert isinstance(LIB.kb_last_error(), bytes)


@pytest.mark.parametrize("fn", ["kb_gelu_tanh_f32", "kb_gelu_erf_f32", "kb_swish_f32", "kb_relu_f32"])
def test_elementwise_rejects_negative_n(fn):
    from kbb200 import LIB

    assert getattr(LIB, fn)(None, None, -1, None) == 1  # KB_ERR_INVALID_ARG
    assert b"negative" in LIB.kb_last_error()


def test_empty_inputs_are_noops():
    from kbb200 import LIB

    assert LIB.kb_relu_f32(None, None, 0, None) == 0
    assert LIB.kb_layernorm_f32(None, None, None, None, 0, 8, 1e-5, None) == 0
    assert LIB.kb_softmax_f32(None, None, 4, 0, None) == 0


def test_workspace_checks_happen_on_host():
    from kbb200 import LIB

    need = LIB.kb_mse_workspace_size(1 << 20)
    assert need >= 8
    # no workspace -> KB_ERR_WORKSPACE before any launch
    assert LIB.kb_mse_f32(1, 1, 1, 1 << 20, None, 0, None) == 3
    assert LIB.kb_frobenius_normalize_f32(1, 1, 16, None, 0, None) == 3
    assert LIB.kb_batchnorm_train_f32(1, None, None, 1, 2, 3, 4, 1e-5, 0.1, None, None, None, 0, None) == 3
    assert LIB.kb_batchnorm_workspace_size(64, 128, 65536) >= 128 * 16


def test_maxpool_validates_window_on_host():
    from kbb200 import LIB

    # output extent that does not match k3 s2 p1 on 8x8 -> invalid
    assert LIB.kb_maxpool2d_f32(1, 1, 1, 1, 8, 8, 5, 5, 3, 2, 1, 1, None) == 1
    assert LIB.kb_maxpool2d_f32(1, 1, 1, 1, 8, 8, 4, 4, 3, 2, 2, 1, None) == 1  # pad > k/2


def test_argmax_rejects_empty_reduced_dim():
    from kbb200 import LIB

    assert LIB.kb_argmax_dim1_f32(None, 1, 2, 0, 3, None) == 1


def test_a_c_program_compiles_links_and_calls_the_abi(tmp_path):
    """The header is plain C: a C translation unit includes it, links
    -lkbb200 and calls host-side entries (no GPU needed for these), as a
    non-Python host would."""
    import os
    import subprocess

    from kbb200 import _lib

    src = tmp_path / "abi.c"
    src.write_text(r'''
#include <stdio.h>
#include "kbb200.h"
int main(void) {
  const char* s = kb_status_string(KB_ERR_WORKSPACE);
  size_t ws = kb_sharded_workspace_size();
  size_t buf = kb_p2p_buffer_bytes(16, 8);
  size_t mse = kb_mse_workspace_size(1000);
  int st = kb_gelu_tanh_f32(0, 0, -1, 0);   /* negative size: rejected on the host */
  printf("%d %s %zu %zu %zu %d\n", kb_version(), s, ws, buf, mse, st);
  return 0;
}
''')
    lib_dir = _lib.LIB_PATH.parent
    exe = tmp_path / "abi"
    cuda_inc = "/usr/local/cuda/include"
    r = subprocess.run(["gcc", "-std=c99", "-I", str(REPO / "include"), "-I", cuda_inc, str(src), "-L", str(lib_dir),
                        "-lkbb200", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    env = dict(os.environ, LD_LIBRARY_PATH=f"{lib_dir}:{os.environ.get('LD_LIBRARY_PATH', '')}")
    out = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=60)
    assert out.returncode == 0, out.stderr
    ver, *rest = out.stdout.split()
    assert int(ver) > 0 and int(rest[-1]) == 1  # KB_ERR_INVALID_ARG
    assert int(rest[-4]) == 256 + 2048 * 8 and int(rest[-3]) == 4096 + 2 * 8 * 256
