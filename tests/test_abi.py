"""The C-ABI library: it loads, exports every symbol the header declares, and
its structs have the layout the Python mirror uses.  No compute (CPU only)."""
import ctypes as C
import os
import re
import subprocess
import sys

import pytest

from tensor_logic_lang_b200 import abi

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "tl_cuda.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tl_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from tensor_logic_lang_b200 import build
    build.build()
    return abi.load_library()


def test_exports_match_header(lib):
    declared = header_functions()
    assert sorted(abi.EXPORTS) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", abi.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (tl_[a-z0-9_]+)", out))
    missing = [f for f in declared if f not in exported]
    assert not missing, missing
    for f in declared:
        assert getattr(lib, f) is not None


def test_struct_layout_matches_c(tmp_path):
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "tl_cuda.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(tl_index), sizeof(tl_ref),'
                   ' sizeof(tl_instr), sizeof(tl_equation), sizeof(tl_statement), sizeof(tl_init_opts),'
                   ' sizeof(tl_kernel_stats), offsetof(tl_statement, eq)); return 0;}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    want = [C.sizeof(abi.Index), C.sizeof(abi.Ref), C.sizeof(abi.Instr), C.sizeof(abi.Equation),
            C.sizeof(abi.Statement), C.sizeof(abi.InitOpts), C.sizeof(abi.KernelStats), abi.Statement.eq.offset]
    assert got == want


def header_defines():
    text = open(HEADER).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"^#define (TL_[A-Z0-9_]+)\s+(-?\d+)", text, re.M)}


def test_header_constants_match_the_python_mirror():
    # every numeric #define of the header against abi.py's copy
    d = header_defines()
    py = {k: getattr(abi, k) for k in dir(abi) if k.startswith("TL_") and isinstance(getattr(abi, k), int)}
    prefixed = {"TL_IX_": "IX_", "TL_OP_": "OP_", "TL_STMT_": "STMT_", "TL_PREC_": "PREC_", "TL_SHARD_": "SHARD_"}
    for k, v in d.items():
        if k in py:
            assert py[k] == v, k
            continue
        for hp, pp in prefixed.items():
            if k.startswith(hp):
                assert getattr(abi, pp + k[len(hp):]) == v, k
                break
        else:
            if k.startswith("TL_NL_"):
                assert abi.NL[k[len("TL_NL_"):].lower()] == v, k
            elif k.startswith("TL_ACC_"):
                sym = {"ASSIGN": "=", "ADD": "+=", "MUL": "*=", "MAX": "max=", "MIN": "min=", "AVG": "avg="}
                assert abi.ACC[sym[k[len("TL_ACC_"):]]] == v, k
            else:
                raise AssertionError(f"{k} has no Python mirror")
    assert d["TL_SHARD_COLS"] == abi.SHARD_COLS == 2


def test_default_opts(lib):
    o = abi.InitOpts()
    lib.tl_default_opts(C.byref(o))
    assert o.device == -1 and o.world_size == 1 and o.max_sweeps == 1000 and o.precision == abi.PREC_TF32


def test_null_arguments_are_rejected(lib):
    # argument checks happen before any device call
    assert lib.tl_init(None, None) == abi.TL_ERR_INVALID
    assert lib.tl_shutdown(None) == abi.TL_OK
    assert lib.tl_sync(None) == abi.TL_ERR_INVALID
    assert lib.tl_last_error(None) == b"no context"
    assert lib.tl_tensor_rank(None) == -1


def test_library_has_no_oracle_dependency():
    out = subprocess.run(["ldd", abi.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in out
    syms = subprocess.run(["nm", "-D", abi.LIB_PATH], capture_output=True, text=True).stdout
    assert "or_program_run" not in syms


def test_library_loads_the_nccl_torch_uses():
    # the library must resolve libnccl.so.2 to the NCCL wheel torch links, also
    # when it is loaded before torch (an older system NCCL would break torch)
    nvidia_nccl = pytest.importorskip("nvidia.nccl")
    want = os.path.realpath(os.path.join(list(nvidia_nccl.__path__)[0], "lib", "libnccl.so.2"))
    code = ("from tensor_logic_lang_b200 import abi; abi.load_library()\n"
            "import os\n"
            "print(sorted({os.path.realpath(l.split()[-1]) for l in open('/proc/self/maps') if 'libnccl' in l}))\n"
            "import torch\n")
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    assert want in out.stdout and out.stdout.count("libnccl") == 1, out.stdout
