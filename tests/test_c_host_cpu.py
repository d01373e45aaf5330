"""A plain C99 host of libtitan_b200 (tests/c_host/host_check.c), no GPU: the public header
compiles as C with -pedantic -Werror, the program links against the in-tree library,
and the host-side entries (SHA-256, canonical JSON, the `.tune` store, the graph
compiler, the operator router) answer through the C ABI alone."""
import pathlib
import shutil
import subprocess

import pytest

from titan_rs_b200 import _native as N

ROOT = pathlib.Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler on this machine")
def test_c_host_uses_the_library_through_the_header(tmp_path):
    N.lib()  # raises when the library is not built
    exe = tmp_path / "host_check"
    subprocess.run(["gcc", "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_host" / "host_check.c"), "-o", str(exe), "-L", str(N.LIB_PATH.parent),
                    "-ltitan_b200", f"-Wl,-rpath,{N.LIB_PATH.parent}"], check=True, capture_output=True, text=True)
    run = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    checks = [line.split()[1] for line in run.stdout.splitlines() if line.startswith("ok ")]
    assert checks == ["version", "sha256", "canonical_json", "tune_open", "tune_insert", "tune_flush", "tune_reopen",
                      "tune_get", "tune_stats", "tune_record", "tune_miss", "short_buffer", "graph_compile",
                      "graph_error", "execute_route"]
    assert (tmp_path / "kernels.tune").read_text().startswith("# titan.tune version=2\n")


STRUCTS = {"tb_fingerprint": "Fingerprint", "tb_launch_arg": "LaunchArg", "tb_launch_metadata": "LaunchMetadata",
           "tb_binding": "Binding", "tb_encoded_args": "EncodedArgs", "tb_launch_geometry": "LaunchGeometry",
           "tb_tensor": "Tensor", "tb_attr": "Attr", "tb_tune_measurement": "TuneMeasurement"}


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler on this machine")
def test_ctypes_structures_match_the_header_layout(tmp_path):
    """Every struct of the header has the size and field offsets of its ctypes mirror."""
    import ctypes
    import re
    header = (ROOT / "include" / "titan_b200.h").read_text()
    assert set(re.findall(r"typedef struct (tb_\w+) \{", header)) == set(STRUCTS)
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "titan_b200.h"', "int main(void) {"]
    expected = []
    for c_name, py_name in STRUCTS.items():
        cls = getattr(N, py_name)
        lines.append(f'  printf("{c_name} %zu\\n", sizeof({c_name}));')
        expected.append(f"{c_name} {ctypes.sizeof(cls)}")
        for field, *_ in cls._fields_:
            lines.append(f'  printf("{c_name}.{field} %zu\\n", offsetof({c_name}, {field}));')
            expected.append(f"{c_name}.{field} {getattr(cls, field).offset}")
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    got = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines()
    assert got == expected
