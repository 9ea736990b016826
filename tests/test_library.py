"""The C-ABI library builds, loads and exports what include/bfknn.h declares
(no compute calls: this runs without a GPU)."""
import ctypes
import os
import re

import pytest

from gpu_algo_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "bfknn.h")).read()
    return sorted(set(re.findall(r"BFK_API\s+[\w\s\*]*?\b(bfk_\w+)\s*\(", src)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = os.popen(f"nm -D --defined-only {_lib.LIB_PATH}").read()
    exported = set(re.findall(r"\bT (bfk_\w+)", out))
    assert exported == set(declared_symbols())


def test_version_and_status_strings(lib):
    assert _lib.version() == (0, 1)
    for code in range(7):
        assert _lib.status_string(code) not in ("", "unknown status")
    assert _lib.status_string(99) == "unknown status"


def test_argument_validation_without_gpu(lib):
    nb = ctypes.c_uint64()
    o = _lib.make_opts()
    assert lib.bfk_workspace_size(-1, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    assert lib.bfk_workspace_size(10, 10, 8, 0, ctypes.byref(o), ctypes.byref(nb)) == 1
    assert lib.bfk_workspace_size(10, 10, 8, 5000, ctypes.byref(o), ctypes.byref(nb)) == 2
    o.reserved[2] = 1
    assert lib.bfk_workspace_size(10, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    o = _lib.make_opts(flags=_lib.FLAG_CTA_PAIR | _lib.FLAG_SINGLE_CTA)  # contradictory
    assert lib.bfk_workspace_size(10, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    o = _lib.make_opts()
    o.shards = -1
    assert lib.bfk_workspace_size(10, 10, 8, 1, ctypes.byref(o), ctypes.byref(nb)) == 1
    o = _lib.make_opts("direct")
    assert lib.bfk_workspace_size(1024, 65536, 128, 10, ctypes.byref(o), ctypes.byref(nb)) == 0
    assert nb.value % 256 == 0 and nb.value >= 256
    # invalid arguments are rejected before any device work
    assert lib.bfk_search(None, 4, None, 4, 8, 1, 0, None, None, None, 0, None, None) == 1
    assert lib.bfk_merge(None, None, 4, 0, 1, None, None, None) == 1
    a = _lib.Attrs()
    assert lib.bfk_merge_attrs(0, 10, ctypes.byref(a)) == 1
    assert lib.bfk_merge_attrs(4, 0, ctypes.byref(a)) == 1
    assert lib.bfk_merge_attrs(4, 10, None) == 1
    assert lib.bfk_merge_attrs(4, 5000, ctypes.byref(a)) == 2


def test_workspace_has_room_for_partials(lib):
    o = _lib.make_opts("direct", slices=8)
    nb = ctypes.c_uint64()
    assert lib.bfk_workspace_size(100, 10_000, 16, 10, ctypes.byref(o), ctypes.byref(nb)) == 0
    assert nb.value >= 8 * 100 * 10 * 8


def test_header_is_plain_c_and_links(tmp_path):
    """include/bfknn.h compiles as C99 and C++11, and a C caller links against the
    library (the ABI a cgo / ctypes / JNI binding would use)."""
    import shutil
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    inc = os.path.join(root, "include")
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "caller.c"
    src.write_text(
        '#include "bfknn.h"\n#include <stdio.h>\n'
        'int main(void) { int32_t a, b; bfk_version(&a, &b);\n'
        '  uint64_t nb = 0; bfk_opts_t o = {0};\n'
        '  int s = bfk_workspace_size(10, 1000, 128, 5, &o, &nb);\n'
        '  printf("%d %d %d %d\\n", a, b, s, nb > 0); return 0; }\n')
    exe = tmp_path / "caller"
    libdir = os.path.join(root, "gpu_algo_b200")
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", inc, str(src), "-o", str(exe),
                    "-L", libdir, "-lbfknn", f"-Wl,-rpath,{libdir}"], check=True)
    subprocess.run(["g++", "-std=c++11", "-fsyntax-only", "-x", "c++",
                    os.path.join(inc, "bfknn.h")], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split()
    assert out[2] == "0" and out[3] == "1"


def test_prepared_sizes_without_gpu(lib):
    """A prepared search's workspace holds no rows; a prepared buffer holds them plus a
    512-byte header, all parts 256-byte aligned."""
    m, d = 40_000, 128
    plain = _lib.make_opts("tc_f16")
    prep = _lib.make_opts("tc_f16", flags=_lib.FLAG_PREPARED)
    full, small, pb = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
    assert lib.bfk_workspace_size(64, m, d, 10, ctypes.byref(plain), ctypes.byref(full)) == 0
    assert lib.bfk_workspace_size(64, m, d, 10, ctypes.byref(prep), ctypes.byref(small)) == 0
    assert full.value - small.value >= m * d * 2
    assert lib.bfk_prepared_size(m, d, ctypes.byref(pb)) == 0
    assert pb.value % 256 == 0 and pb.value >= 512 + m * d * 2 + m * 4
    assert lib.bfk_prepared_size(m, 0, ctypes.byref(pb)) == 1
    # a prepared search needs the flag and the buffer together
    assert lib.bfk_search_prepared(None, 4, None, None, m, d, 10, 0, None, None, None, 0,
                                   ctypes.byref(prep), None) == 1


def test_shards_pick_one_engine(lib):
    """A shard just under the filter engine's row threshold still takes the engine
    its larger sibling shards take (plan_rows), so all make the same hook calls."""
    nb_auto, nb_tc, nb_alone = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
    o = _lib.make_opts()
    o.plan_rows = 4096
    assert lib.bfk_workspace_size(64, 4095, 128, 10, ctypes.byref(o), ctypes.byref(nb_auto)) == 0
    t = _lib.make_opts("tc_f16")
    t.plan_rows = 4096
    assert lib.bfk_workspace_size(64, 4095, 128, 10, ctypes.byref(t), ctypes.byref(nb_tc)) == 0
    assert nb_auto.value == nb_tc.value
    alone = _lib.make_opts()
    assert lib.bfk_workspace_size(64, 4095, 128, 10, ctypes.byref(alone), ctypes.byref(nb_alone)) == 0
    assert nb_alone.value != nb_tc.value  # on its own, the SIMT engine


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors of bfk_opts_t, bfk_attrs_t and bfk_stats_t have the C
    header's size and field offsets (a shifted field would pass options wrongly)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("no C compiler")
    mirrors = {"bfk_opts_t": _lib.Opts, "bfk_attrs_t": _lib.Attrs, "bfk_stats_t": _lib.Stats,
               "bfk_plan_info_t": _lib.PlanInfo}
    lines = ['#include "bfknn.h"', "#include <stddef.h>", "#include <stdio.h>",
             "int main(void) {"]
    for cname, py in mirrors.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], check=True, capture_output=True,
                             text=True).stdout.splitlines():
        cname, field, value = ln.split()
        got[(cname, field)] = int(value)
    for cname, py in mirrors.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, f"{cname}.{fname}"


def test_plan_levels_and_cta_pairs():
    """The planner's choices, computed on the host (bfk_plan_info): the 10M-row workload's
    four levels with CTA pairs; a shard of an 8-GPU search keeps its own full first level
    (the sizes of a lone search of its rows) and, under 4M rows, single CTAs; shards decide
    on the largest shard's rows; pairs can be forced either way; 16 queries take the SIMT
    engine."""
    from gpu_algo_b200 import engine
    p = engine.plan_info(10_000, 10_000_000, 128, 100)
    assert p["engine"] == "tc_f16" and p["cta_pair"]
    assert p["level_tiles"] == [2, 44, 1303, 39063] and p["q_tiles"] == 80
    shard = engine.plan_info(10_000, 1_250_000, 128, 100, plan_rows=1_250_000, shards=8)
    lone = engine.plan_info(10_000, 1_250_000, 128, 100)
    assert shard["level_tiles"] == lone["level_tiles"] == [6, 163, 4883]
    assert not shard["cta_pair"] and shard["q_tiles"] == 79
    small = engine.plan_info(10_000, 3_000_000, 128, 100, plan_rows=5_000_000, shards=2)
    assert small["cta_pair"] and small["levels"] == 4
    assert not engine.plan_info(10_000, 1_000_000, 128, 100)["cta_pair"]
    assert engine.plan_info(10_000, 1_000_000, 128, 100, cta_pair=True)["cta_pair"]
    assert not engine.plan_info(10_000, 10_000_000, 128, 100, cta_pair=False)["cta_pair"]
    assert not engine.plan_info(1_000, 20_000_000, 960, 100)["cta_pair"]
    direct = engine.plan_info(16, 12_500_000, 96, 10)
    assert direct["engine"] == "direct" and direct["levels"] == 0
    with pytest.raises(_lib.BfkError):
        engine.plan_info(10, 100, 0, 10)
