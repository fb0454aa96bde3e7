"""The C-ABI library builds for sm_100a, loads, and exports every symbol include/*.h declares.
No compute calls: runs without a GPU."""

import ctypes
import os
import re

import pytest

from exactattention_b200 import _lib

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"^\s*(?:int|float|void|const char\*)\s+(ea_\w+)\s*\(", src, re.M))
    return names


def test_library_exports_every_declared_symbol(cuda_lib):
    names = declared_functions()
    assert {"ea_attention_cuda", "ea_launch_cuda", "ea_round_ratio_cuda", "ea_synth_fill"} <= names
    for n in names:
        assert hasattr(cuda_lib, n), n
    assert set(_lib.EXPORTS) <= names


@pytest.mark.parametrize("ctype,mirror", [("ea_launch_t", _lib.LaunchArgs), ("ea_partials_t", _lib.PartialsArgs),
                                          ("ea_wide_partials_t", _lib.WidePartialsArgs),
                                          ("ea_kv_append_t", _lib.KvAppendArgs),
                                          ("ea_test_hooks_t", _lib.TestHooks)])
def test_struct_layout_matches_header(cuda_lib, tmp_path, ctype, mirror):
    """The ctypes mirrors of the header's structs have the C compiler's size and field offsets."""
    import subprocess

    fields = [f[0] for f in mirror._fields_]
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "exactattn_cuda.h"\nint main(void){'
                   f'printf("%zu", sizeof({ctype}));'
                   + "".join(f'printf(" %zu", offsetof({ctype}, {f}));' for f in fields) + "return 0;}\n")
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), "-o", str(exe), str(src)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(mirror)
    assert vals[1:] == [getattr(mirror, f).offset for f in fields]


def test_build_targets_sm100a():
    from exactattention_b200 import build

    assert "arch=compute_100a,code=sm_100a" in build.FLAGS


def test_exactattn_import_name():
    """The reference's import name serves the same functions (no GPU call)."""
    import exactattn
    import exactattention_b200 as ea
    from exactattn.cuda import attention_cuda
    from exactattn.torch_impl import attention_torch

    assert exactattn.attention is ea.attention
    assert attention_cuda is ea.cuda.attention_cuda
    assert attention_torch is ea.torch_impl.attention_torch
    assert exactattn.default_alpha(64) == ea.default_alpha(64)


def test_stats_length_matches_header():
    src = open(os.path.join(ROOT, "include", "exactattn_cuda.h")).read()
    assert int(re.search(r"#define EA_STATS_LEN (\d+)", src).group(1)) == _lib.EA_STATS_LEN == len(_lib.STAT_NAMES)
