"""C-ABI library checks that need no GPU: it loads, exports every symbol the
public header declares, and its pure-host queries answer sensibly."""

import ctypes
import glob
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    syms = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(b200_\w+)\s*\(", text):
            syms.add(m.group(1))
    return sorted(syms)


def test_header_declares_the_hot_path():
    syms = header_symbols()
    for s in ("b200_kv_scatter_rows", "b200_kv_scatter_slots", "b200_paged_decode",
              "b200_paged_decode_workspace_size", "b200_varlen_prefill"):
        assert s in syms


def test_library_exports_every_header_symbol(native_lib):
    from qwen3_engine_from_scratch_b200 import _native
    out = subprocess.run(["nm", "-D", "--defined-only", _native.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [s for s in header_symbols() if s not in exported]
    assert not missing, f"declared in include/ but not exported: {missing}"
    # and the ctypes table covers the same set
    assert set(_native.SIGNATURES) == set(header_symbols())
    # no b200_* entry point is exported without a declaration in include/
    undeclared = sorted(s for s in exported if s.startswith("b200_") and s not in header_symbols())
    assert not undeclared, f"exported but not declared in include/: {undeclared}"


def test_library_is_sm100a_only(native_lib):
    from qwen3_engine_from_scratch_b200 import _native
    # the ELF notes the embedded cubin architecture in the fatbin section names;
    # cuobjdump would read compiled code, so only the build flags are checked here
    from qwen3_engine_from_scratch_b200 import build
    assert "arch=compute_100a,code=sm_100a" in build.ARCH_FLAGS
    assert os.path.getsize(_native.LIB_PATH) > 0


def test_status_strings(native_lib):
    from qwen3_engine_from_scratch_b200 import _native
    assert _native.status_string(0) == "ok"
    for code in range(-6, 0):
        assert _native.status_string(code) != "unknown status"
    assert native_lib.b200_abi_version() >= 100


def test_decode_workspace_is_shape_only(native_lib):
    ws = native_lib.b200_paged_decode_workspace_size
    # one split: no workspace
    assert ws(64, 16, 16, 16) == 0
    # 256 pages at 16 pages per split: 256 KiB of split counters, then 16 partials of
    # (128 acc + m + l) floats per (b, h)
    assert ws(64, 16, 256, 16) == (256 << 10) + 64 * 16 * 16 * 130 * 4
    # <= 0: an upper bound for every default split
    assert ws(64, 16, 256, 0) >= ws(64, 16, 256, native_lib.b200_paged_decode_default_split(64, 8, 256))
    assert ws(64, 16, 256, 0) == ws(64, 16, 256, 16)
    assert ws(0, 16, 256, 16) == 0


def test_invalid_arguments_are_rejected_before_any_launch(native_lib):
    """Argument checks run on the host and return a status; nothing touches a GPU."""
    lib = native_lib
    null = None
    # batch < 0
    st = lib.b200_paged_decode(null, 0, 0, null, null, 0, 0, 0, null, 1, null, null, null, 0, 0,
                               -1, 16, 8, 128, 16, 1, 1, 1, 1.0, 0, null, 0, null, null)
    assert st == -1
    # head_dim 64 unsupported (pointers non-null but never dereferenced: checks come first)
    fake = ctypes.c_void_p(16)
    st = lib.b200_paged_decode(fake, 128, 128, fake, fake, 2048, 2048, 128, fake, 1, fake, fake,
                               fake, 128, 128, 1, 16, 8, 64, 16, 1, 1, 1, 1.0, 0, null, 0, null,
                               null)
    assert st == -2
    # empty batch is a no-op
    st = lib.b200_kv_scatter_rows(null, null, 0, 0, 0, 0, 0, 0, null, null, 0, 0, 0, 0, 0, 0, 0, 0,
                                  null, null, 1, null, 0, 1, 8, 128, 16, 1, 1, 1, 0, null, null)
    assert st == 0
    st = lib.b200_kv_scatter_slots(null, null, 0, 0, 0, 0, null, null, 0, 0, 0, 0, 0, 0, 0, 0,
                                   null, 0, 5, 8, 128, 16, 1, 0, null, null)
    assert st == -1


def test_product_does_not_import_the_oracle():
    pkg = os.path.join(REPO, "qwen3_engine_from_scratch_b200")
    for p in glob.glob(os.path.join(pkg, "*.py")):
        src = open(p).read()
        assert "import oracle" not in src and "from oracle" not in src, p


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    from qwen3_engine_from_scratch_b200 import _native
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "absent.so"))
    with pytest.raises(_native.NativeLibraryMissing):
        _native.load()
