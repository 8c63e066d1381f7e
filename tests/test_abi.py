"""The C-ABI library loads, exports every symbol its headers declare, and
fails loudly (no CPU fallback) where there is no GPU. No compute calls."""

import ctypes as C
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(pkv_\w+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    from pagedkv import _lib

    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(_lib.lib, n)]
    assert not missing, missing


def test_every_declared_symbol_has_a_prototype():
    from pagedkv import _lib, host  # noqa: F401  (host.py declares the pkv_host.h prototypes)

    missing = [n for n in declared_functions() if getattr(_lib.lib, n).argtypes is None]
    assert not missing, missing


def test_status_codes_map_to_cache_error_variants():
    from pagedkv import errors as E

    assert E.from_status(7, 99, 2, "") == E.InvalidLayer(99, 2)
    assert E.from_status(2, 99, 8, "") == E.InvalidBlock(99, 8)
    assert E.from_status(5, 99, 4, "") == E.SlotOutOfRange(99, 4)
    assert E.from_status(6, 8, 7, "") == E.ShapeMismatch(8, 7)
    assert E.from_status(9, 0, 0, "boom") == E.Device("boom")
    assert E.InvalidLayer(1, 2) != E.InvalidBlock(1, 2)


def test_null_handle_is_a_device_error_not_a_crash():
    from pagedkv import _lib

    assert _lib.lib.pkv_sync(None) == 9
    code, _, _, msg = _lib.last_error()
    assert code == 9 and "null" in msg


@pytest.mark.parametrize("name", [
    "pkv_reshape_and_cache_dev", "pkv_copy_blocks_dev", "pkv_zero_blocks_dev",
    "pkv_resolve_slots_dev", "pkv_resolve_and_cache_dev", "pkv_paged_attention_dev",
    "pkv_paged_attention_typed_dev", "pkv_paged_attention_multi_dev",
    "pkv_paged_attention_plan_dev", "pkv_digest", "pkv_digest_rows_dev"])
def test_device_entry_points_reject_a_null_handle(name):
    """Every device entry point checks its handle first (status 9, Device)."""
    from pagedkv import _lib

    f = getattr(_lib.lib, name)
    args = [None if t in (C.c_void_p, C.c_char_p) or hasattr(t, "contents") else
            (0.0 if t in (C.c_float, C.c_double) else 0) for t in f.argtypes]
    assert f(*args) == 9
    code, _, _, msg = _lib.last_error()
    assert code == 9 and "null" in msg


def test_unknown_dtype_tag_is_rejected_before_any_device_work():
    from pagedkv import _lib

    cfg = _lib.Config(8, 4, 2, 4, 2, 4)
    h = C.c_void_p()
    assert _lib.lib.pkv_create(C.byref(cfg), 7, 0, 0, 1, C.byref(h)) == 9
    assert h.value is None


def test_create_without_a_gpu_fails_loudly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from pagedkv import B200Backend, CacheConfig, Device

    with pytest.raises(Device):
        B200Backend(CacheConfig.tiny(8))


def test_config_errors_are_reported_before_device_work():
    from pagedkv import B200Backend, CacheConfig, Device

    with pytest.raises(Device, match="dtype_bytes"):
        B200Backend(CacheConfig.tiny(8), dtype="bf16")  # tiny says 4 bytes per element
    with pytest.raises(Device, match="shard"):
        B200Backend(CacheConfig.tiny(8), shard_rank=0, num_shards=3)  # 8 elements / 3


def test_headers_compile_as_c_and_cpp_and_link(tmp_path):
    """The C ABI is consumed from C, Rust (bindgen-style declarations) and
    C++: both headers must compile as strict C99 and C++17, and a C program
    calling the entry points must link against the library."""
    import shutil
    import subprocess

    from pagedkv._lib import LIB_PATH

    inc = ROOT / "include"
    src = tmp_path / "use.c"
    src.write_text(
        "#include <pkv_b200.h>\n#include <pkv_host.h>\n#include <stdio.h>\n"
        "int main(void) {\n"
        "  pkv_config c = {16, 16, 2, 64, 2, 2};\n"
        "  pkv_backend *b = 0;\n"
        "  int rc = pkv_create(&c, 1, 0, 0, 1, &b);\n"
        "  printf(\"%d %s\\n\", rc, pkv_last_error());\n"
        "  if (b) pkv_destroy(b);\n"
        "  return 0;\n}\n")
    cc = shutil.which("gcc")
    cxx = shutil.which("g++")
    assert cc and cxx
    for compiler, std in ((cc, "-std=c99"), (cxx, "-std=c++17")):
        lang = ["-x", "c"] if compiler == cc else ["-x", "c++"]
        subprocess.run([compiler, *lang, std, "-Wall", "-Wextra", "-Werror", "-pedantic",
                        "-fsyntax-only", f"-I{inc}", str(src)], check=True)
    exe = tmp_path / "use"
    subprocess.run([cc, "-std=c99", f"-I{inc}", str(src), str(LIB_PATH), "-o", str(exe),
                    f"-Wl,-rpath,{LIB_PATH.parent}"], check=True)
    assert exe.exists()
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0
    rc = int(out.stdout.split()[0])  # 0 with a GPU; a device error status without one
    assert rc == 0 or rc == 9
