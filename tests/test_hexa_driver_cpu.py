"""The hexa-side decode driver (hexa-lang_b200/hexa/forge_greedy.hexa, the
binding pattern of self/ml/hxflash.hexa: @link extern fn over the C ABI)
without a GPU: the committed C equals what the hexa transpiler makes of the
.hexa source (when the transpiler is at hand), the program links against
the library's own hexa runtime and resolves every extern it declares from
libforge_b200.so, and it reports the library's error with status 1 when no
device is there (no compute runs)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HX = os.path.join(ROOT, "hexa-lang_b200", "hexa")
BIN = os.path.join(HX, "forge_greedy")
HEXAT = os.environ.get("HEXAT", "/root/reference/build/hexat_linux")


@pytest.fixture(scope="module")
def program(forge):
    subprocess.run(["make", "-C", os.path.join(ROOT, "hexa-lang_b200", "csrc"), "../hexa/forge_greedy"], check=True,
                   capture_output=True)
    return BIN


def test_generated_c_is_current(tmp_path):
    if not os.access(HEXAT, os.X_OK):
        pytest.skip("hexa transpiler not present")
    out = tmp_path / "forge_greedy.c"
    r = subprocess.run([HEXAT, os.path.join(HX, "forge_greedy.hexa"), str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    # the transpiler names the output file in its string-table init function
    norm = lambda s: re.sub(r"__hexa_strlit_init_\w+", "INIT", s)
    with open(os.path.join(HX, "forge_greedy.c")) as f:
        assert norm(out.read_text()) == norm(f.read())


def test_externs_resolve_from_the_library(program, forge):
    with open(os.path.join(HX, "forge_greedy.c")) as f:
        src = f.read()
    syms = set(re.findall(r'hexa_ffi_dlsym\(hexa_ffi_dlopen\("forge_b200"\), "(\w+)"\)', src))
    assert {"forge_b200_create_packed", "forge_b200_init_synthetic_d", "forge_b200_generate",
            "forge_b200_decode_step", "forge_b200_reset", "forge_b200_destroy"} <= syms
    lib = forge.lib()
    for s in syms:
        assert hasattr(lib, s), s


def test_library_error_without_gpu(program):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    r = subprocess.run([program], capture_output=True, text=True, timeout=120)
    assert r.returncode == 1, (r.stdout, r.stderr)
    assert r.stdout.strip() == "create failed -4" and "no CUDA device" in r.stderr
