"""The C ABI library loads without a GPU and exports every symbol include/gpt_b200.h declares;
argument validation runs before any CUDA call."""
import ctypes
import os
import re

import pytest

from cutilegpt_b200 import _lib as L

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "gpt_b200.h")


def declared():
    src = open(HEADER).read()
    return re.findall(r"^GPT_API\s+[\w\s\*]+?\b(gpt_\w+)\s*\(", src, flags=re.M)


def test_header_declares_entry_points():
    names = declared()
    assert len(names) >= 14 and len(set(names)) == len(names)


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    for n in declared():
        assert hasattr(lib, n), n


def test_binding_covers_header():
    assert set(declared()) == set(L.SIGNATURES)


def test_no_cuda_runtime_dependency():
    # static cudart: the .so must not need libcudart / libcuda to load
    out = os.popen(f"ldd {L.LIB_PATH}").read()
    assert "libcudart" not in out and "libcuda.so" not in out


def test_version_and_errors_without_gpu():
    lib = L.lib()
    assert lib.gpt_version() == 1
    # bad epilogue: rejected before touching CUDA
    st = lib.gpt_gemm(None, 8, None, None, None, 0, None, 8, 4, 4, 8, 9, L.GPT_F32, None)
    assert st == L.GPT_ERR_ARG
    assert b"epilogue" in lib.gpt_last_error_string()
    assert lib.gpt_gelu(None, None, 0, L.GPT_F32, None) == L.GPT_OK       # empty is a no-op
    assert lib.gpt_gelu(None, None, 4, 7, None) == L.GPT_ERR_DTYPE
    assert lib.gpt_layernorm(None, None, None, None, -1, 8, 1e-5, L.GPT_BF16, None) == L.GPT_ERR_SHAPE
    assert lib.gpt_attention_decode_workspace_size(0, 1, 64, 10) == 0
    assert lib.gpt_embedding_pos(None, 1, 5, None, None, 10, 4, 8, 0, None, None, L.GPT_F32, None) == \
        L.GPT_ERR_SHAPE                                     # T beyond n_pos
    assert lib.gpt_kv_append(None, 1, None, None, 1, 1, 1, 8, 4, 4, None, L.GPT_BF16, None) == L.GPT_ERR_SHAPE


def test_check_maps_status_to_exceptions():
    lib = L.lib()
    lib.gpt_gelu(None, None, 4, 7, None)
    with pytest.raises(ValueError):
        L.check(L.GPT_ERR_DTYPE, "x")
    with pytest.raises(L.GptError):
        L.check(L.GPT_ERR_CUDA, "x")


def test_thread_local_error_string():
    import threading
    lib = L.lib()
    lib.gpt_gelu(None, None, 4, 7, None)
    seen = {}

    def other():
        seen["s"] = lib.gpt_last_error_string()
    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["s"] == b""
    assert b"dtype" in lib.gpt_last_error_string()


def test_gemm_fusion_struct_layout_matches_header(tmp_path):
    """ctypes GemmFusion has the field offsets and size of struct gpt_gemm_fusion (compiled with gcc)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    from cutilegpt_b200 import _lib as L
    fields = [f[0] for f in L.GemmFusion._fields_]
    src = tmp_path / "layout.c"
    hdr = HEADER
    body = "".join(f'  printf("{f} %zu\\n", offsetof(gpt_gemm_fusion, {f}));\n' for f in fields)
    src.write_text(f'#include <stdio.h>\n#include <stddef.h>\n#include "{hdr}"\nint main(void) {{\n{body}'
                   f'  printf("sizeof %zu\\n", sizeof(gpt_gemm_fusion));\n  return 0;\n}}\n')
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-o", str(exe), str(src)], check=True)
    got = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                       check=True).stdout.splitlines())
    for f in fields:
        assert int(got[f]) == getattr(L.GemmFusion, f).offset, f
    assert int(got["sizeof"]) == ctypes.sizeof(L.GemmFusion)
