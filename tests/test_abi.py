"""The C ABI library: loads, exports every symbol include/jx_attn.h declares,
matches the header's struct layouts, and fails loudly without a GPU."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

import jxai_b200 as jx
from jxai_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "jx_attn.h")


def declared_symbols():
    with open(HEADER) as fh:
        text = fh.read()
    return sorted(set(re.findall(r"JX_API\s+(?:const\s+)?\w+\*?\s+\**(jx_\w+)\s*\(", text)))


def test_cmake_build_compiles_the_same_sources():
    """CMakeLists.txt (for engines that build with CMake) lists exactly the
    translation units jxai_b200/build.py compiles, so both libraries export
    the same entry points."""
    from jxai_b200 import build
    with open(os.path.join(ROOT, "CMakeLists.txt")) as fh:
        text = fh.read()
    listed = re.search(r"add_library\(jxattn SHARED(.*?)\)", text, re.S).group(1).split()
    assert sorted(os.path.basename(f) for f in listed) == sorted(build.SOURCES)


def test_header_declares_the_binding_list():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = jx.load_library()
    out = subprocess.run(["nm", "-D", "--defined-only", jx.lib_path()], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    for sym in declared_symbols():
        assert sym in exported, sym
        assert getattr(lib, sym) is not None
    # nothing else leaks out of the C ABI
    assert {s for s in exported if not s.startswith("jx_")} <= {"_init", "_fini"}


def test_version_string():
    assert b"sm_100a" in jx.load_library().jx_version()


def test_struct_layouts_match_header():
    src = r"""
#include <stddef.h>
#include <stdio.h>
#include "jx_attn.h"
int main(void) {
  printf("%zu %zu %zu\n", sizeof(jx_kv_desc), sizeof(jx_layer_desc), sizeof(jx_step_args));
  printf("%zu %zu %zu %zu\n", offsetof(jx_layer_desc, rope_freqs), offsetof(jx_step_args, q),
         offsetof(jx_step_args, q_stride), offsetof(jx_step_args, rope_neox));
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        with open(c, "w") as fh:
            fh.write(src)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe], check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    sizes = [int(x) for x in lines[0].split()]
    offs = [int(x) for x in lines[1].split()]
    assert sizes == [C.sizeof(_lib.KvDesc), C.sizeof(_lib.LayerDesc), C.sizeof(_lib.StepArgs)]
    assert offs == [_lib.LayerDesc.rope_freqs.offset, _lib.StepArgs.q.offset,
                    _lib.StepArgs.q_stride.offset, _lib.StepArgs.rope_neox.offset]


def test_invalid_arguments_rejected_on_host():
    lib = jx.load_library()
    assert lib.jx_kv_create(None, None) == _lib.JX_ERR_INVALID
    assert b"null" in lib.jx_last_error_string()
    assert lib.jx_attn_step(None, None, 0, None, None) == _lib.JX_ERR_INVALID
    assert lib.jx_lse_merge(None, 0, 0, 0, 0, 0, None, 0, None) == _lib.JX_ERR_INVALID
    assert lib.jx_attn_step_sharded(None, None, 0, None, None, 0, None) == _lib.JX_ERR_INVALID
    assert b"communicator" in lib.jx_last_error_string()
    assert lib.jx_noalloc_check_device_error(0, None, None) == _lib.JX_ERR_INVALID
    assert lib.jx_noalloc_set_option(b"no_such_option", 1) == _lib.JX_ERR_INVALID
    assert lib.jx_noalloc_set_option(b"wait_limit_ms", -1) == _lib.JX_ERR_INVALID
    assert lib.jx_noalloc_set_option(b"wait_limit_ms", 0) == _lib.JX_OK
    assert lib.jx_noalloc_set_option(b"test_wait_cta", 0) == _lib.JX_OK


def test_no_gpu_means_a_loud_failure():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(jx.JxError) as e:
        jx.KVCache(1, 1, 16, 64, "f32")
    assert e.value.code == _lib.JX_ERR_CUDA


def test_cmake_project_configures():
    # CMakeLists.txt builds the same library for C++ engines that use CMake
    import shutil
    import tempfile
    cmake = shutil.which("cmake")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if cmake is None or not os.path.exists(nvcc):
        pytest.skip("cmake or nvcc not available")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with tempfile.TemporaryDirectory() as td:
        r = subprocess.run([cmake, "-S", root, "-B", td, f"-DCMAKE_CUDA_COMPILER={nvcc}"],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]


def test_nccl_config_mirror_matches_the_header():
    # jxai_b200.nccl builds ncclConfig_t through ctypes for the non-blocking
    # communicator creation: same size and offsets as the header of the NCCL
    # the process loads (torch's copy)
    import glob
    from jxai_b200.nccl import _Config
    heads = glob.glob(os.path.join(os.path.dirname(os.__file__), "..", "..", "lib", "python3*",
                                   "site-packages", "nvidia", "nccl", "include", "nccl.h"))
    try:
        import nvidia.nccl
        heads += glob.glob(os.path.join(list(nvidia.nccl.__path__)[0], "include", "nccl.h"))
    except ImportError:
        pass
    if not heads:
        pytest.skip("NCCL header not found")
    fields = [name for name, _ in _Config._fields_]
    src = "#include <stdio.h>\n#include <stddef.h>\n#include \"nccl.h\"\nint main(void){\n"
    src += 'printf("%zu\\n", sizeof(ncclConfig_t));\n'
    src += "".join(f'printf("%zu\\n", offsetof(ncclConfig_t, {f}));\n' for f in fields)
    src += "return 0;}\n"
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        with open(c, "w") as fh:
            fh.write(src)
        cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
        subprocess.run(["gcc", "-I", os.path.dirname(heads[0]), "-I", cuda_inc, c, "-o", exe],
                       check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True,
                                               check=True).stdout.split()]
    assert vals[0] == C.sizeof(_Config)
    assert vals[1:] == [getattr(_Config, f).offset for f in fields]
