"""The public headers from a C caller's side: tests/abi_c/abi_caller.c is compiled as strict C11
(and as C++17) against include/plamo.h and include/plamo_kernels.h, linked against the built
libplamo_cuda.so and run without a GPU, so header/ABI drift fails here rather than in a Swift or C
host (a SwiftPM C target imports exactly these headers)."""
import shutil
import subprocess

import pytest

from conftest import REPO


@pytest.mark.parametrize("lang", ["c11", "c++17"])
def test_c_caller_compiles_and_runs(pkg, micro_dir, tmp_path, lang):
    pkg.build.build()
    lib = pkg.runtime.LIB_PATH
    cc = shutil.which("gcc" if lang == "c11" else "g++")
    if not cc:
        pytest.skip("no host compiler")
    exe = tmp_path / f"abi_caller_{lang.replace('+', 'p')}"
    src = REPO / "tests" / "abi_c" / "abi_caller.c"
    std = ["-std=c11", "-pedantic"] if lang == "c11" else ["-x", "c++", "-std=c++17"]
    cmd = [cc, *std, "-Wall", "-Wextra", "-Werror", "-I", str(REPO / "include"), str(src), "-o", str(exe),
           "-L", str(lib.parent), "-lplamo_cuda", f"-Wl,-rpath,{lib.parent}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe), str(micro_dir)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr + r.stdout
    assert "abi_caller: ok" in r.stdout


def test_swift_module_shim_compiles_as_c(tmp_path):
    """The SwiftPM C module (swift/Sources/CPlamo) imports the public headers through shim.h; with
    no Swift toolchain here, the header set it exposes is compiled as C11."""
    cc = shutil.which("gcc")
    if not cc:
        pytest.skip("no host compiler")
    shim = REPO / "plamo3-0.8b-runtime_b200" / "swift" / "Sources" / "CPlamo" / "shim.h"
    src = tmp_path / "use_shim.c"
    src.write_text(f'#include "{shim}"\nint main(void) {{ return plamo_position(0); }}\n')
    subprocess.run([cc, "-std=c11", "-pedantic", "-Wall", "-Werror", "-fsyntax-only", str(src)], check=True,
                   capture_output=True, text=True)
    modulemap = (shim.parent / "module.modulemap").read_text()
    assert 'header "shim.h"' in modulemap and 'link "plamo_cuda"' in modulemap
