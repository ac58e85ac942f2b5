"""The C ABI from a plain C host: include/tideway_b200.h compiles as C99 and a C program links
the library and calls its host-only entry points (no device work, so no GPU is needed)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <stdio.h>
#include "tideway_b200.h"

int main(void) {
  size_t small = tw_moe_workspace_bytes(8, 2048, 768);
  size_t large = tw_moe_workspace_bytes(512, 2048, 768);
  /* a refused argument returns a status and leaves a message, it does not abort */
  int rc = tw_moe_ffn_noalloc_error(-1, 2048, 768, 0, 0);
  const char* msg = tw_last_error();
  printf("%d %d %d %d\n", tw_abi_version(), small > 0 && small < large, rc != 0,
         msg != 0 && msg[0] != 0);
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_program_links_and_calls_the_library(tmp_path):
    from tideway_b200 import _lib, build

    build.build()
    lib_dir = _lib.LIB_PATH.parent
    src = tmp_path / "host.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "host"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(src), "-o", str(exe), "-L", str(lib_dir), "-ltideway_b200",
                    f"-Wl,-rpath,{lib_dir}"], check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["103", "1", "1", "1"], r.stdout
