"""The C ABI from plain C, without a GPU.

``include/leanselect_b200.h`` is compiled by a C compiler (C99, every
warning an error) into a program linked against the in-tree library; the
program calls the entry points a C host binds first: the version string,
the status strings, a workspace-size query and a call that fails argument
validation on the host (no CUDA call is made).
"""
import shutil
import subprocess
from pathlib import Path

import pytest

from leanselect_b200 import _native

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "leanselect_b200.h"

int main(void) {
  if (strstr(ls_version(), "sm_100a") == NULL) return 10;
  if (strcmp(ls_status_string(LS_ERR_UNSUPPORTED), "LS_ERR_UNSUPPORTED") != 0) return 11;
  if (ls_select_pages_workspace_bytes(1000, 2, 1000) != (size_t)2 * 1000 * 16 * 2) return 12;
  /* head_dim 100 is not compiled: rejected on the host before any CUDA call. */
  int rc = ls_sparse_attn((const uint16_t*)0x100000, (const uint16_t*)0x100000,
                          (const uint16_t*)0x100000, (const int32_t*)0x100000,
                          (const int32_t*)0x100000, 1, 64, 64, 64, 64, 32, 2, 100,
                          (const int32_t*)0x100000, 4, 64, 0.0f, 1, (uint16_t*)0x100000,
                          NULL, NULL, NULL);
  if (rc != LS_ERR_UNSUPPORTED) return 13;
  printf("%s\n", ls_last_error());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_header_compiles_as_c_and_links(tmp_path):
    lib = Path(_native.load()._name)
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(ROOT / "include"),
                    str(src), "-o", str(exe), str(lib), f"-Wl,-rpath,{lib.parent}"], check=True)
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0, (run.returncode, run.stdout, run.stderr)
    assert "head_dim" in run.stdout
