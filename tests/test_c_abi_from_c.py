"""The boundary as a C program sees it: ``include/muon_sr_b200.h`` compiles as C99 with all
warnings as errors, every function it declares links against ``libmuon_sr_b200.so``, and the
host-only entry points answer from C (no GPU and no Python involved)."""
import os
import re
import shutil
import subprocess

import pytest

from muon_sr_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "muon_sr_b200.h")

PROGRAM = r"""
#include <stdio.h>
#include "muon_sr_b200.h"

typedef void (*fn_t)(void);
static const fn_t every_entry_point[] = { %s };

int main(void) {
  int64_t n = 0;
  int mode;
  if (msr_set_sr_noise(MSR_SR_NOISE_NONE) != MSR_OK) return 2;
  mode = msr_get_sr_noise();
  msr_set_sr_noise(MSR_SR_NOISE_REFERENCE);
  if (msr_gemm_tile_map(300, 300, 2, 1, 1, NULL, 0, &n) != MSR_OK) return 3;
  printf("%%d %%d %%lld %%d|%%s\n", msr_abi_version(), mode, (long long)n,
         (int)(sizeof(every_entry_point) / sizeof(every_entry_point[0])), msr_status_string(MSR_ERR_INVALID));
  return 0;
}
"""


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(msr_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_compiles_as_c_and_links(tmp_path):
    names = _declared()
    assert set(names) == {n for n, _, _ in _lib.SIGNATURES}  # the Python binding covers the header
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM % ", ".join(f"(fn_t){n}" for n in names))
    exe = tmp_path / "abi"
    libdir = os.path.dirname(_lib.LIB_PATH)
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", os.path.dirname(HEADER), str(src),
                         "-L", libdir, "-lmuon_sr_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, (run.returncode, run.stderr)
    numbers, status = run.stdout.strip().split("|")
    version, mode, tiles, count = (int(v) for v in numbers.split())
    # 2 matrices x the upper-triangle pair tiles of a 300 x 300 output (2 x 2 tiles: 3 of them)
    assert (version, mode, tiles, count) == (2, 2, 6, len(names))
    assert status == "invalid argument"
