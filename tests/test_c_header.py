"""The C ABI from C: a C99 program that includes include/mamba_b200_ss.h, compiled by gcc and linked
against the library, checks without a GPU that the header's struct layouts as a C compiler lays
them out equal the library's (ss_struct_size), the ABI version, the size helpers, and that bad
arguments come back as status codes before any device access.  This is what an FFI binding
(cgo, JNI, a plain C host) relies on."""
import os
import shutil
import subprocess

import pytest

import mamba_b200._lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_SRC = r"""
#include <stdio.h>
#include <string.h>
#include "mamba_b200_ss.h"

#define CHECK(cond) do { if (!(cond)) { printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #cond); return 1; } } while (0)

int main(void) {
  const size_t sizes[] = {sizeof(ss_fwd_args), sizeof(ss_bwd_args), sizeof(ss_step_args), sizeof(ss_conv_args),
                          sizeof(ss_conv_bwd_args), sizeof(ss_conv_step_args), sizeof(ss_rmsnorm_args),
                          sizeof(ss_rmsnorm_bwd_args), sizeof(ss_mamba_step_args)};
  CHECK(ss_abi_version() == SS_ABI_VERSION);
  for (int i = 0; i < (int)(sizeof(sizes) / sizeof(sizes[0])); ++i) CHECK(ss_struct_size(i) == sizes[i]);
  CHECK(ss_struct_size(99) == 0);
  CHECK(ss_ckpt_elems(2, 64, 33, 16) == (size_t)2 * 3 * 16 * 64);
  CHECK(ss_work_elems(2, 64, 33, 16) == 0);
  CHECK(ss_work_elems(2, 64, 33, 32) == (size_t)2 * 2 * 64 * 33);
  CHECK(strcmp(ss_status_string(SS_OK), "ok") == 0);
  ss_fwd_args f;
  memset(&f, 0, sizeof f);
  f.batch = 2; f.dim = 64; f.seqlen = 128; f.dstate = 16; f.ngroups = 1;
  f.io_dtype = f.bc_dtype = SS_F32;
  CHECK(ss_fwd(&f, NULL) == SS_ERR_INVALID);          /* no tensors */
  f.dstate = SS_MAX_DSTATE + 1;
  CHECK(ss_fwd(&f, NULL) == SS_ERR_UNSUPPORTED);
  CHECK(ss_fwd(NULL, NULL) == SS_ERR_INVALID);
  CHECK(ss_bwd(NULL, NULL) == SS_ERR_INVALID);
  CHECK(ss_bwd_noalloc(NULL, NULL) == SS_ERR_INVALID);
  printf("ok\n");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_program_against_the_header(tmp_path):
    L.lib()  # builds nothing; fails loudly when the library is missing
    src = tmp_path / "abi_check.c"
    exe = tmp_path / "abi_check"
    src.write_text(C_SRC)
    libdir = os.path.dirname(L.LIB_PATH)
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
           "-L", libdir, "-lmamba_b200_ss", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
