"""The C ABI from C: both headers compile as C99 and a C program links the two
libraries and runs their host-only entry points (no GPU needed).

This is the boundary a non-Python caller binds (the reference's C++ CLI, a
cgo or JNI stub): plain C types only, status codes, no exceptions.
"""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "quiver_b200.h"
#include "quiver_b200_build.h"

int main(int argc, char** argv) {
  qv_search_opts so;
  qv_stream_opts sto;
  qv_index_info info;
  uint8_t base[40 * 8];
  int i, rc;
  if (argc != 2) return 90;
  if (strncmp(qv_version(), "quiver-b200", 11) != 0) return 91;
  qv_search_opts_default(&so);
  if (so.topk != 10 || so.ef_search <= 0) return 92;
  qv_stream_opts_default(&sto);
  if (sto.admit_min_batch != 32 || sto.prefeed != -1) return 93;
  /* host-only index parse */
  memset(&info, 0, sizeof(info));
  rc = qv_index_probe(argv[1], QV_UINT8, &info);
  if (rc != QV_OK) { fprintf(stderr, "%s\n", qv_last_error()); return 94; }
  printf("%lld %lld %lld %d\n", (long long)info.num_points, (long long)info.dim, (long long)info.max_degree,
         (int)info.num_chunks);
  /* errors come back as codes with a message, never as a crash */
  rc = qv_index_probe("/nonexistent-index-dir", QV_UINT8, &info);
  if (rc != QV_ERR_IO || strlen(qv_last_error()) == 0) return 95;
  if (qv_adc_batch(NULL, 10, 200, NULL, 1, NULL, NULL, 5, NULL, QV_ADC_AUTO, NULL) != QV_ERR_INVALID_ARG) return 96;
  /* the build library: host synthesis is deterministic */
  for (i = 0; i < 2; ++i) {
    uint8_t again[40 * 8];
    if (qvb_synth_mixture(7, 0, 0, 40, 8, 3, 20.0, QV_UINT8, i ? again : base, 1) != 0) {
      fprintf(stderr, "%s\n", qvb_last_error());
      return 97;
    }
    if (i && memcmp(base, again, sizeof(base)) != 0) return 98;
  }
  return 0;
}
"""


@pytest.fixture(scope="module")
def libs():
    from quiver_b200 import _build, _lib
    _build.build_engine()
    _lib.index_lib()  # builds libqv_index.so when missing
    return REPO / "quiver-ae_b200" / "lib"


def test_c_program_links_and_calls_the_abi(tmp_path, libs, u8_index):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    cmd = [gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", str(REPO / "include"), str(src), "-o", str(exe),
           "-L", str(libs), "-lquiver_b200", "-lqv_index", f"-Wl,-rpath,{libs}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe), str(u8_index["dir"])], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, (run.returncode, run.stderr)
    n, dim, R, M = map(int, run.stdout.split())
    assert (n, dim, R, M) == (u8_index["base"].shape[0], u8_index["base"].shape[1], 64, 32)


SIZES = r"""
#include <stdio.h>
#include "quiver_b200.h"
int main(void) {
  printf("qv_index_info %zu\n", sizeof(qv_index_info));
  printf("qv_engine_opts %zu\n", sizeof(qv_engine_opts));
  printf("qv_index_arrays %zu\n", sizeof(qv_index_arrays));
  printf("qv_search_opts %zu\n", sizeof(qv_search_opts));
  printf("qv_search_stats %zu\n", sizeof(qv_search_stats));
  printf("qv_stream_opts %zu\n", sizeof(qv_stream_opts));
  printf("qv_stream_stats %zu\n", sizeof(qv_stream_stats));
  return 0;
}
"""


def test_python_structures_have_the_c_sizes(tmp_path):
    """Every ctypes mirror of a header struct has the size the C compiler gives it, so no field was added
    on one side only."""
    import ctypes as C
    from quiver_b200 import _lib
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = tmp_path / "sizes.c"
    src.write_text(SIZES)
    exe = tmp_path / "sizes"
    res = subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", str(REPO / "include"), str(src), "-o",
                          str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    sizes = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                          check=True).stdout.splitlines())
    mirror = {"qv_index_info": _lib.IndexInfo, "qv_engine_opts": _lib.EngineOpts,
              "qv_index_arrays": _lib.IndexArrays, "qv_search_opts": _lib.SearchOpts,
              "qv_search_stats": _lib.SearchStats, "qv_stream_opts": _lib.StreamOpts,
              "qv_stream_stats": _lib.StreamStats}
    assert set(sizes) == set(mirror)
    for name, cls in mirror.items():
        assert C.sizeof(cls) == int(sizes[name]), f"{name}: C {sizes[name]} bytes, ctypes {C.sizeof(cls)}"
