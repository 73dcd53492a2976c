"""A plain C host compiles against include/gfield.h, links libgfield.so and
uses the host-side entry points (no GPU needed: every call below fails or
returns before the first CUDA operation)."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

from guass_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent

SRC = r'''
#include <stdio.h>
#include <string.h>
#include "gfield.h"
int main(void) {
  if (gf_abi_version() != GF_ABI_VERSION) return 1;
  if (gf_num_tiles(320, 768, 32, 32) != 240) return 2;
  gf_config cfg = {32, 32, 3.0, 0, 1, 80.0, 1.0f, GF_F32, GF_F32};
  gf_field f;
  memset(&f, 0, sizeof(f));
  f.out_features = 320; f.in_features = 768; f.num_gaussians = 256;
  gf_batch b = {1, &f, NULL, 0, NULL};
  size_t fwd = gf_workspace_bytes(&cfg, &b, GF_PASS_FORWARD);
  f.ids_capacity = 5000;
  size_t bwd = gf_workspace_bytes(&cfg, &b, GF_PASS_BACKWARD);
  if (fwd == 0 || bwd < fwd + 32 * 5000) return 3;
  /* missing inputs are rejected before any device work */
  if (gf_forward(&cfg, &b, NULL, 0, NULL) != GF_ERR_INVALID_ARG) return 4;
  if (strstr(gf_last_error(), "non-null") == NULL) return 5;
  cfg.tile_out = 0;
  if (gf_forward(&cfg, &b, NULL, 0, NULL) != GF_ERR_INVALID_ARG) return 6;
  if (strcmp(gf_last_error(), "tile_out must be positive") != 0) return 7;
  if (gf_multicast_store(NULL, NULL, 16, 1, NULL) != GF_ERR_INVALID_ARG) return 8;
  /* extensions: staged forward, densify statistics (argument errors, host side) */
  cfg.tile_out = 32;
  if (gf_forward_stages(&cfg, &b, NULL, 0, 0u, NULL) != GF_ERR_INVALID_ARG) return 9;
  if (gf_forward_stages(&cfg, &b, NULL, 0, GF_STAGE_BIN | 4u, NULL) != GF_ERR_INVALID_ARG) return 10;
  gf_stats_layer layer;
  memset(&layer, 0, sizeof(layer));
  layer.num_gaussians = 8; /* stats missing */
  if (gf_grad_stats_accumulate(1, &layer, NULL) != GF_ERR_INVALID_ARG) return 11;
  if (gf_grad_stats_accumulate(0, NULL, NULL) != GF_OK) return 12;
  cfg.flags = GF_CFG_BWD_EXP2; /* an option bit is accepted by the host checks */
  if (gf_workspace_bytes(&cfg, &b, GF_PASS_BACKWARD) == 0) return 13;
  printf("ok %zu %zu\n", fwd, bwd);
  return 0;
}
'''


def test_c_host_links_and_calls(tmp_path):
    src = tmp_path / "host.c"
    src.write_text(SRC)
    exe = tmp_path / "host"
    libdir = _lib.LIB_PATH.parent
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(src), "-o", str(exe), f"-L{libdir}",
                    "-l:libgfield.so", f"-Wl,-rpath,{libdir}"], check=True)
    env = dict(os.environ)
    env["LD_LIBRARY_PATH"] = ":".join(p for p in ("/usr/local/cuda/lib64", env.get("LD_LIBRARY_PATH", "")) if p)
    out = subprocess.run([str(exe)], capture_output=True, text=True, env=env)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("ok ")
