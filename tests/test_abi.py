"""The drop-in boundary without a GPU: libpacuda.so loads and exports every entry point include/pa_cuda.h declares,
the host-side helpers agree with the reference's formats, and the kernels' head-dim permutations are permutations."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import backburner_b200 as pa

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pa_cuda_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(pa.lib_path)
    names = _declared("pa_cuda.h")
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # the ctypes binding covers them too
    from backburner_b200 import api
    assert not [n for n in names if n not in api._SIGS], [n for n in names if n not in api._SIGS]


def test_abi_version_and_no_gpu_answer():
    L = pa.lib()
    assert L.pa_cuda_abi_version() == 1
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if not has_gpu:
        assert L.pa_cuda_available() == 0
        assert not pa.available()


def test_create_without_gpu_fails_cleanly():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("GPU present")
    except Exception:
        pass
    with pytest.raises(pa.PaCudaError):
        pa.Context(0)


def test_shapes_and_head_bytes():
    assert pa.head_bytes(pa.Q8_0, 128) == 136 and pa.head_bytes(pa.Q4_0, 128) == 72
    assert pa.head_bytes(pa.Q8_0, 256) == 272 and pa.head_bytes(pa.Q4_0, 256) == 144
    s = pa.shape_for(128, 8, 5, pa.Q8_0)
    assert s.rs == 1088 and s.hb == 136
    assert pa.shape_for(256, 4, 48, pa.Q4_0).rs == 576


def test_kernel_head_dim_maps_are_permutations(tmp_path):
    """dK / dV (pa_decode.cuh) decide which head dim each MMA fragment slot carries: compiled as host code they must
    be permutations of 0..hd-1, dK must keep each lane inside its own quant block(s), and dV inside one block (f16
    rows: each k-step / m-tile inside its own 16 dims, the ldmatrix fragment order)."""
    src = tmp_path / "maps.cu"
    src.write_text(r'''
#include <cstdio>
#include "pa_decode.cuh"
int main() {
  for (int quant = 0; quant <= 2; quant++) for (int hd = 128; hd <= 256; hd += 128) {
    int seen[256] = {0};
    for (int s = 0; s < hd / 16; s++) for (int t = 0; t < 4; t++) for (int i = 0; i < 4; i++) {
      int d = pa::dec::dK(quant, s, t, i);
      if (d < 0 || d >= hd) { printf("dK out of range\n"); return 1; }
      if (quant && d / 32 != t + 4 * (s / 8)) { printf("dK leaves the lane's block\n"); return 1; }
      if (!quant && d / 16 != s) { printf("dK (f16) leaves the k-step's 16 dims\n"); return 1; }
      seen[d]++;
    }
    for (int d = 0; d < hd; d++) if (seen[d] != 1) { printf("dK not a permutation q%d hd%d d%d\n", quant, hd, d); return 1; }
    int seen2[256] = {0};
    for (int mt = 0; mt < hd / 16; mt++) for (int g = 0; g < 8; g++) for (int h = 0; h < 2; h++) {
      int d = pa::dec::dV(quant, hd, mt, g, h);
      if (d < 0 || d >= hd) { printf("dV out of range\n"); return 1; }
      if (quant && d / 32 != (hd == 128 ? g / 2 : g)) { printf("dV leaves the lane's block\n"); return 1; }
      if (!quant && d / 16 != mt) { printf("dV (f16) leaves the m-tile's 16 dims\n"); return 1; }
      seen2[d]++;
    }
    for (int d = 0; d < hd; d++) if (seen2[d] != 1) { printf("dV not a permutation q%d hd%d d%d\n", quant, hd, d); return 1; }
  }
  printf("ok\n");
  return 0;
}
''')
    exe = tmp_path / "maps"
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    r = subprocess.run([nvcc, "-std=c++17", "-I", os.path.join(ROOT, "backburner_b200", "csrc"), "-o", str(exe),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and "ok" in out.stdout, out.stdout + out.stderr
