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


def test_int8_qk_lane_words_match_q_order(tmp_path):
    """i8_word / i8_elem (pa_decode.cuh), compiled as host code: for both blocks of a Q8_0 pair and every lane of a
    quad, the two K words the int8-domain QK loads (lane 0's first even-block word joined with word 8 by PRMT 0x5432)
    carry, byte for byte, the block elements the lane's Q bytes are quantised from; the lanes together cover each
    block's 32 elements once; every word is 4-byte aligned inside the 68-byte pair and the scales sit where the kernel
    reads them (even block: word 0 bytes 0-1; odd block: word 8 bytes 2-3)."""
    src = tmp_path / "i8maps.cu"
    src.write_text(r'''
#include <cstdio>
#include <cstdint>
#include "pa_decode.cuh"
static uint32_t word(const uint8_t *p, int off) {
  return (uint32_t) p[off] | (uint32_t) p[off + 1] << 8 | (uint32_t) p[off + 2] << 16 | (uint32_t) p[off + 3] << 24;
}
static uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {   // byte permute of (b:a), the PTX prmt default mode
  uint64_t x = (uint64_t) b << 32 | a;
  uint32_t d = 0;
  for (int i = 0; i < 4; i++) d |= (uint32_t) ((x >> (8 * ((sel >> (4 * i)) & 7))) & 0xFF) << (8 * i);
  return d;
}
int main() {
  // a pair whose element bytes name themselves: even block element e = 0x40 + e, odd block element e = 0x80 + e
  uint8_t pair[68];
  pair[0] = 0xD0; pair[1] = 0xD1; pair[34] = 0xE0; pair[35] = 0xE1;
  for (int e = 0; e < 32; e++) { pair[2 + e] = (uint8_t) (0x40 + e); pair[36 + e] = (uint8_t) (0x80 + e); }
  if ((word(pair, 0) & 0xFFFF) != 0xD1D0u || (word(pair, 32) >> 16) != 0xE1E0u) { printf("scales\n"); return 1; }
  for (int odd = 0; odd < 2; odd++) {
    int seen[32] = {0};
    for (int t = 0; t < 4; t++) {
      uint32_t w[2];
      for (int k = 0; k < 2; k++) {
        const int off = pa::dec::i8_word(odd, t, k);
        if (off % 4 || off < 0 || off + 4 > 68) { printf("word offset %d\n", off); return 1; }
        w[k] = word(pair, off);
      }
      if (!odd) w[0] = prmt(w[0], word(pair, 32), t == 0 ? 0x5432u : 0x3210u);
      for (int i = 0; i < 8; i++) {
        const int e = pa::dec::i8_elem(odd, t, i);
        if (e < 0 || e > 31) { printf("element %d\n", e); return 1; }
        const uint8_t got = (uint8_t) (w[i / 4] >> (8 * (i % 4)));
        if (got != (uint8_t) ((odd ? 0x80 : 0x40) + e)) { printf("odd %d lane %d byte %d: %02x\n", odd, t, i, got); return 1; }
        seen[e]++;
      }
    }
    for (int e = 0; e < 32; e++) if (seen[e] != 1) { printf("element %d seen %d times\n", e, seen[e]); return 1; }
  }
  printf("ok\n");
  return 0;
}
''')
    exe = tmp_path / "i8maps"
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    r = subprocess.run([nvcc, "-std=c++17", "-I", os.path.join(ROOT, "backburner_b200", "csrc"), "-o", str(exe),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and "ok" in out.stdout, out.stdout + out.stderr


def test_pair_kernel_layouts_and_dequant_maps(tmp_path):
    """The CTA-pair tcgen05 kernel's shared-memory map and dequant addressing (pa_prefill_pair.cuh), compiled as host
    code, for Q8_0 / Q4_0, head dim 128 (NT = 1, 2) and 256, both CTAs of a pair and every head offset: the layout fits
    227 KB with 1024-aligned operand tiles and the TMEM columns fit 512; every raw-stage read of a lane (scale, three or
    two 16-byte words) stays inside its stage and covers its block's data bytes; and the items of one block write every
    16-byte chunk of the K and V operand buffers exactly once (dq_item / dq_row / dq_chunk)."""
    src = tmp_path / "pair_maps.cu"
    src.write_text(r'''
#include <cstdio>
#include <vector>
#include "pa_prefill_pair.cuh"
using namespace pa::pre;
template <int Q, int NT, int D> int check() {
  using L = PairSmem<Q, NT, D>;
  constexpr int GB = pa::dec::q_group_bytes(Q), HB = (D / 32) * GB, RAWB = L::RAWB;
  if (L::TOTAL + 1024 > 227 * 1024) { printf("smem %d\n", L::TOTAL); return 1; }
  if (L::K % 1024 || L::V % 1024 || L::RAW % 1024 || L::RAW_STAGE % 1024 || L::K_BUF % 1024 || L::V_BUF % 1024 ||
      L::RAW_V % 128) { printf("alignment\n"); return 1; }
  if (NT * L::TS > L::TMEM_COLS || L::TMEM_COLS > 512) { printf("tmem\n"); return 1; }
  const int nload = Q == 1 ? 3 : 2;
  for (uint32_t hoff : {0u, 8u}) {
    if (HB % 16 == 0 && hoff) continue;                 // heads of these sizes start 16-aligned
    if ((int) hoff + HB > RAWB) { printf("window\n"); return 1; }
    for (uint32_t cr = 0; cr < 2; cr++) for (int kv = 0; kv < 2; kv++) {
      std::vector<int> hit((kv == 0 ? L::K_BUF : L::V_BUF) / 16, 0);
      constexpr int NDQ = pair_dq_warps(D), NPASS = (D / 128) * 4 / NDQ;
      for (int ps = 0; ps < NPASS; ps++) for (uint32_t dw = 0; dw < (uint32_t) NDQ; dw++) for (uint32_t lane = 0; lane < 32; lane++) {
        uint32_t ql, qb, key;
        dq_item<D, NDQ>(kv, ps, dw, lane, cr, ql, qb, key);
        if (qb >= (uint32_t) (D / 32) || key >= (uint32_t) (kv == 0 ? BN / 2 : BN)) { printf("item\n"); return 1; }
        if (kv == 1 && qb / (D / 64) != cr) { printf("V block of the other CTA\n"); return 1; }
        const uint32_t rb = (kv == 0 ? 0u : (uint32_t) L::RAW_V) + key * RAWB;
        const uint32_t bo = hoff + GB * qb, w16 = bo & ~15u, lo = rb + w16, hi = rb + w16 + 16 * nload;
        if (hi > (uint32_t) L::RAW_STAGE || rb + bo + 2 > (uint32_t) L::RAW_STAGE) { printf("read past stage\n"); return 1; }
        if (bo + GB > w16 + 16 * nload) { printf("block not covered\n"); return 1; }
        (void) lo;
        for (uint32_t cc = 0; cc < 4; cc++) {
          const uint32_t off = dq_row(kv, ql, key) + dq_chunk(ql, key, cc);
          // the UMMA K-major 128-byte-swizzle layout: chunk cc holds tile dims 32 ql + 8 cc of row `key`; 8-row atoms
          // 1024 B apart, 64-dim atom columns (rows x 128 B) apart, 16-byte chunk j of row r at (j ^ r % 8) * 16
          const uint32_t dd = 32 * ql + 8 * cc, rows = kv == 0 ? BN / 2 : BN, j = (dd % 64) / 8;
          const uint32_t want = (dd / 64) * rows * 128 + (key / 8) * 1024 + (key % 8) * 128 + ((j ^ (key % 8)) * 16);
          if (off != want) { printf("not the swizzled layout (kv%d ql%u key%u cc%u)\n", kv, ql, key, cc); return 1; }
          if (off % 16 || off + 16 > (uint32_t) (kv == 0 ? L::K_BUF : L::V_BUF)) { printf("write out of buffer\n"); return 1; }
          hit[off / 16]++;
        }
      }
      for (int h : hit) if (h != 1) { printf("chunk written %d times (q%d nt%d d%d kv%d)\n", h, Q, NT, D, kv); return 1; }
    }
  }
  return 0;
}
int main() {
  if (check<1, 1, 128>() || check<1, 2, 128>() || check<2, 1, 128>() || check<2, 2, 128>() || check<1, 1, 256>() ||
      check<2, 1, 256>()) return 1;
  printf("ok\n");
  return 0;
}
''')
    exe = tmp_path / "pair_maps"
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    r = subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-I",
                        os.path.join(ROOT, "backburner_b200", "csrc"), "-I", os.path.join(ROOT, "include"), "-o", str(exe),
                        str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and "ok" in out.stdout, out.stdout + out.stderr


def test_nccl_unique_id_without_a_gpu():
    """pa_cuda_nccl_unique_id opens NCCL on first use (no link dependency of libpacuda.so on it) and needs no GPU."""
    import backburner_b200 as pa
    a, b = pa.nccl_unique_id(), pa.nccl_unique_id()
    assert len(a) == 128 and a != b
