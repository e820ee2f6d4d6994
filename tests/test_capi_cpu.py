"""libblut.so without a GPU: it loads, exports every symbol of include/blut.h,
and its host-side argument checks answer before any CUDA call."""
import ctypes as C
import inspect
import os
import re
import shutil
import subprocess
from types import SimpleNamespace

import pytest
import torch

from tests.conftest import ROOT

from block_lut_b200 import _lib
from block_lut_b200.formats import LUTFormat, tiled_bytes
from block_lut_b200.moe import LUTMoELayer

HEADER = os.path.join(ROOT, "include", "blut.h")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"BLUT_API\s+[\w\s\*]+?\b(blut_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = header_symbols()
    assert len(declared) >= 15
    for name in declared:
        assert hasattr(lib, name), name
    # the ctypes table covers exactly the header
    assert sorted(n for n, _, _ in _lib.SIGNATURES) == declared
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = sorted(set(re.findall(r"\bT (blut_\w+)", out)))
    assert exported == declared


def test_status_strings():
    for rc in (0, -1, -2, -3, -4, -5, -6):
        assert _lib.status_string(rc)
    assert "unknown" in _lib.status_string(-99)


@pytest.mark.parametrize("fmt,bpw", [
    (LUTFormat("b", 4, 64), 1.0), (LUTFormat("b", 2, 64), 0.375), (LUTFormat("b", 3, 64), 0.625),
    (LUTFormat("b", 4, 32), 1.5), (LUTFormat("b", 2, 128), 0.3125),
    (LUTFormat("nested", 4, 64, 1), 0.375), (LUTFormat("r8", 8, 128), 1 + 2 / 128),
])
def test_tiled_bytes_match_format_bytes(fmt, bpw):
    rows, cols = 1408, 2048
    n = tiled_bytes(fmt, rows, cols)
    assert abs(fmt.bytes_per_weight() - bpw) < 1e-9
    # the buffer holds every plane (NestedLUT: both tiers, 0.25+0.125+0.25+0.5 B per
    # weight); planes are 256-aligned, so at most 256 B of padding per plane
    stored = 1.125 if fmt.kind == "nested" else bpw
    assert rows * cols * stored <= n <= rows * cols * stored + 4 * 256


@pytest.mark.parametrize("fmt,bpw", [
    (LUTFormat("b", 4, 64), 1.0), (LUTFormat("b", 4, 32), 1.5), (LUTFormat("b", 4, 128), 0.75),
    (LUTFormat("b", 3, 32), 0.875), (LUTFormat("b", 3, 64), 0.625), (LUTFormat("b", 3, 128), 0.5),
    (LUTFormat("b", 2, 32), 0.5), (LUTFormat("b", 2, 64), 0.375), (LUTFormat("b", 2, 128), 0.3125),
    # NestedLUT stores both tiers: 2 x 0.25 B of codes + (8 + 32) B of tables per block
    (LUTFormat("nested", 4, 32, 0), 1.75), (LUTFormat("nested", 4, 64, 1), 1.125),
    (LUTFormat("nested", 4, 128, 0), 0.8125),
    # Format R stores its absmax once per 64 columns in this layout (1 + 2/64)
    (LUTFormat("r8", 8, 128), 1 + 2 / 64),
    (LUTFormat("dense", 16, 0, dense_dtype=torch.float16), 2.0),
    (LUTFormat("dense", 16, 0, dense_dtype=torch.bfloat16), 2.0),
])
@pytest.mark.parametrize("paired", [False, True])
def test_tc_tiled_bytes_are_the_format_bytes(fmt, bpw, paired):
    """The tcgen05 layout stores exactly the format's bytes (no padding at these shapes)."""
    for rows, cols in ((2816, 2048), (2048, 1408), (11264, 2048), (2048, 5632)):
        assert tiled_bytes(fmt, rows, cols, paired, tc=True) == rows * cols * bpw


def test_tc_layout_availability():
    b4 = LUTFormat("b", 4, 64)
    assert b4.has_tc_layout(2816, 2048, paired=True) and b4.has_tc_layout(2048, 1408)
    assert not b4.has_tc_layout(2688, 2048, paired=True)        # paired rows % 256
    assert not b4.has_tc_layout(2048 + 48, 2048)                 # rows % 128
    assert not b4.has_tc_layout(2048, 1408 + 32)                 # cols % 64
    for fmt in (LUTFormat("b", 2, 64), LUTFormat("b", 3, 32), LUTFormat("b", 3, 128),
                LUTFormat("nested", 4, 64, 0), LUTFormat("nested", 4, 64, 1)):
        assert fmt.has_tc_layout(1536, 2048, paired=True) and fmt.has_tc_layout(2048, 768)
    r8 = LUTFormat("r8", 8, 128)
    assert r8.has_tc_layout(2816, 2048, paired=True) and r8.has_tc_layout(2048, 1408)
    assert not r8.has_tc_layout(2048, 1408 + 64)                    # absmax blocks must stay in a row


def test_moe_forward_rejects_mixed_matmul_paths():
    fmt = LUTFormat("b", 4, 64)
    a = _args(w13=fmt.desc(2816, 2048, paired=True, tc=True),
              w13_stride=tiled_bytes(fmt, 2816, 2048, True, tc=True))
    assert _lib.lib().blut_moe_forward(C.byref(a), None, 0, None) == _lib.BLUT_ERR_INVALID


def test_tiled_bytes_rejects_bad_shapes():
    with pytest.raises(ValueError):
        tiled_bytes(LUTFormat("b", 4, 64), 1400, 2048)  # rows % 16
    with pytest.raises(ValueError):
        tiled_bytes(LUTFormat("b", 4, 64), 1408, 2000)  # cols % 128


def _args(**kw):
    fmt = LUTFormat("b", 4, 64)
    a = _lib.MoEArgs()
    a.num_tokens, a.hidden, a.inter, a.num_experts, a.top_k, a.dtype = 8, 2048, 1408, 60, 4, _lib.F16
    a.w13, a.w2 = fmt.desc(2816, 2048, paired=True), fmt.desc(2048, 1408)
    a.w13_tiled = a.w2_tiled = a.x = a.out = 1 << 20
    a.w13_stride, a.w2_stride = tiled_bytes(fmt, 2816, 2048), tiled_bytes(fmt, 2048, 1408)
    a.topk_ids = a.topk_weights = 1 << 21
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_moe_workspace_size_host_only():
    lib = _lib.lib()
    n = lib.blut_moe_workspace_size(C.byref(_args()))
    assert n > 8 * 4 * 2048 * 4  # holds at least the fp32 expert outputs
    assert lib.blut_moe_workspace_size(C.byref(_args(num_tokens=0))) == 0
    assert lib.blut_moe_workspace_size(C.byref(_args(hidden=2000))) == 0


@pytest.mark.parametrize("kw,rc", [
    (dict(num_tokens=0), _lib.BLUT_ERR_INVALID),
    (dict(x=None), _lib.BLUT_ERR_INVALID),
    (dict(topk_ids=None), _lib.BLUT_ERR_INVALID),  # no routing and no router weights
    (dict(num_tokens=1 << 21), _lib.BLUT_ERR_UNSUPPORTED),  # T*k beyond 4M slots
    (dict(x=(1 << 20) + 2), _lib.BLUT_ERR_INVALID),  # misaligned activations
    (dict(w13_stride=1024), _lib.BLUT_ERR_INVALID),
])
def test_moe_forward_rejects_bad_arguments_before_launching(kw, rc):
    lib = _lib.lib()
    assert lib.blut_moe_forward(C.byref(_args(**kw)), None, 0, None) == rc


def test_top_k_above_the_expert_count_needs_caller_routing():
    """The router picks k distinct experts, so k > E is refused when the
    library routes.  With the caller's ids it is a valid layer: under expert
    parallelism a rank may own fewer experts than k (its other slots are -1)."""
    lib = _lib.lib()
    a = _args(num_experts=2, top_k=8)
    assert lib.blut_moe_workspace_size(C.byref(a)) > 0
    a.topk_ids, a.router_w = None, 1 << 22
    assert lib.blut_moe_workspace_size(C.byref(a)) == 0
    assert lib.blut_moe_forward(C.byref(a), None, 0, None) == _lib.BLUT_ERR_UNSUPPORTED
    a.top_k = 2
    assert lib.blut_moe_workspace_size(C.byref(a)) > 0
    assert lib.blut_moe_workspace_size(C.byref(_args(top_k=33))) == 0


def test_moe_forward_rejects_small_workspace():
    lib = _lib.lib()
    assert lib.blut_moe_forward(C.byref(_args()), 1 << 22, 16, None) == _lib.BLUT_ERR_WORKSPACE


def test_launch_count():
    lib = _lib.lib()
    # plan, gather, gate/up, down, combine; the tcgen05 layout at T = 8 also
    # splits the gate/up pass over K, which adds its slice-sum kernel
    assert lib.blut_moe_launch_count(C.byref(_args())) == 5
    fmt = LUTFormat("b", 4, 64)
    tc = _args(w13=fmt.desc(2816, 2048, paired=True, tc=True), w2=fmt.desc(2048, 1408, tc=True))
    assert lib.blut_moe_launch_count(C.byref(tc)) == 6
    tc.num_tokens = 256  # enough items without a split
    assert lib.blut_moe_launch_count(C.byref(tc)) == 5
    tc.num_tokens, tc.topk_ids = 4096, None  # prefill with routing: router, top-k, plan, gather, 2 matmuls, combine
    tc.router_w = 1 << 22
    assert lib.blut_moe_launch_count(C.byref(tc)) == 7
    # one token on the tcgen05 layout runs the single-token path: route,
    # gate/up (with SiLU * up), down (with the combine), routed or not
    tc.num_tokens = 1
    assert lib.blut_moe_launch_count(C.byref(tc)) == 3
    tc.topk_ids, tc.router_w = 1 << 22, None
    assert lib.blut_moe_launch_count(C.byref(tc)) == 3
    mma = _args(num_tokens=1, topk_ids=None, router_w=1 << 22)
    assert lib.blut_moe_launch_count(C.byref(mma)) == 6


@pytest.mark.parametrize("E,k,I,world,cap", [(60, 4, 1408, 8, 32), (128, 8, 768, 8, 64)])
def test_expected_slots_steer_the_split_of_expert_parallel_rows(E, k, I, world, cap):
    """One rank of an 8-way expert-parallel decode gets world * cap rows with
    all k slots each, about E_local / E of them non-empty.  Counted as full,
    the slots look like a prefill batch (128-token groups, no K split, too
    few work items for the SMs); with expected_slots the gate/up pass is
    split over K again, which adds its slice-sum launch.  Buffers still
    cover every slot, so the workspace only grows."""
    lib = _lib.lib()
    fmt = LUTFormat("b", 4, 64)
    e_local = -(-E // world)
    a = _args(num_experts=e_local, top_k=k, inter=I, num_tokens=world * cap,
              w13=fmt.desc(2 * I, 2048, paired=True, tc=True), w2=fmt.desc(2048, I, tc=True),
              w13_stride=tiled_bytes(fmt, 2 * I, 2048, True, tc=True), w2_stride=tiled_bytes(fmt, 2048, I, tc=True))
    n_full, ws_full = lib.blut_moe_launch_count(C.byref(a)), lib.blut_moe_workspace_size(C.byref(a))
    layer = SimpleNamespace(top_k=k, slot_fraction=e_local / E)
    a.expected_slots = LUTMoELayer._expected_slots(layer, world * cap)
    assert 0 < a.expected_slots < world * cap * k
    assert lib.blut_moe_launch_count(C.byref(a)) == n_full + 1
    assert lib.blut_moe_workspace_size(C.byref(a)) >= ws_full
    # no hint (0) or a count of at least T*k leaves the split as it was
    for v in (0, world * cap * k, 1 << 30):
        a.expected_slots = v
        assert lib.blut_moe_launch_count(C.byref(a)) == n_full
        assert lib.blut_moe_workspace_size(C.byref(a)) == ws_full
    assert LUTMoELayer._expected_slots(SimpleNamespace(top_k=k, slot_fraction=1.0), 64) == 0


LAYOUT_PROBE = r"""
#include <cstdio>
#include <set>
#include "blut_common.cuh"
using namespace blut;
// every (row, k) of a (tile, chunk) piece must map to a distinct bit range inside the piece
template <class F> int check(const char* name, int piece_bytes, int bits, F pos) {
  std::set<long> used;
  for (int r = 0; r < 16; ++r)
    for (int k = 0; k < 128; ++k) {
      int word, bit;
      pos(r, k, word, bit);
      for (int b = 0; b < bits; ++b) {
        long g = (long)word * 32 + bit + b;
        if (g < 0 || g >= (long)piece_bytes * 8 || bit + b >= 32 || !used.insert(g).second) {
          printf("%s: bad position r=%d k=%d\n", name, r, k);
          return 1;
        }
      }
    }
  if ((long)used.size() != (long)piece_bytes * 8) { printf("%s: not dense\n", name); return 1; }
  return 0;
}
int main() {
  int bad = 0;
  bad |= check("codes4", 1024, 4, codes4_pos);
  bad |= check("codes2", 512, 2, codes2_pos);
  bad |= check("codes1", 256, 1, codes1_pos);
  bad |= check("codes8", 2048, 8, codes8_pos);
  bad |= check("dense", 4096, 16, [](int r, int k, int& w, int& b) { int o = dense_byte(r, k); w = o / 4; b = 8 * (o % 4); });
  bad |= check("bfrag", 2048, 16, [](int n, int k, int& w, int& b) { int o = bfrag_byte(n % 8, k); w = o / 4 + (n / 8) * 512; b = 8 * (o % 4); });
  // fragment ownership: lane (g, t) holds rows g, g+8 and columns {2t, 2t+1, 2t+8, 2t+9} of each slab
  for (int r = 0; r < 16; ++r) for (int k = 0; k < 128; ++k) {
    FragPos p = frag_pos(r, k);
    int kk = k & 15, col = 2 * (p.lane & 3) + (p.q & 1) + 8 * (p.q >> 1);
    if (p.lane / 4 != (r & 7) || p.h != r / 8 || col != kk || p.s != k / 16) { printf("frag_pos r=%d k=%d\n", r, k); bad = 1; }
  }
  printf(bad ? "FAIL\n" : "OK\n");
  return bad;
}
"""


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="needs nvcc for the host-side layout probe")
def test_tiled_layout_position_maps_are_bijective(tmp_path):
    # dense bfrag check covers 16 tokens (two n-tiles side by side) -> use a 2-tile piece size
    src = tmp_path / "probe.cu"
    src.write_text(LAYOUT_PROBE.replace('check("bfrag", 2048', 'check("bfrag", 4096'))
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "probe"
    r = subprocess.run([nvcc, "-std=c++17", "-I", os.path.join(ROOT, "block_lut_b200", "csrc"), str(src), "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout


def test_matmul_workspace_and_launches():
    """blut_matmul's host-side checks: sizes, layouts and launch count, without a GPU call."""
    lib = _lib.lib()
    for fmt, tc in ((LUTFormat("b", 4, 64), True), (LUTFormat("b", 2, 64), False), (LUTFormat("r8", 8, 128), False)):
        d = fmt.desc(2048, 1408, tc=tc)
        for m in (1, 32, 4096):
            n = lib.blut_matmul_workspace_size(C.byref(d), m)
            assert n >= m * 1408 * 2 + m * 2048 * 4          # activations + fp32 rows
            # one token on the TC layout: the single-token GEMV alone
            assert lib.blut_matmul_launch_count(C.byref(d), m) == (1 if m == 1 and d.layout & _lib.LAYOUT_TC else 3)
        assert lib.blut_matmul_workspace_size(C.byref(d), 0) == 0
        assert lib.blut_matmul_workspace_size(C.byref(d), (1 << 20) + 1) == 0
    paired = LUTFormat("b", 4, 64).desc(2816, 2048, paired=True, tc=True)
    assert lib.blut_matmul_workspace_size(C.byref(paired), 8) == 0
    assert lib.blut_matmul_launch_count(C.byref(paired), 8) == _lib.BLUT_ERR_INVALID
    d = LUTFormat("b", 4, 64).desc(2048, 1408, tc=True)
    assert lib.blut_matmul(C.byref(d), None, None, None, 8, None, 0, None, 0, None) == _lib.BLUT_ERR_INVALID


def test_bitplane_host_checks():
    lib = _lib.lib()
    # sections read per tier: low (n/2), low + mid (3n/4), all (n)
    assert [lib.blut_bitplane_bytes(4100, t) for t in (2, 1, 0)] == [2050, 3075, 4100]
    for n, t in ((4102, 0), (0, 0), (-4, 1), (64, 3), (64, -1)):
        assert lib.blut_bitplane_bytes(n, t) == _lib.BLUT_ERR_INVALID
    # argument checks answer before any launch
    assert lib.blut_bitplane_pack(None, None, 64, None) == _lib.BLUT_ERR_INVALID
    assert lib.blut_bitplane_pack(1 << 20, 1 << 21, 66, None) == _lib.BLUT_ERR_UNSUPPORTED
    assert lib.blut_bitplane_recover(1 << 20, 1 << 21, 1 << 22, 1 << 23, 64, 3, 128, None) == _lib.BLUT_ERR_INVALID
    assert lib.blut_bitplane_recover(1 << 20, 1 << 21, 1 << 22, 1 << 23, 66, 0, 128, None) == \
        _lib.BLUT_ERR_UNSUPPORTED
    assert lib.blut_bitplane_recover(1 << 20, 1 << 21, 1 << 22, 1 << 23, 64, 0, 0, None) == _lib.BLUT_ERR_INVALID


C_CALLER = r"""
#include <stdio.h>
#include <string.h>
#include "blut.h"

int main(void) {
  blut_mat_desc d;
  memset(&d, 0, sizeof d);
  d.format = BLUT_FMT_B; d.bits = 4; d.group = 64; d.dtype = BLUT_F16;
  d.layout = BLUT_LAYOUT_TC; d.rows = 2816; d.cols = 2048;
  if (blut_tiled_bytes(&d) != 2816LL * 2048) return 1;            /* 1 byte per weight at 4-bit g64 */
  if (blut_bitplane_bytes(4100, 1) != 3075) return 2;
  if (blut_bitplane_bytes(4102, 0) != BLUT_ERR_INVALID) return 3;
  if (blut_bitplane_pack(NULL, NULL, 64, NULL) != BLUT_ERR_INVALID) return 4;
  if (strcmp(blut_status_string(BLUT_OK), "ok") != 0) return 5;
  blut_moe_args a;
  memset(&a, 0, sizeof a);
  if (blut_moe_workspace_size(&a) != 0) return 6;                  /* an empty layer needs nothing */
  puts("c caller ok");
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_compiles_as_c99_and_links(tmp_path):
    """A native caller (the HF engine's C/C++ side) includes blut.h as plain C,
    links libblut.so, and gets host-side answers without a GPU."""
    src = tmp_path / "caller.c"
    src.write_text(C_CALLER)
    exe = tmp_path / "caller"
    libdir = os.path.dirname(_lib.LIB_PATH)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(src), "-L", libdir, "-lblut", "-Wl,-rpath," + libdir, "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "c caller ok" in r.stdout, (r.returncode, r.stdout, r.stderr)


def test_fused_lut_gemv_rejects_blocks_below_128():
    from block_lut_b200.fused_kernel import fused_lut_gemv
    z = torch.zeros(4)
    with pytest.raises(ValueError, match="128"):
        fused_lut_gemv(z, torch.zeros(2, 4, dtype=torch.uint8), z, z, block_size=64)


@pytest.mark.parametrize("block,nb_short", [(256, 0), (384, 0), (512, 3)])
def test_fused_lut_gemv_absmax_expansion_keeps_the_reference_block_index(block, nb_short):
    """Blocks of a multiple of 128 reach the 128-element kernel through one
    scale per 128 elements; each flat element must get the scale of the
    reference's saturating block index, min(flat // block, nb - 1)
    (fused_kernel.py:40-44), including an absmax shorter than the matrix
    needs (nb_short scales missing)."""
    from block_lut_b200.fused_kernel import absmax_per_128
    m, k = 6, 640
    n = m * k
    nb = -(-n // block) - nb_short
    am = torch.arange(1, nb + 1, dtype=torch.float32)
    e = absmax_per_128(am, block, n)
    assert e.numel() == -(-n // 128)
    flat = torch.arange(n)
    kernel_scale = e[(flat // 128).clamp(max=e.numel() - 1)]  # what blut_lut_gemv reads
    reference_scale = am[(flat // block).clamp(max=nb - 1)]
    assert torch.equal(kernel_scale, reference_scale)


def test_ep_window_layout_and_argument_checks():
    """The expert-parallel window: a 256-byte header, the slot table, then the
    received rows, ids, weights and fp32 output rows of every source, each
    256-aligned; out-of-range sizes give 0 and the entry points refuse bad
    descriptors before any CUDA call."""
    lib = _lib.lib()

    def al(v):
        return (v + 255) // 256 * 256

    for world, cap, hidden, k in ((2, 24, 256, 2), (8, 64, 2048, 8), (3, 5, 8, 1)):
        o = al(256 + cap * 8 * 4)
        o = al(o + world * cap * hidden * 2)
        o = al(o + world * cap * k * 4)
        o = al(o + world * cap * k * 4)
        o = al(o + world * cap * hidden * 4)
        assert lib.blut_ep_window_bytes(world, cap, hidden, k) == o
    for bad in ((0, 8, 256, 2), (9, 8, 256, 2), (2, 0, 256, 2), (2, 8, 100, 2), (2, 8, 256, 0), (2, 8, 256, 65)):
        assert lib.blut_ep_window_bytes(*bad) == 0
    d = _lib.EpDesc()
    d.world, d.rank, d.capacity, d.hidden, d.top_k, d.dtype = 2, 2, 8, 256, 2, _lib.F16  # rank out of range
    assert lib.blut_ep_dispatch(C.byref(d), None, None, None, 0, None, None, 4, None) == _lib.BLUT_ERR_INVALID
    d.rank = 0  # windows missing
    assert lib.blut_ep_combine(C.byref(d), 0, None, None, 0, None) == _lib.BLUT_ERR_INVALID
    assert lib.blut_ep_views(C.byref(d), None, None, None, None) == _lib.BLUT_ERR_INVALID
    assert lib.blut_ep_alloc(0, C.byref(C.c_void_p())) == _lib.BLUT_ERR_INVALID


def test_layer_workspace_size_follows_the_expected_slots(monkeypatch):
    """LUTMoELayer caches blut_moe_workspace_size per call shape.  The split,
    and so the size, depends on the expected slots as well as the token
    count: a layer whose slot_fraction changes between calls at the same
    token count must ask again, not reuse the smaller size (which the
    library refuses with BLUT_ERR_WORKSPACE).  The library is stubbed: this
    checks the host bookkeeping only."""
    from block_lut_b200 import moe as M

    class FakeLib:
        def __init__(self):
            self.sizes, self.launched = [], []

        def blut_moe_workspace_size(self, ap):
            n = 1000 + 10 * ap._obj.expected_slots
            self.sizes.append(n)
            return n

        def blut_moe_forward(self, ap, ws, nbytes, stream):
            self.launched.append((ap._obj.expected_slots, nbytes))
            return _lib.BLUT_OK

    fake = FakeLib()
    got = []

    class Buf:
        def __init__(self, n):
            self.n = n

        def data_ptr(self):
            return 256

        def numel(self):
            return self.n

    def fake_workspace(device, nbytes, slot=0, stream=None):
        got.append(nbytes)
        return Buf(nbytes)

    monkeypatch.setattr(M._lib, "lib", lambda: fake)
    monkeypatch.setattr(M._lib, "stream_ptr", lambda stream=None: 0)
    monkeypatch.setattr(M, "workspace", fake_workspace)
    layer = M.LUTMoELayer.__new__(M.LUTMoELayer)
    layer.top_k, layer.slot_fraction, layer.ws_slot, layer._ws_need = 4, 1.0, 0, {}
    x2 = torch.zeros(128, 8)
    for frac, want_slots in ((1.0, 0), (0.2, 103), (1.0, 0), (0.2, 103)):
        layer.slot_fraction = frac
        a = _lib.MoEArgs()
        a.num_tokens = 128
        a.expected_slots = layer._expected_slots(128)
        assert a.expected_slots == want_slots
        layer._launch(a, x2, None)
        assert got[-1] == 1000 + 10 * want_slots
    assert fake.sizes == [1000, 2030]  # one size query per (tokens, expected slots)
    assert fake.launched == [(0, 1000), (103, 2030), (0, 1000), (103, 2030)]


def test_stream_ordered_wrappers_run_on_the_callers_stream(monkeypatch):
    """Wrappers given a stream run their body with it as torch's current
    stream (inputs converted and outputs allocated there); without one they
    run as before.  Positional and keyword stream arguments both count."""
    import contextlib
    entered = []

    @contextlib.contextmanager
    def fake_stream(s):
        entered.append(s)
        yield

    monkeypatch.setattr(torch.cuda, "stream", fake_stream)

    @_lib.stream_ordered
    def op(x, y=1, stream=None, z=0):
        return (x, y, stream, z, list(entered))

    assert op(1) == (1, 1, None, 0, [])
    assert op(1, 2, "s1") == (1, 2, "s1", 0, ["s1"])
    assert op(1, stream="s2", z=3) == (1, 1, "s2", 3, ["s1", "s2"])
    from block_lut_b200 import bitplanes, formats
    for fn in (formats.encode, formats.encode_r, formats.encode_lut_f32, formats.dequant, formats.pack_tiled,
               formats.dequant_tiled, bitplanes.pack_bitplanes, bitplanes.recover_tier):
        assert "stream" in inspect.signature(fn).parameters and hasattr(fn, "__wrapped__"), fn.__name__
