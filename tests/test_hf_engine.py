"""The HF offload engine's C++ side on libblut (include/blut_hf.hpp): a C++
caller, built with g++ against libblut.so and the CUDA runtime (no torch), does
what the engine's dispatcher does for a few experts -- recover one tensor with
the drop-in ``lut_moe_launch_blocklut_recover`` and run each expert module
(``DeepSeekMoEDenseActDense`` replaced by ``blut_hf::LutExpertModule``) on a
token batch -- and writes the results to a file.

On CPU the caller only has to compile and link.  On a GPU its outputs are
checked against the oracle: the recovered tensor bit for bit, the expert
outputs within the bf16 layer tolerance of tests/_helpers.check_layer.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

from oracle import blut_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")

CALLER = r"""
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <memory>
#include "blut_hf.hpp"

// input: int32 H, I, T, E, tier; lut[256] bf16; per expert gate/up/down indices and absmax; x [T][H] bf16
// output: recovered gate_proj of expert 0 [I][H] bf16, then y [E][T][H] bf16
static void* upload(const void* h, size_t n) {
  void* d = nullptr;
  blut_hf::check_cuda(cudaMalloc(&d, n), "cudaMalloc");
  blut_hf::check_cuda(cudaMemcpy(d, h, n, cudaMemcpyHostToDevice), "upload");
  return d;
}

int main(int argc, char** argv) {
  if (argc != 3) return 2;
  FILE* f = std::fopen(argv[1], "rb");
  if (!f) return 3;
  int hdr[5];
  if (std::fread(hdr, 4, 5, f) != 5) return 4;
  const int H = hdr[0], I = hdr[1], T = hdr[2], E = hdr[3], tier = hdr[4];
  const size_t n = (size_t)I * H, nb = n / 128;
  std::vector<uint16_t> lut(256);
  if (std::fread(lut.data(), 2, 256, f) != 256) return 5;
  std::vector<std::vector<uint8_t>> idx(3 * E, std::vector<uint8_t>(n));
  std::vector<std::vector<uint16_t>> am(3 * E, std::vector<uint16_t>(nb));
  for (int i = 0; i < 3 * E; ++i) {
    if (std::fread(idx[i].data(), 1, n, f) != n) return 6;
    if (std::fread(am[i].data(), 2, nb, f) != nb) return 7;
  }
  std::vector<uint16_t> x((size_t)T * H);
  if (std::fread(x.data(), 2, x.size(), f) != x.size()) return 8;
  std::fclose(f);
  try {
    cudaStream_t s;
    blut_hf::check_cuda(cudaStreamCreate(&s), "stream");
    auto* d_lut = static_cast<uint16_t*>(upload(lut.data(), 512));
    std::vector<void*> d_idx(3 * E), d_am(3 * E);
    for (int i = 0; i < 3 * E; ++i) {
      d_idx[i] = upload(idx[i].data(), n);
      d_am[i] = upload(am[i].data(), nb * 2);
    }
    void* d_x = upload(x.data(), x.size() * 2);
    // the engine's recover of one tensor, through the drop-in launcher
    uint16_t* d_rec = nullptr;
    blut_hf::check_cuda(cudaMalloc(&d_rec, n * 2), "cudaMalloc");
    blut_hf::check(lut_moe_launch_blocklut_recover(d_rec, static_cast<uint8_t*>(d_idx[0]),
                                                   static_cast<uint16_t*>(d_am[0]), d_lut, n, s), "recover");
    // one module per expert, as the dispatcher keeps them
    std::vector<std::unique_ptr<blut_hf::LutExpertModule>> mods;
    void* d_y = nullptr;
    blut_hf::check_cuda(cudaMalloc(&d_y, (size_t)E * T * H * 2), "cudaMalloc");
    blut_hf::check_cuda(cudaMemset(d_y, 0, (size_t)E * T * H * 2), "cudaMemset");
    for (int e = 0; e < E; ++e) {
      mods.emplace_back(new blut_hf::LutExpertModule(H, I, d_lut, tier));
      blut_hf::ExpertBlob b{static_cast<uint8_t*>(d_idx[3 * e]), static_cast<uint16_t*>(d_am[3 * e]),
                            static_cast<uint8_t*>(d_idx[3 * e + 1]), static_cast<uint16_t*>(d_am[3 * e + 1]),
                            static_cast<uint8_t*>(d_idx[3 * e + 2]), static_cast<uint16_t*>(d_am[3 * e + 2])};
      mods.back()->SetTensorsFromBlob(b, s);
    }
    for (int e = 0; e < E; ++e) {
      // expert e runs on the first T - e tokens (the dispatcher's per-expert batches differ)
      mods[e]->forward(d_x, T - e, static_cast<uint16_t*>(d_y) + (size_t)e * T * H, s);
      mods[e]->check_status(s);
    }
    std::vector<uint16_t> rec(n), y((size_t)E * T * H, 0);
    blut_hf::check_cuda(cudaMemcpy(rec.data(), d_rec, n * 2, cudaMemcpyDeviceToHost), "download");
    blut_hf::check_cuda(cudaMemcpy(y.data(), d_y, y.size() * 2, cudaMemcpyDeviceToHost), "download");
    FILE* o = std::fopen(argv[2], "wb");
    if (!o) return 9;
    std::fwrite(rec.data(), 2, n, o);
    std::fwrite(y.data(), 2, y.size(), o);
    std::fclose(o);
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "error: %s\n", ex.what());
    return 10;
  }
  std::puts("hf caller ok");
  return 0;
}
"""


def _build(tmp_path):
    if shutil.which("g++") is None:
        pytest.skip("needs g++")
    from block_lut_b200 import _lib
    src = tmp_path / "hf_caller.cpp"
    src.write_text(CALLER)
    exe = tmp_path / "hf_caller"
    libdir = os.path.dirname(_lib.LIB_PATH)
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        "-I", os.path.join(CUDA, "include"), str(src), "-L", libdir, "-lblut",
                        "-Wl,-rpath," + libdir, "-L", os.path.join(CUDA, "lib64"), "-lcudart",
                        "-Wl,-rpath," + os.path.join(CUDA, "lib64"), "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_hf_engine_caller_builds(tmp_path):
    """blut_hf.hpp compiles as C++17 with warnings as errors and links libblut.so."""
    _build(tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("tier", [0, 2])
def test_hf_engine_expert_modules_match_oracle(tmp_path, tier):
    exe = _build(tmp_path)
    H, I, T, E = 2048, 1408, 12, 3  # Qwen1.5-MoE / DeepSeek-V2-Lite expert shapes
    rng = np.random.Generator(np.random.PCG64(90 + tier))
    lut = O.f32_to_bf16(np.sort(rng.uniform(-1, 1, 256)).astype(np.float32))
    n = I * H
    mats = []
    for _ in range(3 * E):
        mats.append((rng.integers(0, 256, n, dtype=np.uint8),
                     O.f32_to_bf16(rng.uniform(0.01, 0.05, n // 128).astype(np.float32))))
    x = O.f32_to_bf16(O.rms_activations(rng, T, H).astype(np.float32))
    inp = tmp_path / "in.bin"
    with open(inp, "wb") as f:
        f.write(np.array([H, I, T, E, tier], dtype=np.int32).tobytes())
        f.write(lut.tobytes())
        for idx, am in mats:
            f.write(idx.tobytes())
            f.write(am.tobytes())
        f.write(x.tobytes())
    out = tmp_path / "out.bin"
    r = subprocess.run([str(exe), str(inp), str(out)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "hf caller ok" in r.stdout, (r.returncode, r.stdout, r.stderr)
    res = np.fromfile(out, dtype=np.uint16)
    rec, y = res[:n], res[n:].reshape(E, T, H)
    # the recover drop-in reads all 8 index bits (the engine masks tiers before it)
    assert np.array_equal(rec, O.dequant_r(mats[0][0], mats[0][1], lut, 128, 0))
    xf = O.bf16_to_f32(x).reshape(T, H).astype(np.float64)
    from tests._helpers import MAX_ABS, REL_L2
    for e in range(E):
        g, u, d = (O.bf16_to_f32(O.dequant_r(idx, am, lut, 128, tier)).astype(np.float64) for idx, am in
                   mats[3 * e:3 * e + 3])
        t = T - e
        h1, h3 = xf[:t] @ g.reshape(I, H).T, xf[:t] @ u.reshape(I, H).T
        a = O.round_to((O.silu(h1) * h3).astype(np.float32), "bf16").astype(np.float64)
        ref = a @ d.reshape(H, I).T
        got = O.bf16_to_f32(y[e, :t]).astype(np.float64)
        rb = O.round_to(ref.astype(np.float32), "bf16").astype(np.float64)
        ulp = np.exp2(np.floor(np.log2(np.maximum(np.abs(rb), 1e-30))) - 7)
        assert (np.abs(got - rb) <= np.maximum(ulp, MAX_ABS)).all(), f"expert {e}"
        assert O.rel_l2(got, rb) <= REL_L2, f"expert {e}"
        assert not y[e, t:].any()  # rows past the expert's batch are untouched
