"""The kernel decodes work items with a multiply and shift instead of integer
division (DivMagic in csrc/afa_fwd_kernel.cuh).  This compiles the header's
DivMagic into a small host program and checks floor(x / d) for divisors from 1
to 2^31 - 1 against the numerators where a wrong multiplier would show first:
0..2^16, the top of the range, multiples of d and their neighbours, and random
values.  Runs on the CPU (nvcc only compiles; no GPU is used)."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CSRC = ROOT / "ampere_flash_attention_from_scratch_b200" / "csrc"

PROGRAM = r"""
#include <cstdio>
#include <cstdint>
#include <random>
#include "afa_fwd_kernel.cuh"
int main() {
  std::mt19937_64 rng(7);
  long long bad = 0, n = 0;
  auto check = [&](int d, uint32_t x, const afa100::DivMagic& m) {
    const uint32_t q = static_cast<uint32_t>((static_cast<unsigned long long>(x) * m.mul) >> m.shift);
    ++n;
    if (q != x / static_cast<uint32_t>(d)) ++bad;
  };
  const int ds[] = {1, 2, 3, 5, 7, 31, 32, 33, 100, 127, 128, 1000, 4095, 65535, 65536, 1000003,
                    (1 << 30) + 1, 2147483647};
  for (int d : ds) {
    const afa100::DivMagic m = afa100::DivMagic::make(d);
    for (uint32_t x = 0; x <= 65536u; ++x) check(d, x, m);
    for (uint32_t x = 0x7FFFFFFFu - 65536u; x <= 0x7FFFFFFFu; ++x) check(d, x, m);
    for (uint32_t k = 1; k < 65536u; ++k) {
      const unsigned long long x = static_cast<unsigned long long>(k) * static_cast<unsigned>(d);
      if (x >= 0x80000000ull) break;
      check(d, static_cast<uint32_t>(x), m);
      check(d, static_cast<uint32_t>(x - 1), m);
    }
    for (int i = 0; i < 200000; ++i) check(d, static_cast<uint32_t>(rng() & 0x7FFFFFFFu), m);
  }
  for (int d = 1; d <= 4096; ++d) {
    const afa100::DivMagic m = afa100::DivMagic::make(d);
    for (int i = 0; i < 256; ++i) check(d, static_cast<uint32_t>(rng() & 0x7FFFFFFFu), m);
  }
  std::printf("%lld %lld\n", n, bad);
  return bad != 0;
}
"""


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not installed")
def test_div_magic_matches_integer_division(tmp_path):
    src = tmp_path / "div_magic.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "div_magic"
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2", f"-I{CSRC}",
                    "-o", str(exe), str(src)], check=True, capture_output=True, timeout=600)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    checks, wrong = map(int, out.stdout.split())
    assert checks > 5_000_000 and wrong == 0 and out.returncode == 0
