"""The multiply-high division the prefill kernel uses to decode its work items (FastDiv in
warpforth_b200/csrc/wfattn_internal.h), checked on the host against plain division for the
divisors the launcher builds (group * B * H, group, the last group's size, H) and the extremes
of 32-bit numerators.  The device form is the same expression with __umulhi."""

from __future__ import annotations

import shutil
import subprocess

import pytest

from conftest import ROOT

SRC = r"""
#include <cstdint>
#include <cstdio>
#include <random>
#include "wfattn_internal.h"
using namespace wfattn;
static uint32_t umulhi(uint32_t a, uint32_t b) { return (uint32_t)(((uint64_t)a * b) >> 32); }
int main() {
  std::mt19937_64 rng(7);
  const uint32_t ds[] = {1, 2, 3, 5, 6, 7, 8, 12, 25, 48, 96, 136, 272, 768, 1088, 6144,
                         65535, 65536, 100000007u, 0x7fffffffu};
  long bad = 0;
  for (uint32_t d : ds) {
    const FastDiv f = make_fastdiv(d);
    for (int i = 0; i < 200000; ++i) {
      const uint32_t n = i < 1000 ? (uint32_t)i
                         : i < 2000 ? 0xffffffffu - (uint32_t)(i - 1000) : (uint32_t)rng();
      const uint32_t q = (uint32_t)(((uint64_t)umulhi(n, f.m) + n) >> f.s);
      if (q != n / d) ++bad;
    }
  }
  printf("%ld\n", bad);
  return bad != 0;
}
"""


def test_fast_division_matches_integer_division(tmp_path):
    if shutil.which("g++") is None:
        pytest.skip("no C++ compiler")
    src = tmp_path / "fd.cpp"
    src.write_text(SRC)
    exe = tmp_path / "fd"
    res = subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(ROOT / "warpforth_b200" / "csrc"),
                          "-I", "/usr/local/cuda/include", str(src), "-o", str(exe)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "0", run.stdout
