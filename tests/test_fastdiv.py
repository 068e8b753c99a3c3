"""The multiply-shift division the kernel's schedule decode uses
(``csrc/fastdiv.h``), compiled with g++ and checked against ``/``.

Divisors cover every value the launcher passes (units per row, tiles per
segment, query chunks, page size, group count): all of 1..4096, powers of two
and their neighbours up to 2^31 - 1, and seeded random ones; numerators cover
0, the multiples of d and their neighbours, and 2^32 - 1.
"""
import os
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(REPO, "paged-attention-triton_b200", "csrc")

PROGRAM = r"""
#include <stdio.h>
#include <stdint.h>
#include "fastdiv.h"

static uint64_t state = 0x9E3779B97F4A7C15ull;
static uint32_t next_u32() {   // xorshift64*
  state ^= state >> 12; state ^= state << 25; state ^= state >> 27;
  return static_cast<uint32_t>((state * 0x2545F4914F6CDD1Dull) >> 32);
}

static int check(uint32_t d, uint32_t n) {
  const pa::FastDiv f = pa::make_fastdiv(d);
  if (pa::fast_div(n, f) != n / d) {
    printf("FAIL d=%u n=%u got=%u want=%u\n", d, n, pa::fast_div(n, f), n / d);
    return 1;
  }
  return 0;
}

static int check_divisor(uint32_t d) {
  int bad = 0;
  const uint32_t fixed[] = {0u, 1u, 2u, 0x7fffffffu, 0x80000000u, 0xfffffffeu, 0xffffffffu};
  for (uint32_t n : fixed) bad += check(d, n);
  for (uint32_t k = 1; k < 64; ++k) {
    const uint64_t m = static_cast<uint64_t>(d) * k;
    if (m > 0xffffffffull) break;
    bad += check(d, static_cast<uint32_t>(m));
    bad += check(d, static_cast<uint32_t>(m - 1));
    if (m < 0xffffffffull) bad += check(d, static_cast<uint32_t>(m + 1));
  }
  const uint64_t top = (0xffffffffull / d) * d;
  bad += check(d, static_cast<uint32_t>(top));
  bad += check(d, static_cast<uint32_t>(top - 1));
  for (int i = 0; i < 64; ++i) bad += check(d, next_u32());
  for (int i = 0; i < 64; ++i) bad += check(d, next_u32() % (d * 70u + 1u));
  return bad;
}

int main() {
  int bad = 0;
  long tested = 0;
  for (uint32_t d = 1; d <= 4096; ++d, ++tested) bad += check_divisor(d);
  for (int e = 12; e < 31; ++e)
    for (int delta = -2; delta <= 2; ++delta, ++tested)
      bad += check_divisor(static_cast<uint32_t>((1u << e) + delta));
  bad += check_divisor(0x7fffffffu);
  for (int i = 0; i < 4000; ++i, ++tested) bad += check_divisor(1u + next_u32() % 0x7ffffffeu);
  // a zero divisor is clamped to 1
  const pa::FastDiv z = pa::make_fastdiv(0);
  if (z.d != 1 || pa::fast_div(12345u, z) != 12345u) { printf("FAIL zero divisor\n"); ++bad; }
  printf("divisors %ld failures %d\n", tested, bad);
  return bad != 0;
}
"""


def test_fast_div_matches_integer_division(tmp_path):
    src = tmp_path / "fd.cpp"
    exe = tmp_path / "fd"
    src.write_text(PROGRAM)
    r = subprocess.run(["g++", "-O2", "-std=c++17", f"-I{HEADER_DIR}", str(src), "-o", str(exe)],
                       capture_output=True, text=True)
    if r.returncode != 0:
        pytest.fail(f"g++ failed:\n{r.stderr}")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout[-2000:]
    assert "failures 0" in r.stdout
