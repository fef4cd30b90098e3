"""The invariant-divisor division the kernels index with (csrc/fastdiv.h), checked on the host:
exhaustive over small numerators and every edge for a spread of divisors."""

import os
import subprocess
import textwrap

from conftest import ROOT

SRC = textwrap.dedent("""
    #include <cstdio>
    #include <cstdint>
    #include "fastdiv.h"
    int main() {
      const uint32_t divs[] = {1u, 2u, 3u, 5u, 6u, 7u, 8u, 32u, 64u, 96u, 100u, 128u, 255u, 256u,
                               512u, 1120u, 4096u, 8960u, 65535u, 65536u, 1000003u, 0x7fffffffu,
                               0x80000000u, 0xfffffffeu, 0xffffffffu};
      long bad = 0;
      for (uint32_t d : divs) {
        tb::FastDiv f(d);
        for (uint32_t n = 0; n < 300000u; ++n) bad += f.div(n) != n / d;
        const uint32_t edges[] = {d - 1u, d, d + 1u, 2u * d - 1u, 0x7fffffffu, 0x80000000u,
                                  0xfffffffeu, 0xffffffffu, 0xffffffffu - d};
        for (uint32_t n : edges) bad += f.div(n) != n / d;
        for (uint64_t n = 0; n <= 0xffffffffull; n += 2654435761ull % 1000003ull)
          bad += f.div((uint32_t)n) != (uint32_t)n / d;
        uint32_t q, r;
        f.divmod(123456789u, q, r);
        bad += (q != 123456789u / d) || (r != 123456789u % d);
      }
      printf("%ld\\n", bad);
      return bad != 0;
    }
""")


def test_fastdiv_is_exact(tmp_path):
    src = tmp_path / "fd.cpp"
    src.write_text(SRC)
    exe = tmp_path / "fd"
    inc = os.path.join(ROOT, "testt_b200", "csrc")
    subprocess.run(["g++", "-O2", "-std=c++17", "-I" + inc, str(src), "-o", str(exe)], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0 and res.stdout.strip() == "0", res.stdout
