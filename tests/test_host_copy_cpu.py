"""The streaming-store copy the host PCM gather uses (csrc/host_copy.h) against memcpy:
every destination / source misalignment 0..15, lengths around the 16-byte head and the
64-byte loop edges and large clips, and the bytes just outside each copied range left
untouched. Compiled with the host compiler and run on the CPU."""
import subprocess
from pathlib import Path

import pytest

CSRC = Path(__file__).resolve().parents[1] / "voice-detect.cpp_b200" / "csrc"

HARNESS = r"""
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>
#include "host_copy.h"
int main() {
    std::mt19937 rng(7);
    const size_t cap = (1u << 20) + 256;
    std::vector<unsigned char> src(cap), dst(cap), want(cap);
    for (auto& c : src) c = (unsigned char)rng();
    std::vector<size_t> lens = {0, 1, 15, 16, 17, 31, 63, 64, 65, 79, 80, 127, 128, 129,
                                1000, 4096, 4099, 700 * 1024 + 3, (1u << 20)};
    long checks = 0;
    for (size_t n : lens)
        for (size_t od = 0; od < 16; ++od)
            for (size_t os = 0; os < 16; os += 3) {
                if (od + n + 64 > cap || os + n > cap) continue;
                for (size_t i = 0; i < cap; ++i) dst[i] = want[i] = (unsigned char)(i * 31 + 7);
                vdb_stream_copy(dst.data() + od + 32, src.data() + os, n);
                vdb_stream_fence();
                std::memcpy(want.data() + od + 32, src.data() + os, n);
                if (std::memcmp(dst.data(), want.data(), cap) != 0) {
                    std::printf("mismatch n=%zu od=%zu os=%zu\n", n, od, os);
                    return 1;
                }
                ++checks;
            }
    std::printf("ok %ld\n", checks);
    return 0;
}
"""


def test_stream_copy_matches_memcpy(tmp_path):
    src = tmp_path / "t.cpp"
    exe = tmp_path / "t"
    src.write_text(HARNESS)
    try:
        subprocess.run(["g++", "-O2", "-std=c++17", f"-I{CSRC}", str(src), "-o", str(exe)],
                       check=True, capture_output=True, text=True)
    except FileNotFoundError:
        pytest.skip("no host C++ compiler")
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.startswith("ok ")
