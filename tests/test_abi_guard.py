"""The C ABI's exception guard (csrc/abi_guard.h), compiled on the host: a failed host
allocation becomes QASR_ERR_OOM, any other C++ exception QASR_ERR_STATE, each with its
message passed to the entry point's error slot; a body that returns passes its status
through.  No GPU."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include <cstdio>
#include <new>
#include <stdexcept>
#include <string>
#include "abi_guard.h"

static std::string last;
static qasr_status report(qasr_status s, const std::string& m) { last = m; return s; }

int main() {
  int bad = 0;
  qasr_status s = qasr::guard([] { return QASR_ERR_CAPACITY; }, report);
  bad |= (s != QASR_ERR_CAPACITY) << 0;
  s = qasr::guard([]() -> qasr_status { throw std::bad_alloc(); }, report);
  bad |= (s != QASR_ERR_OOM || last != "out of host memory") << 1;
  s = qasr::guard([]() -> qasr_status { throw std::length_error("vector"); }, report);
  bad |= (s != QASR_ERR_STATE || last != "host error: vector") << 2;
  s = qasr::guard([]() -> qasr_status { throw 7; }, report);
  bad |= (s != QASR_ERR_STATE || last != "host error") << 3;
  // a report that throws itself still yields the status
  s = qasr::guard([]() -> qasr_status { throw std::bad_alloc(); },
                  [](qasr_status, const std::string&) -> qasr_status { throw std::bad_alloc(); });
  bad |= (s != QASR_ERR_OOM) << 4;
  std::printf("%d\n", bad);
  return bad;
}
"""


def test_guard_maps_exceptions_to_status_codes(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no host C++ compiler")
    src = tmp_path / "guard.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "guard"
    subprocess.run([gxx, "-std=c++17", "-O1", "-I", str(ROOT / "qwen3-asr-wgpu_b200" / "csrc"),
                    "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout
