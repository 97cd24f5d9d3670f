"""The alias rules of the C ABI's batch mode (go-infer_b200/csrc/batch_alias.h),
compiled with g++ and run on the CPU.

Inside metal_begin_batch / metal_end_batch go-infer chains calls through
host slices (pkg/engine/forward.go:607-640: gate/up -> batchGate, down from
batchGate -> batchFFNDown, residual add from batchFFNDown); a later call's
input must come from the newest pending output that holds its bytes, and a
slice that straddles outputs must be written back before it is read."""
import subprocess

from _util import ROOT

SRC = r'''
#include <cstdio>
#include "batch_alias.h"
#define CHECK(c) do { if (!(c)) { std::printf("FAIL line %d\n", __LINE__); return 1; } } while (0)
int main() {
  using gi::PendingOutputs;
  using gi::Resolve;
  static char host[1000], dev1[1000], dev2[1000], dev3[1000];
  PendingOutputs p;
  const void* d = nullptr;
  CHECK(p.resolve(host, 10, &d) == Resolve::kHost && d == nullptr);
  p.add(host, 400, dev1);                                        // output [0, 400)
  CHECK(p.resolve(host + 100, 50, &d) == Resolve::kDevice && d == dev1 + 100);
  CHECK(p.resolve(host, 400, &d) == Resolve::kDevice && d == dev1);
  CHECK(p.resolve(host + 400, 8, &d) == Resolve::kHost && d == nullptr);  // adjacent: disjoint
  CHECK(p.resolve(host + 392, 16, &d) == Resolve::kFlush);       // straddles its end
  p.add(host + 100, 50, dev2);                                   // a newer output inside it
  CHECK(p.resolve(host + 100, 50, &d) == Resolve::kDevice && d == dev2);
  CHECK(p.resolve(host + 110, 10, &d) == Resolve::kDevice && d == dev2 + 10);
  CHECK(p.resolve(host, 50, &d) == Resolve::kDevice && d == dev1);        // untouched by the newer
  CHECK(p.resolve(host + 200, 100, &d) == Resolve::kDevice && d == dev1 + 200);
  CHECK(p.resolve(host + 90, 20, &d) == Resolve::kFlush);        // part newer, part older
  CHECK(p.resolve(host, 400, &d) == Resolve::kFlush);            // contains the newer one
  p.add(host, 400, dev3);                                        // newest covers everything
  CHECK(p.resolve(host + 90, 20, &d) == Resolve::kDevice && d == dev3 + 90);
  CHECK(p.list().size() == 3 && p.list()[1].dev == dev2);        // call order kept
  p.clear();
  CHECK(p.empty() && p.resolve(host, 10, &d) == Resolve::kHost);
  std::printf("ok\n");
  return 0;
}
'''


def test_batch_alias_rules(tmp_path):
    src = tmp_path / "alias.cc"
    src.write_text(SRC)
    exe = tmp_path / "alias"
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-I", f"{ROOT}/go-infer_b200/csrc", str(src), "-o",
                    str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
