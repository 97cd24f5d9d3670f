"""The C ABI's host code (go-infer_b200/csrc/capi.cu) on the CPU.

capi.cu is compiled with g++ against the fake CUDA runtime of
tests/fakecuda/ (device memory kept in a registry, synchronous streams,
stand-in kernels with a predictable result), under AddressSanitizer and
UndefinedBehaviorSanitizer.  The driver runs go-infer's batch call chains
(pkg/engine/forward.go:604-642: gate, up, SwiGLU, down from the gate slice,
residual add) call by call and inside one metal_begin_batch/metal_end_batch
pair, and requires bit-identical host slices; it also checks the status codes
of the fused gate/up, residual and SwiGLU entry points, a batch larger than
the activation arena, and the no-alloc prefill against gi_cuda_gemm_dev.
A host pointer handed to a fake kernel, or a device pointer copied as host
memory, aborts the run.
"""
import os
import shutil
import subprocess

import pytest

from _util import ROOT

FAKE = os.path.join(ROOT, "tests", "fakecuda")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_batch_mode_on_fake_runtime(tmp_path):
    inc = ["-I", FAKE, "-I", os.path.join(ROOT, "go-infer_b200", "csrc"), "-I", os.path.join(ROOT, "include")]
    flags = ["-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"]
    capi = tmp_path / "capi.o"
    subprocess.run(["g++", *flags, "-x", "c++", *inc, "-c", os.path.join(ROOT, "go-infer_b200", "csrc", "capi.cu"),
                    "-o", str(capi)], check=True)
    exe = tmp_path / "batch_driver"
    subprocess.run(["g++", *flags, *inc, os.path.join(FAKE, "fake_device.cc"), os.path.join(FAKE, "batch_driver.cc"),
                    str(capi), "-o", str(exe), "-lpthread"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout[-4000:] + r.stderr[-4000:]
