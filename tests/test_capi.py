"""The C-ABI library without a GPU: it loads, exports exactly what
include/goinfer_cuda.h declares, and answers with the status codes of the
metal_bridge convention when no device is bound."""
import ctypes
import os
import re

import numpy as np
import pytest

import goinfer_cuda as G
from _util import ROOT

HEADER = os.path.join(ROOT, "include", "goinfer_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(gi_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = G.load_library()
    names = declared_functions()
    assert names == set(G.EXPORTS)
    for n in names:
        assert hasattr(lib, n), n


def test_header_compiles_as_c():
    import subprocess, tempfile
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "t.c")
        open(src, "w").write('#include "goinfer_cuda.h"\nint main(void){return GI_TYPE_Q4_K == 12 ? 0 : 1;}\n')
        subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), src,
                        "-o", os.path.join(d, "t")], check=True)


def test_c_program_links_and_calls_the_library(tmp_path):
    """What cgo does with INTEGRATION.md's preamble: compile C against the
    header, link libgoinfer_cuda.so, call entry points that answer without
    a device (row sizes of pkg/math/gemv.go, the nil handle of
    metal.CreateBuffer before Init)."""
    import subprocess
    src = tmp_path / "use.c"
    src.write_text(
        '#include <stdio.h>\n#include "goinfer_cuda.h"\n'
        "int main(void) {\n"
        "  if (gi_quant_row_bytes(GI_TYPE_Q4_K, 4096) != 16 * 144) return 2;\n"
        "  if (gi_quant_row_bytes(GI_TYPE_Q6_K, 11008) != 43 * 210) return 3;\n"
        "  if (gi_quant_row_bytes(GI_TYPE_Q8_0, 4096) != 128 * 34) return 4;\n"
        "  if (gi_quant_row_bytes(3, 4096) != -1) return 5;\n"
        "  if (gi_cuda_is_available()) return 0;  /* bound elsewhere: nothing more to check */\n"
        "  unsigned char w[16] = {0};\n"
        "  if (gi_cuda_create_buffer(w, sizeof w) != NULL) return 6;\n"
        "  printf(\"%s\\n\", gi_cuda_last_error());\n"
        "  return 0;\n}\n")
    lib_dir = os.path.dirname(G.LIB_PATH)
    exe = tmp_path / "use"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe),
                    "-L", lib_dir, "-lgoinfer_cuda", "-Wl,-rpath," + lib_dir], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)


GO_BINDING = os.path.join(ROOT, "bindings", "go", "pkg", "cuda")


def go_sources():
    """The committed cgo binding (cuda_linux.go) and its stubs (cuda_fallback.go)."""
    return {f: open(os.path.join(GO_BINDING, f)).read() for f in ("cuda_linux.go", "cuda_fallback.go")}


def test_go_binding_names_declared_functions():
    """Every C function and type the cgo binding uses is declared in the header."""
    text = open(HEADER).read()
    src = go_sources()["cuda_linux.go"]
    used = set(re.findall(r"\bC\.(gi_\w+)", src))
    assert used
    for name in used:
        assert re.search(r"\b" + name + r"\b", text), name


def test_go_fallback_covers_the_binding():
    """cuda_fallback.go defines every exported package-level function of
    cuda_linux.go with the same parameters (metal_fallback.go's role)."""
    def funcs(src):
        return {m.group(1): re.sub(r"\s+", " ", m.group(2)) for m in
                re.finditer(r"^func ([A-Z]\w*)\(([^)]*)\)", src, flags=re.M)}
    srcs = go_sources()
    linux, stub = funcs(srcs["cuda_linux.go"]), funcs(srcs["cuda_fallback.go"])
    missing = {n for n in linux if n not in stub and n not in ("AllocBuffers", "ForwardTransformer", "NewModel")}
    assert not missing, missing
    for n, params in stub.items():
        assert linux.get(n) == params, (n, params, linux.get(n))
    assert "//go:build linux && cgo && cuda" in srcs["cuda_linux.go"]
    assert "//go:build !linux || !cgo || !cuda" in srcs["cuda_fallback.go"]


def _split_args(text, start):
    """Top-level comma-separated arguments of the call whose '(' is at start."""
    depth, args, cur = 0, [], ""
    for ch in text[start:]:
        if ch in "([{":
            depth += 1
            if depth == 1:
                continue
        elif ch in ")]}":
            depth -= 1
            if depth == 0:
                args.append(cur)
                break
        if depth == 1 and ch == ",":
            args.append(cur)
            cur = ""
        elif depth >= 1:
            cur += ch
    return [a for a in (x.strip() for x in args) if a]


def test_go_binding_argument_counts():
    """Each C.gi_*(...) call in the cgo binding passes as many arguments as
    include/goinfer_cuda.h declares."""
    header = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    decl = {}
    for m in re.finditer(r"\b(gi_\w+)\s*\(", header):
        params = _split_args(header, m.end() - 1)
        decl[m.group(1)] = 0 if params == ["void"] else len(params)
    src = go_sources()["cuda_linux.go"]
    checked = 0
    for m in re.finditer(r"\bC\.(gi_\w+)\(", src):
        name = m.group(1)
        if name not in decl:
            continue  # a type conversion such as C.gi_cuda_buffer_t(x)
        n = len(_split_args(src, m.end() - 1))
        assert n == decl[name], f"{name}: {n} arguments in cuda_linux.go, {decl[name]} declared"
        checked += 1
    assert checked >= 20


def test_row_bytes_follow_gemv_go():
    # pkg/math/gemv.go:99,135,171
    assert G.row_bytes(G.TYPE_Q8_0, 4096) == 128 * 34
    assert G.row_bytes(G.TYPE_Q4_K, 4096) == 16 * 144
    assert G.row_bytes(G.TYPE_Q6_K, 11008) == 43 * 210
    assert G.row_bytes(3, 4096) == -1


@pytest.mark.skipif(os.path.exists("/dev/nvidia0"), reason="a GPU is present")
def test_no_device_status_codes():
    lib = G.load_library()
    assert lib.gi_cuda_init() == G.ERR_UNAVAILABLE
    assert not G.IsAvailable()
    y = np.zeros(16, np.float32)
    x = np.zeros(256, np.float32)
    raw = np.zeros(16 * 144, np.uint8)
    rc = lib.gi_cuda_gemv_q4_k(y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                               x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                               ctypes.c_void_p(raw.ctypes.data), 16, 256)
    assert rc == G.ERR_UNAVAILABLE
    assert G.CreateBuffer(raw) is None  # nil handle, as metal.CreateBuffer
    assert lib.gi_cuda_gemm_fused_gate_up_buf(G.TYPE_Q4_K, y.ctypes.data, x.ctypes.data, None, None, 1, 16,
                                              256) == G.ERR_UNAVAILABLE
    assert lib.gi_cuda_add_residual(y.ctypes.data, y.ctypes.data, 16) == G.ERR_UNAVAILABLE
    assert lib.gi_cuda_swiglu(y.ctypes.data, y.ctypes.data, 16) == G.ERR_UNAVAILABLE
    with pytest.raises(G.GoInferCudaError) as e:
        G.MatMulQ4_K(y, x, raw, 16, 256)
    assert e.value.code == G.ERR_UNAVAILABLE
    assert "init" in lib.gi_cuda_last_error().decode()


def test_weights_mirror_batch_fallbacks(monkeypatch):
    """weights.go's MatMulBatch / MatMulFusedGateUpBatch report false (the
    engine then loops per token, or runs gate, up and SwiGLU apart) for an
    unknown tensor, mismatched gate/up types or a failing call (library
    calls stubbed: no device)."""
    calls = []

    def fake_batch(qt, y, x, buf, batch, rows, cols):
        calls.append(("batch", qt, buf, batch, rows, cols))
        if qt == G.TYPE_Q8_0:
            raise G.GoInferCudaError("gi_cuda_gemm_buf", G.ERR_SHAPE)

    def fake_fused(qt, y, x, gb, ub, batch, rows, cols):
        calls.append(("fused", qt, gb, ub, batch, rows, cols))
        if qt != G.TYPE_Q4_K:
            raise G.GoInferCudaError("gi_cuda_gemm_fused_gate_up_buf", G.ERR_UNSUPPORTED_TYPE)

    monkeypatch.setattr(G, "MatMulBatchBuf", fake_batch)
    monkeypatch.setattr(G, "MatMulFusedGateUpBatchBuf", fake_fused)
    w = G.Weights()
    w.meta = {"g": (G.TYPE_Q4_K, 8, 256), "u": (G.TYPE_Q4_K, 8, 256), "u6": (G.TYPE_Q6_K, 8, 256),
              "q8": (G.TYPE_Q8_0, 8, 256), "g6": (G.TYPE_Q6_K, 8, 256)}
    w.bufs = {k: f"buf-{k}" for k in w.meta}
    y, x = np.zeros(16), np.zeros(512)
    assert w.MatMulBatch(y, x, "g", 2, 8, 256) and calls[-1] == ("batch", G.TYPE_Q4_K, "buf-g", 2, 8, 256)
    assert not w.MatMulBatch(y, x, "q8", 2, 8, 256)          # the call failed
    assert not w.MatMulBatch(y, x, "missing", 2, 8, 256)
    n = len(calls)
    assert not w.MatMulFusedGateUpBatch(y, x, "g", "u6", 2, 8, 256) and len(calls) == n  # types differ: no call
    assert w.MatMulFusedGateUpBatch(y, x, "g", "u", 2, 8, 256)
    assert calls[-1] == ("fused", G.TYPE_Q4_K, "buf-g", "buf-u", 2, 8, 256)
    assert not w.MatMulFusedGateUpBatch(y, x, "g6", "u6", 2, 8, 256)  # Q6_K: -2, as the reference
