"""Host checks of the Rust backend crate rust/opencuda-cuda (no Rust toolchain
in this image, so it is not compiled here): every `extern "C"` function its
ffi.rs declares exists in include/opencuda_cuda.h with the same number of
arguments and is exported by the built library; the kernel names the crate
documents as routed are the names oc_device_launch accepts; the opencuda-blas
patch is a well-formed unified diff that adds the CuBlas arm, the explicit
transpose_b argument and the weight-only matmuls."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CRATE = os.path.join(ROOT, "rust", "opencuda-cuda")
HEADER = os.path.join(ROOT, "include", "opencuda_cuda.h")


def _arity(params: str) -> int:
    params = params.strip()
    if params in ("", "void"):
        return 0
    depth, n = 0, 1
    for ch in params:
        if ch in "([":
            depth += 1
        elif ch in ")]":
            depth -= 1
        elif ch == "," and depth == 0:
            n += 1
    return n


def header_prototypes() -> dict:
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(oc_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        out[m.group(1)] = _arity(m.group(2))
    return out


def rust_externs() -> dict:
    text = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    block = text[text.index('extern "C" {'):]
    out = {}
    for m in re.finditer(r"pub fn (oc_[a-z0-9_]+)\s*\((.*?)\)\s*(?:->\s*[^;]+)?;", block, flags=re.S):
        params = re.sub(r"//.*", "", m.group(2)).strip().rstrip(",")
        out[m.group(1)] = _arity(params)
    return out


def test_ffi_matches_header():
    h, r = header_prototypes(), rust_externs()
    assert len(r) >= 30
    missing = sorted(set(r) - set(h))
    assert not missing, f"ffi.rs declares functions the header does not: {missing}"
    wrong = {k: (r[k], h[k]) for k in r if r[k] != h[k]}
    assert not wrong, f"argument counts differ (rust, header): {wrong}"


def test_ffi_symbols_exported():
    lib = os.path.join(ROOT, "open-cuda_b200", "libopencuda_cuda.so")
    if not os.path.exists(lib):
        pytest.skip("library not built")
    import ctypes
    L = ctypes.CDLL(lib)
    for name in rust_externs():
        assert hasattr(L, name), name


def test_routed_kernel_names_match_the_launcher():
    src = open(os.path.join(ROOT, "open-cuda_b200", "csrc", "oc_blas_dense_host.cu")).read()
    routed = set(re.findall(r'kname == "([a-z_0-9]+)"', src))
    doc = open(os.path.join(CRATE, "src", "lib.rs")).read()
    listed = set(re.findall(r"`([a-z_0-9]+)`", doc[doc.index("routes by kernel name"):doc.index("other names fail")]))
    assert listed == routed, (listed, routed)


def test_constants_match_header():
    text = open(HEADER).read()
    ffi = open(os.path.join(CRATE, "src", "ffi.rs")).read()
    for name, val in re.findall(r"#define (OC_[A-Z_]+) (\d+)", text):
        m = re.search(rf"pub const {name}: c_int = (\d+);", ffi)
        assert m and int(m.group(1)) == int(val), name
    for name, val in re.findall(r"(OC_ARG_[A-Z]+) = (\d+)", text):
        m = re.search(rf"pub const {name}: c_int = (\d+);", ffi)
        assert m and int(m.group(1)) == int(val), name


def _hunks(path):
    lines = open(path).read().splitlines()
    assert lines[0].startswith("--- a/") and lines[1].startswith("+++ b/")
    hunks, i = [], 2
    while i < len(lines):
        m = re.match(r"@@ -(\d+),(\d+) \+(\d+),(\d+) @@", lines[i])
        assert m, lines[i]
        old_n, new_n = int(m.group(2)), int(m.group(4))
        i += 1
        body = []
        while i < len(lines) and not lines[i].startswith("@@"):
            body.append(lines[i])
            i += 1
        assert sum(1 for b in body if b[:1] in (" ", "-")) == old_n
        assert sum(1 for b in body if b[:1] in (" ", "+")) == new_n
        hunks.append(body)
    return hunks


def test_blas_patch_is_well_formed():
    hunks = _hunks(os.path.join(ROOT, "rust", "patches", "opencuda-blas-cuda.patch"))
    added = "\n".join(b[1:] for h in hunks for b in h if b.startswith("+"))
    assert "KernelArg::U32(transpose_b as u32)" in added
    assert "GemmPath::CuBlas => launch_naive_gemm(" in added
    assert "pub fn qgemm_w8(" in added and "pub fn qgemm_w4(" in added
    assert '"qgemm_w8"' in added and '"qgemm_w4"' in added
    _hunks(os.path.join(ROOT, "rust", "patches", "workspace-members.patch"))
