"""CPU checks of the C ABI: the library builds, loads without a GPU driver and
exports every symbol the public header declares; the product package never
imports the oracle."""

import ast
import os
import subprocess

import pytest

from tests.conftest import ROOT


@pytest.fixture(scope="module")
def lib():
    from lastkv_b200 import _capi, build

    build.build()
    return _capi.load()


def test_header_symbols_are_exported(lib):
    from lastkv_b200 import _capi

    declared = _capi.declared_symbols()
    assert "lkv_decode_paged" in declared and "lkv_rope_norm_append" in declared
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/lastkv_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", _capi.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T lkv_" in line}
    assert exported == set(declared), exported ^ set(declared)


def test_library_has_no_driver_link():
    from lastkv_b200 import _capi

    out = subprocess.run(["readelf", "-d", _capi.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out and "libcudart.so" not in out


def test_host_only_entry_points(lib):
    assert lib.lkv_abi_version() >= 100
    assert lib.lkv_status_string(0) == b"ok"
    assert lib.lkv_status_string(6).startswith(b"workspace")
    small = lib.lkv_decode_workspace_bytes(1, 4, 128, 1)
    big = lib.lkv_decode_workspace_bytes(64, 32, 128, 512)
    assert 256 < small < big
    # context-parallel state: epoch, done counter, one arrival counter per (sequence, KV head)
    import ctypes

    words = ctypes.c_int64(0)
    assert lib.lkv_decode_cp_state_words(4, 8, ctypes.byref(words)) == 0 and words.value == 2 + 32
    assert lib.lkv_decode_cp_state_words(0, 8, ctypes.byref(words)) == 1
    send, recv = ctypes.c_int64(0), ctypes.c_int64(0)
    assert lib.lkv_cp_combine_sizes(128, 128, 8, ctypes.byref(send), ctypes.byref(recv)) == 0
    assert recv.value == 2 * 8 * (128 * 129)  # two epoch slots x ranks x {value, epoch} words per float


def test_argument_validation_needs_no_gpu(lib):
    # unsupported head_dim / GQA group are rejected before any CUDA call
    st = lib.lkv_decode_paged(None, 0, None, None, 1, None, 0, None, None, 0, None, None, None, None,
                              1, 4, 1, 96, 1, 1.0, None, 0, 0, None)
    assert st == 2
    st = lib.lkv_decode_paged(None, 0, None, None, 1, None, 0, None, None, 0, None, None, None, None,
                              1, 12, 1, 128, 1, 1.0, None, 0, 0, None)
    assert st == 2
    assert lib.lkv_decode_paged(None, 0, None, None, 1, None, 0, None, None, 0, None, None, None, None,
                                1, 8, 3, 128, 1, 1.0, None, 0, 0, None) == 1
    # empty batch is a no-op
    assert lib.lkv_decode_paged(None, 0, None, None, 1, None, 0, None, None, 0, None, None, None, None,
                                0, 8, 8, 128, 1, 1.0, None, 0, 0, None) == 0
    # the fused context-parallel decode needs its peers and state: rejected before any CUDA call
    assert lib.lkv_decode_paged_cp(None, 0, None, None, 1, None, 0, None, None, 0, None, 2, 8, 8, 128, 1, 1.0,
                                   None, 0, None, 0, 2, None, None, 0, None) == 1
    # the key-split prefill validates its shape first (head_dim 96 is unsupported)
    assert lib.lkv_prefill_paged_split(None, 0, None, None, 1, None, 0, None, None, None, 0, None, None,
                                       1, 1, 1, 8, 8, 96, 1, 1.0, 2, None, None, None, None) == 2


def test_append_commit_validation_needs_no_gpu(lib):
    def call(T=0, hq=8, hkv=8, d=128, flags=0, layers=0, rows=0, ppc=0, blocks=0):
        return lib.lkv_rope_norm_append_commit(
            None, 0, None, 0, None, 0, None, None, 0, 0, None, None, 1e-6, None, None, 0, None, None, None, 0,
            None, None, None, 0, T, hq, hkv, d, flags,
            None, None, 0, None, None, 0, None, layers, rows, ppc, None, blocks, None, None)

    assert call(d=96) == 2                       # head_dim 64 or 128 only
    assert call(flags=4) == 2                    # fp32 pools: append, then lkv_blend_chunk_f32
    assert call(blocks=-1) == 1                  # negative commit block count
    assert call(layers=2, rows=1, ppc=4) == 1    # a commit without its pools and page lists
    assert call() == 0                           # no tokens and no commit: nothing to launch


def test_product_package_never_imports_oracle():
    pkg = os.path.join(ROOT, "lastkv_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if not f.endswith(".py"):
                continue
            tree = ast.parse(open(os.path.join(dirpath, f)).read())
            for node in ast.walk(tree):
                names = []
                if isinstance(node, ast.Import):
                    names = [a.name for a in node.names]
                elif isinstance(node, ast.ImportFrom):
                    names = [node.module or ""]
                assert not any(n.split(".")[0] == "oracle" for n in names), f"{f} imports the oracle"


def test_ops_fail_loudly_without_library(tmp_path, monkeypatch):
    from lastkv_b200 import _capi
    from lastkv_b200.contract import RMarinBackendContractError

    monkeypatch.setattr(_capi, "_lib", None)
    with pytest.raises(RMarinBackendContractError, match="not built"):
        _capi.load(str(tmp_path / "missing.so"))


def test_binding_arities_match_the_header():
    """Every ctypes signature in ``_capi._SIGNATURES`` passes exactly as many arguments as
    the function's declaration in include/lastkv_b200.h, and every declared function is
    bound (the header is the ABI; the bindings are what a caller copies)."""
    import re

    from lastkv_b200 import _capi

    text = re.sub(r"/\*.*?\*/", "", open(_capi.HEADER).read(), flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(lkv_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        params = m.group(2).strip()
        decls[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    assert set(decls) == set(_capi.declared_symbols())
    assert set(decls) == set(_capi._SIGNATURES), set(decls) ^ set(_capi._SIGNATURES)
    for name, n in decls.items():
        assert len(_capi._SIGNATURES[name][1]) == n, (name, n, len(_capi._SIGNATURES[name][1]))


def test_nvtx_ranges_are_opt_in():
    """LKV_NVTX=1 wraps every kernel-launching op in an NVTX range; without it the ops are
    the plain functions (no per-call range overhead)."""
    import subprocess
    import sys

    code = ("import lastkv_b200.ops as o; "
            "names = ['decode_paged', 'prefill_paged', 'rope_norm_append', 'decode_gemm', 'decode_paged_cp']; "
            "print(sum(hasattr(getattr(o, n), '__wrapped__') for n in names))")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=root)
    env.pop("LKV_NVTX", None)
    off = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, cwd=root)
    on = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=dict(env, LKV_NVTX="1"),
                        cwd=root)
    assert off.stdout.strip() == "0", off.stderr
    assert on.stdout.strip() == "5", on.stderr
