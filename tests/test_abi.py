"""The C-ABI library: loads, exports every declared symbol, validates arguments.

CPU-only: nothing here launches a kernel (every call below fails validation
or has zero rows, which returns before any CUDA call).
"""

from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import REPO
from flash_head import _lib

HEADER = os.path.join(REPO, "include", "flashhead.h")


def declared_functions() -> list[str]:
    text = open(HEADER).read()
    return re.findall(r"FH_API\s+[\w\s\*]+?\b(fh_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    from importlib import util
    build = util.spec_from_file_location("fh_build", os.path.join(REPO, "flash-head_b200", "build.py"))
    mod = util.module_from_spec(build)
    build.loader.exec_module(mod)
    mod.build()
    return _lib.load_library()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r"\bT (fh_\w+)", out))
    assert exported == set(names), exported.symmetric_difference(names)


def test_desc_layout_matches_the_header(tmp_path):
    """ctypes' fh_head_desc has the C compiler's size and field offsets."""
    fields = [f for f, _ in _lib.HeadDesc._fields_]
    src = tmp_path / "layout.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "flashhead.h"\n'
                   "int main(void){printf(\"%zu\\n\", sizeof(fh_head_desc));\n"
                   + "".join(f'printf("%zu\\n", offsetof(fh_head_desc, {f}));\n' for f in fields)
                   + "return 0;}\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(_lib.HeadDesc)
    for f, off in zip(fields, vals[1:]):
        assert getattr(_lib.HeadDesc, f).offset == off, f


def _desc(**kw):
    d = _lib.HeadDesc()
    d.hidden, d.n_clusters, d.cluster_size, d.n_probes = 2048, 8016, 16, 256
    d.weight_dtype, d.score_dtype, d.sample_dtype = _lib.FH_BF16, _lib.FH_FP8_E4M3, _lib.FH_BF16
    fake = 1 << 20  # aligned, never dereferenced by validation
    d.w_perm, d.vocab_map, d.cluster_w, d.cluster_scale = fake, fake, fake, fake
    d.centroid_w = fake
    for k, v in kw.items():
        setattr(d, k, v)
    return d


def _create(lib, d):
    h = ctypes.c_void_p()
    st = lib.fh_head_create(ctypes.byref(d), ctypes.byref(h))
    return st, h


def test_version_and_error_string(lib):
    assert lib.fh_version() >= 1
    h = ctypes.c_void_p()
    assert lib.fh_head_create(None, ctypes.byref(h)) == _lib.FH_ERR_INVALID_ARGUMENT
    assert "null descriptor" in _lib.last_error()


@pytest.mark.parametrize("field,value,msg", [
    ("hidden", 100, "multiple of 16"),
    ("hidden", 0, "multiple of 16"),
    ("n_clusters", 0, "n_clusters"),
    ("n_clusters", 20000, "n_clusters"),
    ("cluster_size", 33, "cluster_size"),
    ("n_probes", 0, "n_probes"),
    ("n_probes", 9000, "n_probes"),
    ("weight_dtype", _lib.FH_FP8_E4M3, "weight_dtype"),
    ("score_dtype", _lib.FH_FP16, "score_dtype"),
    ("cluster_scale", None, "cluster_scale"),
    ("w_perm", None, "required"),
    ("w_perm", (1 << 20) + 4, "16-byte aligned"),
    ("n_special", 2, "special_slots"),
    ("cluster_base", -1, "cluster_base"),
])
def test_descriptor_validation(lib, field, value, msg):
    st, _ = _create(lib, _desc(**{field: value}))
    assert st == _lib.FH_ERR_INVALID_ARGUMENT
    assert msg in _lib.last_error()


def test_valid_descriptor_and_workspace_size(lib):
    st, h = _create(lib, _desc())
    assert st == _lib.FH_OK
    try:
        def rnd(x):
            return (x + 255) // 256 * 256
        for rows in (1, 8, 256):
            hist = 2 * 4 * (256 + 65536) * 4  # two epochs of 4 rows' histograms
            # tensor-core stage 1 from 5 rows: partial scores of every split of
            # the hidden dimension (tiles x splits fill the SMs once; no GPU
            # here, so the library assumes 148), and an f16 copy of the bf16
            # hidden rows for the fp8 stage-1 matrix
            splits = 1
            if rows >= 5:
                splits = max(1, min(2048 // 64, 148 // ((8016 + 127) // 128)))
            want = (256 + hist + rnd(rows * 8) + rnd(rows * 256 * 4)
                    + rnd(splits * rows * 8064 * 4) + 256)
            if rows >= 5:
                want += rnd(rows * 2048 * 2)
            if rows >= 16:  # batched steps: stage-2 index (row bit maps + meta, tiles)
                K = 8016
                tiles = -(-K // 8) + -(-K // 64) + 1
                want += rnd(K * 32) + 256 + rnd(tiles * 640)
            assert lib.fh_workspace_bytes(h, rows) == want
        assert lib.fh_workspace_bytes(None, 1) == 0
    finally:
        assert lib.fh_head_destroy(h) == _lib.FH_OK


def test_call_validation_needs_no_gpu(lib):
    st, h = _create(lib, _desc())
    assert st == _lib.FH_OK
    fake = 1 << 20
    ws = lib.fh_workspace_bytes(h, 4)
    s = None
    try:
        # zero rows: nothing to do
        assert lib.fh_get_next_token(h, None, 0, None, None, 0, s) == _lib.FH_OK
        assert lib.fh_tp_finalize(None, 0, None, s) == _lib.FH_OK
        assert lib.fh_block_sparse_argmax_atomic(None, 0, 64, None, None, 8, None, 8, 16,
                                                 _lib.FH_BF16, None, s) == _lib.FH_OK
        # bad arguments
        assert lib.fh_get_next_token(None, fake, 1, fake, fake, ws, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert lib.fh_get_next_token(h, fake, -1, fake, fake, ws, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert lib.fh_get_next_token(h, fake + 2, 1, fake, fake, ws, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert "16-byte" in _lib.last_error()
        assert lib.fh_get_next_token(h, fake, 4, fake, fake, ws - 1, s) == _lib.FH_ERR_WORKSPACE
        assert lib.fh_get_next_token(h, fake, 4, fake, None, ws, s) == _lib.FH_ERR_WORKSPACE
        assert lib.fh_get_next_token_sample(h, fake, 1, 0.0, 1, 0, fake, fake, ws, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert "temperature" in _lib.last_error()
        assert lib.fh_tp_select_and_score(h, fake, 1, 100, fake, 0, 1.0, 0, 0, fake, fake, ws,
                                          s) == _lib.FH_ERR_INVALID_ARGUMENT
        assert lib.fh_block_sparse_logits(fake, 1, 60, fake, fake, 8, 8, 16, _lib.FH_BF16, fake,
                                          s) == _lib.FH_ERR_INVALID_ARGUMENT
        assert lib.fh_block_sparse_logits(fake, 1, 64, fake, fake, 8, 8, 16, _lib.FH_FP8_E4M3,
                                          fake, s) == _lib.FH_ERR_INVALID_ARGUMENT
        # draft acceptance: empty batch, then bad sizes and pointers
        assert lib.fh_spec_accept(None, None, None, None, 0, 4, -1, None, s) == _lib.FH_OK
        assert lib.fh_spec_accept(fake, fake, fake, fake, -1, 4, -1, fake, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert lib.fh_spec_accept(fake, fake, fake, fake, 2, 4097, -1, fake, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert "max_spec_len" in _lib.last_error()
        assert lib.fh_spec_accept(None, fake, fake, fake, 2, 3, -1, fake, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
        assert lib.fh_spec_accept(fake, fake, None, fake, 2, 3, -1, fake, s) == \
            _lib.FH_ERR_INVALID_ARGUMENT
    finally:
        lib.fh_head_destroy(h)


def test_sampling_needs_raw_centroids(lib):
    st, h = _create(lib, _desc(centroid_w=None))
    assert st == _lib.FH_OK
    fake = 1 << 20
    ws = lib.fh_workspace_bytes(h, 1)
    try:
        assert lib.fh_get_next_token_sample(h, fake, 1, 1.0, 1, 0, fake, fake, ws, None) == \
            _lib.FH_ERR_UNSUPPORTED
    finally:
        lib.fh_head_destroy(h)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.load_library(str(tmp_path / "missing.so"))
