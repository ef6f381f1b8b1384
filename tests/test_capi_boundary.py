"""The C ABI library loads on a CPU-only host and exports every symbol the
header declares; host-only entry points answer without a GPU."""

import ctypes
import os
import re

import pytest

from gmmxx_b200 import _native, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gmmxx_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"GMMXX_API\s+[\w\s\*]+?\b(gmmxx_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_native.LIB_PATH):
        build.build()
    return _native.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "gmmxx_em_accumulate" in syms and "gmmxx_assign" in syms
    assert len(syms) >= 14


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_binding_covers_the_header(lib):
    assert sorted(_native.exported_symbols()) == declared_symbols()


def test_abi_version(lib):
    assert lib.gmmxx_abi_version() == 1


def test_stat_width_matches_layout(lib):
    d = 16
    assert _native.stat_width(_native.SPHERICAL, d) == d + 2
    assert _native.stat_width(_native.DIAG, d) == 2 * d + 1
    assert _native.stat_width(_native.TIED, d) == d + 1
    assert _native.stat_width(_native.FULL, d) == 1 + d + d * (d + 1) // 2
    assert lib.gmmxx_stat_width(9, 4) == -1


def test_workspace_bytes_monotone(lib):
    a = _native.workspace_bytes(_native.DIAG, 1, 1000, 64, 512)
    b = _native.workspace_bytes(_native.DIAG, 1, 2000, 64, 512)
    assert 0 < a < b
    assert a % 256 == 0
    assert _native.workspace_bytes(7, 1, 10, 4, 4) == 0


def test_invalid_arguments_rejected_without_gpu(lib):
    # validation runs before any CUDA call
    rc = lib.gmmxx_em_prepare(9, 1, 4, 4, None, None, None, 1e-6, 1e-8, None, 0, None)
    assert rc == _native.ERR_INVALID
    assert b"covariance" in lib.gmmxx_last_error()
    rc = lib.gmmxx_assign(_native.DIAG, _native.FLOAT32, None, 1, 10, 4096, 3, None, None, None, None, None, 0, None)
    assert rc == _native.ERR_UNSUPPORTED
    with pytest.raises(_native.UnsupportedShape):
        _native.call("gmmxx_assign", _native.FULL, _native.FLOAT32, None, 1, 10, 64, 3, None, None, None, None,
                     None, 0, None)


def test_workspace_too_small_is_reported(lib):
    buf = ctypes.create_string_buffer(1024 + 256)
    addr = (ctypes.addressof(buf) + 255) // 256 * 256
    m = ctypes.c_float(0.0)
    rc = lib.gmmxx_em_prepare(_native.DIAG, 1, 4, 3, ctypes.addressof(m), ctypes.addressof(m), ctypes.addressof(m),
                              1e-6, 1e-8, addr, 16, None)
    assert rc == _native.ERR_WORKSPACE


def test_accumulate_path_selection(lib, monkeypatch):
    """Host-side kernel selection: config-1 shapes take the tensor-core kernel,
    fp32 / tied / small-N shapes and GMMXX_B200_KERNEL=simt the CUDA-core ones."""
    from gmmxx_b200 import _native as nat

    monkeypatch.delenv("GMMXX_B200_KERNEL", raising=False)
    assert nat.accumulate_path(nat.DIAG, nat.BFLOAT16, 1, 50_000_000, 64, 512) == 1
    assert nat.accumulate_path(nat.SPHERICAL, nat.BFLOAT16, 1, 1 << 20, 128, 1024) == 1
    assert nat.accumulate_path(nat.DIAG, nat.FLOAT32, 1, 50_000_000, 64, 512) == 0
    assert nat.accumulate_path(nat.TIED, nat.BFLOAT16, 1, 1 << 20, 64, 256) == 0
    assert nat.accumulate_path(nat.DIAG, nat.BFLOAT16, 1, 1000, 64, 512) == 0
    assert nat.accumulate_path(nat.DIAG, nat.BFLOAT16, 2, 1 << 20, 64, 512) == 0
    monkeypatch.setenv("GMMXX_B200_KERNEL", "simt")
    assert nat.accumulate_path(nat.DIAG, nat.BFLOAT16, 1, 50_000_000, 64, 512) == 0
    with pytest.raises(nat.GmmxxError):
        nat.accumulate_path(7, nat.BFLOAT16, 1, 10, 4, 4)


def test_large_k_spherical_workspace_has_per_group_row_partials(lib):
    """Spherical K > 1024: the first pass writes (max, sum) row partials per
    group of 256 components (2 chunks), so the workspace grows by 8 B per
    row per such group, plus the per-row log-sum-exp buffers, over the
    fixed-size tables."""
    k, d = 8192, 128
    n1, n2 = 1 << 20, 1 << 21
    slope = (_native.workspace_bytes(_native.SPHERICAL, 1, n2, d, k) -
             _native.workspace_bytes(_native.SPHERICAL, 1, n1, d, k)) / (n2 - n1)
    groups = k // 256
    per_row = 8 * groups + 4 + 4 + 8 / 64  # row partials, tc log-sum-exp, CUDA-core lse, LL partials
    assert abs(slope - per_row) < 0.01
    # one-pass window (K <= 1024): no per-group partials
    slope1 = (_native.workspace_bytes(_native.SPHERICAL, 1, n2, d, 1024) -
              _native.workspace_bytes(_native.SPHERICAL, 1, n1, d, 1024)) / (n2 - n1)
    assert abs(slope1 - (4 + 8 / 64)) < 0.01


def test_topk_scratch_bytes(lib):
    """Two [B][N][top_k] lists (component indices, responsibilities), each
    rounded up to 256 bytes; 0 for invalid sizes."""
    assert _native.topk_scratch_bytes(2, 1000, 8) == 2 * ((2 * 1000 * 8 * 4 + 255) // 256 * 256)
    assert _native.topk_scratch_bytes(1, 0, 4) == 0
    assert lib.gmmxx_topk_scratch_bytes(0, 10, 4) == 0
    assert lib.gmmxx_topk_scratch_bytes(1, 10, 0) == 0


def _aligned(nbytes, align=256):
    buf = ctypes.create_string_buffer(nbytes + align)
    return buf, (ctypes.addressof(buf) + align - 1) // align * align


def test_topk_arguments_rejected_without_gpu(lib):
    """top_k outside [1, K - 1], above the engine window, or a scratch buffer
    that is too small or misaligned: refused before any CUDA call."""
    b, n, d, k = 1, 10, 4, 100
    wsb = _native.workspace_bytes(_native.SPHERICAL, b, n, d, k)
    ws_buf, ws = _aligned(wsb)
    x = ctypes.c_float(0.0)
    stats = ctypes.c_float(0.0)
    ll = ctypes.c_double(0.0)
    sb = _native.topk_scratch_bytes(b, n, 4)
    sc_buf, sc = _aligned(sb)

    def call(top_k, scratch=sc, scratch_bytes=sb):
        return lib.gmmxx_em_accumulate_topk(_native.SPHERICAL, _native.FLOAT32, ctypes.addressof(x), b, n, d, k,
                                            top_k, ws, wsb, scratch, scratch_bytes, ctypes.addressof(stats),
                                            ctypes.addressof(ll), None)

    assert call(0) == _native.ERR_INVALID and b"top_k" in lib.gmmxx_last_error()
    assert call(k) == _native.ERR_INVALID
    assert call(65) == _native.ERR_UNSUPPORTED
    assert call(4, scratch_bytes=sb - 1) == _native.ERR_WORKSPACE
    assert call(4, scratch=None) == _native.ERR_INVALID
    assert call(4, scratch=sc + 4) == _native.ERR_INVALID
    assert b"aligned" in lib.gmmxx_last_error()


def test_resolve_approx_top_k():
    """The reference's _resolve_approx_top_k (torch_fallback.py:599-607) plus
    the engine window."""
    from gmmxx_b200 import engine

    assert engine.resolve_approx_top_k(None, 8) is None
    assert engine.resolve_approx_top_k(8, 8) is None
    assert engine.resolve_approx_top_k(9, 8) is None
    assert engine.resolve_approx_top_k(3, 8) == 3
    with pytest.raises(ValueError):
        engine.resolve_approx_top_k(0, 8)
    with pytest.raises(_native.UnsupportedShape):
        engine.resolve_approx_top_k(engine.MAX_APPROX_TOP_K + 1, 1000)


def test_entry_points_validate_every_pointer_before_launching(lib):
    """Each entry point refuses a NULL output, parameter or workspace, or a bad
    scalar, with GMMXX_ERR_INVALID and a message naming it -- before any CUDA
    call, so a CPU-only host answers too."""
    b, n, d, k = 1, 10, 4, 3
    wsb = _native.workspace_bytes(_native.TIED, b, n, d, k)
    ws_buf, ws = _aligned(wsb)
    f = ctypes.c_float(1.0)
    p = ctypes.addressof(f)
    dbl = ctypes.c_double(0.0)
    pd = ctypes.addressof(dbl)
    cov, dt = _native.DIAG, _native.FLOAT32
    infer_args = lambda out: (cov, dt, p, b, n, d, k, p, p, p, out, ws, wsb, None)
    cases = [
        ("labels_out", lib.gmmxx_assign, infer_args(None)),
        ("lse_out", lib.gmmxx_logsumexp, infer_args(None)),
        ("proba_out", lib.gmmxx_predict_proba, infer_args(None)),
        ("log_norm", lib.gmmxx_resp, (cov, dt, p, b, n, d, k, p, p, p, None, p, ws, wsb, None)),
        ("resp_out", lib.gmmxx_resp, (cov, dt, p, b, n, d, k, p, p, p, p, None, ws, wsb, None)),
        ("means", lib.gmmxx_assign, (cov, dt, p, b, n, d, k, None, p, p, p, ws, wsb, None)),
        ("x", lib.gmmxx_logsumexp, (cov, dt, None, b, n, d, k, p, p, p, p, ws, wsb, None)),
        ("workspace", lib.gmmxx_predict_proba, (cov, dt, p, b, n, d, k, p, p, p, p, None, wsb, None)),
        ("stats", lib.gmmxx_em_accumulate, (cov, dt, p, b, n, d, k, ws, wsb, None, pd, None)),
        ("log_likelihood", lib.gmmxx_em_accumulate, (cov, dt, p, b, n, d, k, ws, wsb, p, None, None)),
        ("x", lib.gmmxx_em_accumulate, (cov, dt, None, b, n, d, k, ws, wsb, p, pd, None)),
        ("xx_total", lib.gmmxx_em_finalize, (_native.TIED, b, d, k, n, p, pd, None, 1e-6, 1e-8, p, p, p, None,
                                             None)),
        ("n_total", lib.gmmxx_em_finalize, (cov, b, d, k, 0, p, pd, None, 1e-6, 1e-8, p, p, p, None, None)),
        ("min_weight", lib.gmmxx_em_finalize, (cov, b, d, k, n, p, pd, None, 1e-6, 0.0, p, p, p, None, None)),
        ("weights", lib.gmmxx_em_prepare, (cov, b, d, k, p, p, None, 1e-6, 1e-8, ws, wsb, None)),
        ("reg_covar", lib.gmmxx_em_prepare, (cov, b, d, k, p, p, p, -1.0, 1e-8, ws, wsb, None)),
        ("xx_out", lib.gmmxx_xx_total, (dt, p, b, n, d, None, ws, wsb, None)),
        ("status_out", lib.gmmxx_workspace_status, (ws, None, None)),
        ("in", lib.gmmxx_canary_add_offset, (None, p, 4, 1, None)),
    ]
    for name, fn, args in cases:
        assert fn(*args) == _native.ERR_INVALID, name
        assert name.encode() in lib.gmmxx_last_error(), (name, lib.gmmxx_last_error())
    # a misaligned workspace is refused the same way
    assert lib.gmmxx_assign(*infer_args(p)[:11], ws + 8, wsb, None) == _native.ERR_INVALID
    assert b"aligned" in lib.gmmxx_last_error()


def test_missing_library_raises_cuda_backend_unavailable():
    """No fallback when the native library is absent (the reference's
    CudaBackendUnavailable, gmmxx/_cuda.py:57-64): a fresh interpreter whose
    library path does not exist gets the exception from load(), with the
    build command in its message."""
    import subprocess
    import sys

    code = (
        "from gmmxx_b200 import _native as nat\n"
        "try:\n"
        "    nat.load('/nonexistent/libgmmxx_b200.so')\n"
        "except nat.CudaBackendUnavailable as e:\n"
        "    print('unavailable:', 'not built' in str(e))\n"
    )
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert "unavailable: True" in out.stdout


def test_last_accumulate_path_before_any_call(lib):
    # no accumulate call has succeeded on this thread (none can without a GPU)
    assert lib.gmmxx_last_accumulate_path() in (-1, 0, 1, 2)
    assert _native.PATH_NAMES[-1] is None
