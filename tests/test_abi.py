"""The C-ABI library loads, exports every symbol include/w8a8.h declares, and
rejects bad arguments on the host before touching a GPU (no compute calls)."""
import ctypes
import os
import subprocess

import pytest

from imagine_b200 import _native as N


def test_library_exports_every_declared_symbol():
    declared = N.header_symbols()
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(N.LIB, name), f"{name} declared in include/w8a8.h but not exported"
    assert set(declared) == set(N.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version():
    assert N.LIB.w8a8_abi_version() == 103


def test_header_compiles_as_c():
    src = os.path.join(os.path.dirname(N.HEADER), "w8a8.h")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-fsyntax-only", "-x", "c", src],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def _err():
    return N.LIB.w8a8_last_error().decode()


def test_quantize_rejects_bad_arguments():
    rc = N.LIB.w8a8_quantize_rowwise(None, N.BF16, -1, 4, 4, None, 4, None, 0, 0, 0, None)
    assert rc == N.ERR_VALUE and "negative" in _err()
    rc = N.LIB.w8a8_quantize_rowwise(None, 7, 1, 4, 4, None, 4, None, 0, 0, 0, None)
    assert rc == N.ERR_VALUE and "dtype" in _err()
    rc = N.LIB.w8a8_quantize_rowwise(None, N.BF16, 1, 4, 4, None, 4, None, 9, 0, 0, None)
    assert rc == N.ERR_VALUE and "scale mode" in _err()
    rc = N.LIB.w8a8_quantize_rowwise(None, N.BF16, 1, 4, 4, None, 4, None, N.SCALE_KITCHEN_CUDA, 0,
                                     0, None)
    assert rc == N.ERR_VALUE and "NULL" in _err()  # mode accepted, then the pointers checked
    rc = N.LIB.w8a8_quantize_rowwise(None, N.BF16, 1, 4, 4, None, 4, None, 0, 0, 0, None)
    assert rc == N.ERR_VALUE and "NULL" in _err()
    # empty input is a no-op success, like the reference launcher's early return
    assert N.LIB.w8a8_quantize_rowwise(None, N.BF16, 0, 4, 4, None, 4, None, 0, 0, 0, None) == 0


def test_gemm_rejects_bad_epilogue():
    ep = N.Epilogue()
    ep.ws = None
    rc = N.LIB.w8a8_gemm_dequant(None, 16, None, 16, None, ctypes.byref(ep), None, N.BF16, 8, 4, 8,
                                 16, None, None)
    assert rc == N.ERR_VALUE and "weight scale" in _err()
    ep.ws = 16  # any non-null address; never dereferenced on this path
    ep.ws_numel = 3
    rc = N.LIB.w8a8_gemm_dequant(None, 16, None, 16, None, ctypes.byref(ep), None, N.BF16, 8, 4, 8,
                                 16, None, None)
    assert rc == N.ERR_VALUE and "scalar or per-output-channel" in _err()
    ep.ws_numel = 1
    ep.residual = 16
    rc = N.LIB.w8a8_gemm_dequant(None, 16, None, 16, None, ctypes.byref(ep), None, N.BF16, 8, 4, 8,
                                 16, None, None)
    assert rc == N.ERR_VALUE and "residual requires residual_scale" in _err()
    ep.residual = None
    ep.dequant_order = 7
    rc = N.LIB.w8a8_gemm_dequant(None, 16, None, 16, None, ctypes.byref(ep), None, N.BF16, 8, 4, 8,
                                 16, None, None)
    assert rc == N.ERR_VALUE and "dequant order" in _err()
    # the uncontracted Kitchen order exists on the CUDA-core paths only
    ep.dequant_order = N.DQ_SEPARATE
    rc = N.LIB.w8a8_gemm_dequant(None, 16, None, 16, None, ctypes.byref(ep), None, N.BF16, 8, 4, 8,
                                 16, None, None)
    assert rc == N.ERR_VALUE and "SEPARATE" in _err()
    rc = N.LIB.w8a8_dequantize_linear(None, None, ctypes.byref(ep), None, N.BF16, 4, 8, None)
    assert rc == N.ERR_VALUE and "NULL" in _err()  # order accepted, then the pointers checked
    ep.dequant_order = 0
    rc = N.LIB.w8a8_gemm_dequant(None, 16, None, 16, None, ctypes.byref(ep), None, N.S8, 8, 4, 8,
                                 16, None, None)
    assert rc == N.ERR_VALUE


def test_gemv_rejects_large_m():
    ep = N.Epilogue()
    ep.ws = 16
    ep.ws_numel = 1
    rc = N.LIB.w8a8_gemv_dequant(None, None, None, ctypes.byref(ep), None, N.BF16, 3, 8, 16, None)
    assert rc == N.ERR_VALUE and "M in {1, 2}" in _err()


def test_python_errors_map_to_exceptions():
    with pytest.raises(ValueError):
        N.check(N.ERR_VALUE)
    with pytest.raises(IndexError):
        N.check(N.ERR_INDEX)
    with pytest.raises(MemoryError):
        N.check(N.ERR_OOM)
    with pytest.raises(N.W8A8Error):
        N.check(N.ERR_ACCELERATOR)


def test_residual_scale_broadcasting():
    """The host side of the gated residual: how a residual_scale broadcast
    against the output becomes the table and rows-per-row the epilogue reads."""
    import torch
    from imagine_b200.linear import _residual_scale

    n = 8
    cpu = torch.device("cpu")
    t, rows = _residual_scale(torch.ones(n), (2, 5), n, torch.float32, cpu)
    assert t.shape == (n,) and rows == 0
    t, rows = _residual_scale(torch.ones(1, 1, n), (2, 5), n, torch.float32, cpu)
    assert t.shape == (n,) and rows == 0
    gate = torch.arange(2 * n, dtype=torch.float32).reshape(2, 1, n)
    t, rows = _residual_scale(gate, (2, 5), n, torch.float32, cpu)
    assert rows == 5 and torch.equal(t, gate.reshape(2, n))
    full = torch.randn(2, 5, n)
    t, rows = _residual_scale(full, (2, 5), n, torch.float32, cpu)
    assert rows == 1 and torch.equal(t, full.reshape(10, n))
    col = torch.randn(5, 1)  # broadcast along N: expanded to one row per output row
    t, rows = _residual_scale(col, (2, 5), n, torch.float32, cpu)
    assert rows == 1 and torch.equal(t, col.expand(2, 5, n).reshape(10, n))
    with pytest.raises(ValueError):
        _residual_scale(torch.ones(3, 1, n), (2, 5), n, torch.float32, cpu)


def test_fused_allgather_argument_errors():
    """The fused column-parallel entry points refuse bad ranks and pointers on
    the host, before any launch."""
    flags = (ctypes.c_void_p * 2)(0x1000, 0x2000)
    assert N.LIB.w8a8_peer_barrier(flags, 0, 1, 1, None) == N.ERR_VALUE  # one rank
    assert N.LIB.w8a8_peer_barrier(flags, 2, 2, 1, None) == N.ERR_VALUE  # rank outside
    recvs = (ctypes.c_void_p * 2)(0x4000, 0x5000)
    assert N.LIB.w8a8_allgather_finish(0x9000, N.BF16, 256, 16, 128, recvs, flags, 0, 9, 1,
                                       None) == N.ERR_VALUE  # too many ranks
    assert N.LIB.w8a8_allgather_finish(0x9000, N.BF16, 256, 16, 128, recvs, flags, 0, 2, 0,
                                       None) == N.ERR_VALUE  # epoch 0
    null_flags = (ctypes.c_void_p * 2)(0x1000, 0)
    assert N.LIB.w8a8_peer_barrier(null_flags, 0, 2, 1, None) == N.ERR_VALUE
    ep = N.Epilogue()
    ep.ws = 0x3000
    ep.ws_numel = 1
    # the output's row is narrower than world * N_shard
    rc = N.LIB.w8a8_gemm_dequant_allgather(0x6000, 64, 0x7000, 64, 0x8000, ctypes.byref(ep), 0x9000,
                                           N.BF16, 128, 16, 128, 64, recvs, flags, 0, 2, 1, None,
                                           None)
    assert rc == N.ERR_VALUE and b"ldo" in N.LIB.w8a8_last_error()
    # a receive buffer: every shard's 32 x 32 chunks, for every rank
    assert N.LIB.w8a8_allgather_recv_bytes(40, 72, N.BF16, 2) == 2 * 2 * 3 * 2048
    # row-parallel reduce-scatter: owned row blocks of a multiple of 32 rows,
    # one int32 chunk slot per sender, owned row block and column block
    assert N.LIB.w8a8_reduce_scatter_rows(600, 2) == 320
    assert N.LIB.w8a8_reduce_scatter_rows(10, 4) == 32
    assert N.LIB.w8a8_reduce_scatter_recv_bytes(600, 1536, 2) == 2 * 10 * 48 * 4096
    rc = N.LIB.w8a8_gemm_s32_reduce_scatter(0x6000, 64, 0x7000, 64, 16, 130, 64, recvs, flags, 0, 2,
                                            1, None, None)
    assert rc == N.ERR_VALUE and b"multiple of 4" in N.LIB.w8a8_last_error()
    assert N.LIB.w8a8_gemm_s32_reduce_scatter(0x6000, 64, 0x7000, 64, 16, 128, 64, recvs, flags, 0,
                                              9, 1, None, None) == N.ERR_VALUE  # too many ranks
    stages = (ctypes.c_void_p * 2)(0x8000, 0x9000)
    rc = N.LIB.w8a8_reduce_scatter_finish(0xa000, ctypes.byref(ep), 0xb000, N.BF16, 100, 16, 128,
                                          recvs, stages, flags, 0, 2, 1, None)
    assert rc == N.ERR_VALUE and b"ldo" in N.LIB.w8a8_last_error()
