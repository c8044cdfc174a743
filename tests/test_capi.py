"""CPU checks of the C-ABI library: it loads, exports every declared symbol, and the host
logic (argument checks, workspace sizing, error mapping) behaves without a GPU."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from exp3_b200 import _capi, ops
from exp3_b200.attention import AttentionBackend

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(fpx_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = _capi.lib()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(_capi.SIGNATURES) | {"fpx_get_device_error"}


def test_status_strings_and_version():
    lib = _capi.lib()
    assert lib.fpx_version() >= 1
    assert lib.fpx_status_string(0) == b"ok"
    assert b"workspace" in lib.fpx_status_string(-5)


def test_workspace_sizes_grow_with_length():
    small = ops.workspace_bytes("mean_native", 1, 4096, 28, 4)
    big = ops.workspace_bytes("mean_native", 1, 32768, 28, 4)
    assert 0 < small < big
    assert big % 256 == 0
    # lists of (b, h, t) dominate: B * H * nb * nb int32
    assert big >= 28 * 256 * 256 * 4


def test_argument_errors_are_statuses_not_crashes():
    lib = _capi.lib()
    # null pointers and bad sizes are rejected on the host before any launch
    rc = lib.fpx_block_mean_k(None, 0, 0, 0, 1, 128, 1, 128, 128, None, None)
    assert rc == -1
    rc = lib.fpx_block_mean_k(ctypes.c_void_p(16), 0, 0, 0, 1, 128, 1, 64, 128, ctypes.c_void_p(16), None)
    assert rc == -3  # head_dim 64 is not compiled
    rc = lib.fpx_prefill_attention(6, 0.08, 2, 4, 2, *([None, 0, 0, 0] * 3), 1, 128, 28, 4, 128, 128,
                                   0.088, 0, 4, 0, 1, None, 0, 0, 0, None, None, 0, 7, None)
    assert rc == -1  # null tensors
    rc = lib.fpx_prefill_attention(8, 0.08, 2, 4, 2, *([None, 0, 0, 0] * 3), 1, 128, 28, 4, 128, 128,
                                   0.088, 0, 4, 0, 1, None, 0, 0, 0, None, None, 0, 7, None)
    assert rc == -1  # no method 8
    assert lib.fpx_rescue_tail_workspace_bytes(1, 1153, 4, 2, 128, 128) >= 4 * 10 * 10
    assert lib.fpx_rescue_tail_workspace_bytes(1, 1153, 4, 2, 64, 128) == 0


def test_ops_refuse_cpu_tensors():
    q = torch.zeros(1, 128, 28, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 128, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(_capi.FpxError):
        ops.prefill_attention(q, k, k, "mean_native", 0.08, 128 ** -0.5)


def test_backend_configure_matches_reference_errors():
    backend = AttentionBackend(alpha=0.08)
    backend.configure("cgf_mean", 0.16)
    assert (backend.method, backend.alpha) == ("cgf_mean", 0.16)
    with pytest.raises(ValueError):
        backend.configure("flash")
    with pytest.raises(ValueError):
        ops.prefill_attention(None, None, None, "flash", 0.08, 1.0)


def test_options_and_head_dims_on_the_host():
    """fpx_set_option takes exactly the documented values; workspace sizes exist for head dims
    128 and 256 and for nothing else (no GPU needed)."""
    lib = _capi.lib()
    for key, values in ((1, (0, 1, 2)), (2, (0, 2, 3)), (3, (0, 1)), (4, (0, 1)), (5, (0, 1))):
        for value in values:
            assert lib.fpx_set_option(key, value) == 0, (key, value)
        assert lib.fpx_set_option(key, 7) == -1
    for key, value in ((1, 0), (2, 0), (3, 0), (4, 0), (5, 0)):  # back to the defaults
        assert lib.fpx_set_option(key, value) == 0
    assert lib.fpx_set_option(6, 0) == -1 and lib.fpx_set_option(0, 0) == -1
    for d, ok in ((128, True), (256, True), (64, False), (192, False)):
        assert (lib.fpx_prefill_workspace_bytes(2, 1, 4096, 16, 4, d, 128) > 0) == ok, d
        assert (lib.fpx_decode_workspace_bytes(1, 1, 16, 4, 4096, d) > 0) == ok, d
        assert (lib.fpx_rescue_tail_workspace_bytes(1, 4096, 16, 4, d, 128) > 0) == ok, d
    # the d = 256 workspace holds twice the descriptor bytes
    assert lib.fpx_prefill_workspace_bytes(2, 1, 4096, 16, 4, 256, 128) > lib.fpx_prefill_workspace_bytes(
        2, 1, 4096, 16, 4, 128, 128)
    assert lib.fpx_ar_buffer_bytes(28672) == 768 + 2 * 8 * 28672 * 2 and lib.fpx_ar_buffer_bytes(12) == 0
