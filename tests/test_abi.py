"""CPU: the C-ABI library loads, exports every symbol include/ctfa.h declares,
and rejects bad arguments on the host before any CUDA call."""
import ctypes
import re

import pytest

from cudatransformer_b200 import _lib


def declared_functions():
    text = _lib.HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ctfa_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("ctfa_forward", "ctfa_backward", "ctfa_backward_workspace_bytes", "ctfa_version"):
        assert required in names


def test_every_declared_symbol_is_exported(ctfa):
    for name in declared_functions():
        assert hasattr(ctfa, name), f"{name} declared in include/ctfa.h but not exported"


def test_binding_table_matches_header():
    assert set(_lib.SIGNATURES) == set(declared_functions())


def test_version_and_status_strings(ctfa):
    assert ctfa.ctfa_version() >= 10000
    for code in range(7):
        assert ctfa.ctfa_status_string(code).decode().startswith("CTFA_")


FAKE = ctypes.c_void_p(4096)  # never dereferenced: every call below fails validation first


@pytest.mark.parametrize(
    "args,status",
    [
        ((None, FAKE, FAKE, FAKE, None, 1, 1, 8, 64, 0, 0, None, 0, None), _lib.CTFA_ERR_INVALID_ARGUMENT),
        ((FAKE, FAKE, FAKE, FAKE, None, 0, 1, 8, 64, 0, 0, None, 0, None), _lib.CTFA_ERR_INVALID_ARGUMENT),
        ((FAKE, FAKE, FAKE, FAKE, None, 1, 1, -3, 64, 0, 0, None, 0, None), _lib.CTFA_ERR_INVALID_ARGUMENT),
        ((FAKE, FAKE, FAKE, FAKE, None, 1, 1, 8, 64, 7, 0, None, 0, None), _lib.CTFA_ERR_INVALID_ARGUMENT),
        ((FAKE, FAKE, FAKE, FAKE, None, 1, 1, 8, 300, 0, 0, None, 0, None), _lib.CTFA_ERR_UNSUPPORTED),
        # fp32 on the tensor-core path needs the rounding workspace
        ((FAKE, FAKE, FAKE, FAKE, None, 1, 1, 8, 64, 0, 0, None, 0, None), _lib.CTFA_ERR_WORKSPACE),
    ],
)
def test_forward_argument_validation(ctfa, args, status):
    assert ctfa.ctfa_forward(*args) == status
    assert _lib.last_error()


def test_workspace_sizes(ctfa):
    n = 2 * 3 * 100 * 64
    assert ctfa.ctfa_forward_workspace_bytes(2, 3, 100, 64, _lib.CTFA_DTYPE_F32) >= 3 * n * 4
    assert ctfa.ctfa_forward_workspace_bytes(2, 3, 100, 64, _lib.CTFA_DTYPE_BF16) == 0
    assert ctfa.ctfa_forward_workspace_bytes(2, 3, 100, 32, _lib.CTFA_DTYPE_F32) == 0  # SIMT path
    assert ctfa.ctfa_backward_workspace_bytes(2, 3, 100, 64, _lib.CTFA_DTYPE_F32) >= 4 * n * 4


def test_backward_argument_validation(ctfa):
    ws = ctfa.ctfa_backward_workspace_bytes(2, 3, 100, 64, _lib.CTFA_DTYPE_BF16)
    assert ws >= 2 * 3 * 100 * 4 and ws % 256 == 0
    args = [FAKE] * 9 + [None, 0, 2, 3, 100, 64, _lib.CTFA_DTYPE_BF16, 1, None]
    assert ctfa.ctfa_backward(*args) == _lib.CTFA_ERR_WORKSPACE
    args[5] = None  # lse
    assert ctfa.ctfa_backward(*args) == _lib.CTFA_ERR_INVALID_ARGUMENT
    args = [FAKE] * 9 + [ctypes.c_void_p(4096 + 8), ws, 2, 3, 100, 64, _lib.CTFA_DTYPE_BF16, 1, None]
    assert ctfa.ctfa_backward(*args) == _lib.CTFA_ERR_MISALIGNED  # workspace not 256-byte aligned
    assert ctfa.ctfa_backward_workspace_bytes(0, 1, 1, 64, 0) == 0


def test_wait_limit_validation(ctfa):
    assert ctfa.ctfa_set_wait_limit_ns(0) == _lib.CTFA_ERR_INVALID_ARGUMENT
    assert ctfa.ctfa_set_wait_limit_ns(2_000_000_000) == _lib.CTFA_OK
    assert ctfa.ctfa_selftest_wait_timeout(0, None) == _lib.CTFA_ERR_INVALID_ARGUMENT


def test_projection_argument_validation(ctfa):
    """The projection entry points reject null tensors, non-positive sizes,
    unknown dtypes and inconsistent gradient requests before any CUDA call."""
    E = _lib.CTFA_ERR_INVALID_ARGUMENT
    fwd = [FAKE] * 10 + [2, 16, 64, 1, 64, _lib.CTFA_DTYPE_F32, None]
    for i in (0, 1, 3, 5, 7, 8, 9):  # x, wq, wk, wv, q, k, v are required (biases are optional)
        a = list(fwd)
        a[i] = None
        assert ctfa.ctfa_qkv_forward(*a) == E
    for i, bad in ((10, 0), (11, -1), (12, 0), (13, 0), (14, 0), (15, 9)):
        a = list(fwd)
        a[i] = bad
        assert ctfa.ctfa_qkv_forward(*a) == E
    bwd = [FAKE] * 14 + [2, 16, 64, 1, 64, _lib.CTFA_DTYPE_F32, None]
    a = list(bwd)
    a[1] = None  # dq
    assert ctfa.ctfa_qkv_backward(*a) == E
    a = list(bwd)
    a[9] = None  # dwk missing while dwq, dwv given
    assert ctfa.ctfa_qkv_backward(*a) == E
    a = list(bwd)
    a[0] = None  # x needed for the weight gradients
    assert ctfa.ctfa_qkv_backward(*a) == E
    a = list(bwd)
    a[4] = None  # wq needed for dx
    assert ctfa.ctfa_qkv_backward(*a) == E
    ofwd = [FAKE] * 4 + [2, 16, 64, 1, 64, _lib.CTFA_DTYPE_BF16, None]
    for i in (0, 1, 3):
        a = list(ofwd)
        a[i] = None
        assert ctfa.ctfa_out_proj_forward(*a) == E
    obwd = [FAKE] * 6 + [2, 16, 64, 1, 64, _lib.CTFA_DTYPE_BF16, None]
    a = list(obwd)
    a[1] = None  # dy
    assert ctfa.ctfa_out_proj_backward(*a) == E
    a = list(obwd)
    a[0] = None  # a needed for dWo
    assert ctfa.ctfa_out_proj_backward(*a) == E
    a = list(obwd)
    a[2] = None  # wo needed for da
    assert ctfa.ctfa_out_proj_backward(*a) == E


def test_linear_and_layernorm_argument_validation(ctfa):
    E = _lib.CTFA_ERR_INVALID_ARGUMENT
    lf = [FAKE] * 4 + [16, 64, 64, 0, _lib.CTFA_DTYPE_F32, None]
    for i in (0, 1, 3):  # x, w, y required; b optional
        a = list(lf)
        a[i] = None
        assert ctfa.ctfa_linear_forward(*a) == E
    for i in (4, 5, 6):
        a = list(lf)
        a[i] = 0
        assert ctfa.ctfa_linear_forward(*a) == E
    lb = [FAKE] * 7 + [16, 64, 64, _lib.CTFA_DTYPE_F32, None]
    a = list(lb)
    a[1] = None  # dy
    assert ctfa.ctfa_linear_backward(*a) == E
    a = list(lb)
    a[0] = None  # x needed for dw
    assert ctfa.ctfa_linear_backward(*a) == E
    a = list(lb)
    a[2] = None  # w needed for dx
    assert ctfa.ctfa_linear_backward(*a) == E
    nf = [FAKE] * 6 + [16, 64, 1e-5, _lib.CTFA_DTYPE_F32, None]
    a = list(nf)
    a[8] = 0.0  # eps
    assert ctfa.ctfa_layernorm_forward(*a) == E
    a = list(nf)
    a[2] = None  # b
    assert ctfa.ctfa_layernorm_forward(*a) == E
    nb = [FAKE] * 8 + [16, 64, 1e-5, _lib.CTFA_DTYPE_F32, None]
    nb[5] = None  # dx
    assert ctfa.ctfa_layernorm_backward(*nb) == E
