"""The C ABI without a GPU: the library loads, exports every symbol include/hsd.h
declares, and its host-side argument checks return the documented status codes with a
message (no kernel is launched by any of these calls)."""
import ctypes
import os
import re

import pytest

from conftest import REPO

import hsd_b200._lib as L

HEADER = os.path.join(REPO, "include", "hsd.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(hsd_\w+)\s*\(", text)))


def test_library_is_built_and_loads():
    assert os.path.exists(L.LIB_PATH)
    L.lib()


def test_every_declared_symbol_is_exported_and_bound():
    lib = L.lib()
    names = declared_symbols()
    assert names, "no declarations parsed from include/hsd.h"
    for n in names:
        assert hasattr(lib, n), f"{n} declared in hsd.h but not exported by libhsd.so"
    assert sorted(L.SIGNATURES) == names, "the ctypes signature table must match hsd.h"


def test_abi_version():
    assert L.lib().hsd_abi_version() == 1


def _rc(name, *args):
    return getattr(L.lib(), name)(*args)


def test_null_pointer_is_arg_error_with_message():
    rc = _rc("hsd_nibble_transpose", None, None, 1, 8, 1, None)
    assert rc == L.HSD_ERR_ARG
    assert b"null" in L.lib().hsd_last_error_string()


def test_transpose_shape_checks():
    p = ctypes.c_void_p(16)
    q = ctypes.c_void_p(32)
    assert _rc("hsd_nibble_transpose", p, q, 1, 12, 1, None) == L.HSD_ERR_SHAPE   # R % 8 != 0
    assert _rc("hsd_nibble_transpose", p, p, 1, 8, 1, None) == L.HSD_ERR_ARG      # aliasing
    assert _rc("hsd_swap_last2_u16", p, q, 0, 8, 1, None) == L.HSD_ERR_SHAPE


def test_decode_argument_checks():
    p = ctypes.c_void_p(256)
    args = dict(h_dtype=L.HSD_BF16, s_dtype=L.HSD_BF16, y_dtype=L.HSD_BF16, B=1, D=2688, F=1856,
                FS=3712, topk=6, E=128, loadsc=1)

    def call(**kw):
        a = dict(args, **kw)
        return _rc("hsd_sparse_down_decode", p, a["h_dtype"], p, p, p, p, p, a["s_dtype"], p, p, p,
                   None, p, a["y_dtype"], a["B"], a["D"], a["F"], a["FS"], a["topk"], a["E"],
                   a["loadsc"], None)

    assert call(D=2680) == L.HSD_ERR_SHAPE          # D % 32
    assert call(F=1850) == L.HSD_ERR_SHAPE          # F % 64
    assert call(B=0) == L.HSD_ERR_SHAPE
    assert call(s_dtype=L.HSD_F32) == L.HSD_ERR_DTYPE
    assert call(h_dtype=9) == L.HSD_ERR_DTYPE
    misaligned = ctypes.c_void_p(258)
    rc = _rc("hsd_sparse_down_decode", p, L.HSD_BF16, p, p, misaligned, p, p, L.HSD_BF16, p, p, p,
             None, p, L.HSD_BF16, 1, 2688, 1856, 3712, 6, 128, 1, None)
    assert rc == L.HSD_ERR_ALIGN
    rc = _rc("hsd_sparse_down_decode", None, L.HSD_BF16, p, p, p, p, p, L.HSD_BF16, p, p, p,
             None, p, L.HSD_BF16, 1, 2688, 1856, 3712, 6, 128, 1, None)
    assert rc == L.HSD_ERR_ARG


def test_python_wrappers_refuse_cpu_tensors():
    import torch
    import hsd_b200
    with pytest.raises(ValueError):
        hsd_b200.nibble_transpose(torch.zeros((8, 1), dtype=torch.int32))


def test_ep_buffer_sizes_and_argument_checks():
    ib, wb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert _rc("hsd_ep_buffer_bytes", 8, 512, 6, 1856, 3712, 2688, 128, 0, ctypes.byref(ib), ctypes.byref(wb)) == L.HSD_OK
    # inbox: 8 ranks x 3072 slots of h rows + ids, gains, return addresses, + 3072 + 512 fp32 partial rows
    assert 130e6 < ib.value < 131e6
    assert 201e6 < wb.value < 203e6         # dominated by the gathered fp16 A tiles (K up to FS)
    one_i, one_w = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert _rc("hsd_ep_buffer_bytes", 1, 512, 6, 1856, 3712, 2688, 128, 0, ctypes.byref(one_i), ctypes.byref(one_w)) == 0
    assert one_i.value < ib.value
    assert _rc("hsd_ep_buffer_bytes", 3, 512, 6, 1856, 3712, 2688, 128, 0, ctypes.byref(ib), ctypes.byref(wb)) == L.HSD_ERR_SHAPE
    assert _rc("hsd_ep_buffer_bytes", 17, 512, 6, 1856, 3712, 2688, 128, 0, ctypes.byref(ib), ctypes.byref(wb)) == L.HSD_ERR_SHAPE
    assert _rc("hsd_ep_buffer_bytes", 8, 512, 6, 1856, 3712, 2680, 128, 0, ctypes.byref(ib), ctypes.byref(wb)) == L.HSD_ERR_SHAPE
    ws = ctypes.c_void_p(1 << 20)
    p = ctypes.c_void_p(256)
    d = lambda rank, B, ws=ws, h=L.HSD_BF16: _rc("hsd_ep_dispatch", ws, rank, 8, 512, p, h, p, p, B, 6, 1856,  # noqa: E731
                                                 3712, 2688, 128, None, 1.0, None)
    assert d(8, 4) == L.HSD_ERR_ARG             # rank outside the world
    assert d(0, 513) == L.HSD_ERR_SHAPE         # more tokens than max_tokens
    assert d(0, 4, ws=ctypes.c_void_p((1 << 20) + 16)) == L.HSD_ERR_ALIGN
    assert d(0, 4, h=L.HSD_F32) == L.HSD_ERR_DTYPE
    assert _rc("hsd_ep_expert", ws, None, 0, 8, 512, p, L.HSD_BF16, 4, p, p, p, p, p, p, L.HSD_BF16, 6, 1856, 3712,
               2688, 128, 0, 1.0, None) == L.HSD_ERR_ARG            # no inbox
    assert _rc("hsd_ep_expert", ws, p, 0, 8, 512, p, L.HSD_BF16, 4, p, p, p, None, p, p, L.HSD_BF16, 6, 1856, 3712,
               2688, 128, 0, 1.0, None) == L.HSD_ERR_ARG            # no shared weights with FS > 0
    assert _rc("hsd_ep_expert", ws, p, 0, 8, 512, p, L.HSD_BF16, 4, p, p, p, p, p, p, L.HSD_BF16, 6, 1856, 3712,
               2688, 128, 300, 1.0, None) == L.HSD_ERR_SHAPE          # more than 256 local experts
    assert _rc("hsd_ep_combine", ws, 0, 8, 512, None, 4, 6, 1856, 3712, 2688, 128, 1.0, None) == L.HSD_ERR_ARG
    assert _rc("hsd_ep_set_peers", ws, None, 2, None) == L.HSD_ERR_ARG
    assert _rc("hsd_ep_alloc", 0, ctypes.byref(ctypes.c_void_p())) == L.HSD_ERR_ARG
