"""Argument checks of the allocation-free cascade attention entry point (csrc/phx_noalloc.h). A pass that
has tiles but no work list is rejected with PHX_NOALLOC_ERR_BAD_ARGS before anything is launched, so these
calls run without a GPU (the pointers are never dereferenced)."""
import ctypes

import pytest

BAD_ARGS = 2


def _fn():
    try:
        import phung5_b200._C as C
    except ImportError:
        pytest.skip("extension not built")
    lib = ctypes.CDLL(C.__file__)
    f = lib.phx_cascade_attention_noalloc
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    f.argtypes = [vp] * 8 + [vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, ctypes.c_float, vp, vp, vp, vp]
    f.restype = ctypes.c_int
    return f


def _call(f, lists1, n1, lists2, n2):
    fake = ctypes.c_void_p(256)            # never dereferenced: the checks return first
    return f(fake, fake, fake, fake, fake, fake, fake, fake, *lists1, n1, *lists2, n2, 64, 8, 2, 0, 0.1,
             fake, None, None, None)


def test_missing_suffix_work_list_is_rejected():
    f = _fn()
    fake = ctypes.c_void_p(256)
    for missing in range(3):
        l2 = [fake, fake, fake]
        l2[missing] = None
        assert _call(f, [None, None, None], 0, l2, 4) == BAD_ARGS


def test_missing_prefix_work_list_is_rejected():
    f = _fn()
    fake = ctypes.c_void_p(256)
    for missing in range(3):
        l1 = [fake, fake, fake]
        l1[missing] = None
        assert _call(f, l1, 2, [fake, fake, fake], 4) == BAD_ARGS
