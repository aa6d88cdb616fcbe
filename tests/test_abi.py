"""The C ABI library: it loads without a GPU, exports every function that
include/tgsample.h declares, and its host-side checks reject bad arguments with
status codes (no GPU work is started by these calls)."""
import ctypes
import os
import re

from tinygpt_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "tgsample.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int32_t|const char\*)\s+(tg_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol(cuda_lib):
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(cuda_lib, n), f"{n} declared in tgsample.h but not exported"
    assert set(_lib.EXPORTED) <= set(names)


def test_abi_version_and_errors_without_device(cuda_lib):
    assert cuda_lib.tg_abi_version() >> 16 == 1
    h = ctypes.c_void_p()
    rc = cuda_lib.tg_sampler_create(0, 0, 16, ctypes.byref(h))
    assert rc == _lib.TG_ERR_UNSUPPORTED and b"vocab" in cuda_lib.tg_last_error_string()
    rc = cuda_lib.tg_sampler_create(0, 1000, 0, ctypes.byref(h))
    assert rc == _lib.TG_ERR_INVALID_ARG
    rc = cuda_lib.tg_sampler_create(0, 1000, 16, None)
    assert rc == _lib.TG_ERR_INVALID_ARG
    rc = cuda_lib.tg_sample(None, None, 0, 0, 1, None, None, None, 0, None, 0, None, None, None,
                            None, None)
    assert rc == _lib.TG_ERR_INVALID_ARG and b"sampler is NULL" in cuda_lib.tg_last_error_string()
    rc = cuda_lib.tg_spec_verify_static(0, 100, None, None, 7, 1, 1, None, None, None, None, None,
                                        None, None)
    assert rc == _lib.TG_ERR_INVALID_ARG
    rc = cuda_lib.tg_spec_verify_masked(None, None, None, 0, 1, 1, None, None, None, None, None, 1, None,
                                        None, None, None)
    assert rc == _lib.TG_ERR_INVALID_ARG
    rc = cuda_lib.tg_sample_sharded(None, None, 1, 0, 100, None, 0, 100, 1, None, None, None, 0, None, 0,
                                    None, None, None, None, None)
    assert rc == _lib.TG_ERR_INVALID_ARG and b"sampler is NULL" in cuda_lib.tg_last_error_string()


def test_row_params_layout():
    from tinygpt_b200.sampler import row_params
    p = row_params(3, temperature=0.5, top_k=None, top_p=0.9)
    assert p.dtype.itemsize == 32
    assert list(p.dtype.names) == ["temperature", "top_p", "min_p", "repetition_penalty",
                                   "presence_penalty", "frequency_penalty", "top_k", "flags"]
    assert (p["top_k"] == 0).all() and (p["temperature"] == 0.5).all()
