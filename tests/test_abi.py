"""C ABI checks that need no GPU: the library loads, exports every entry
point include/rl_sampler.h declares, and rejects bad arguments with a status
and a message instead of crashing."""
import ctypes

import pytest

import rlsampler


def test_library_exports_every_declared_symbol():
    L = rlsampler.lib()
    declared = rlsampler.declared_symbols()
    assert len(declared) >= 10
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing


def test_version_string():
    assert b"sm_100a" in rlsampler.lib().rl_version()


def test_create_rejects_null_and_bad_limits():
    L = rlsampler.lib()
    assert L.rl_sampler_create(None, 0, 1, 1, 0, 0) == rlsampler.RL_ERR_INVALID_ARG
    assert "NULL" in rlsampler.last_error()
    h = ctypes.c_void_p()
    assert L.rl_sampler_create(ctypes.byref(h), 0, 0, 10, 0, 0) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_sampler_create(ctypes.byref(h), 0, 1, 10, 4096, 0) == rlsampler.RL_ERR_SHAPE
    assert not h.value


def test_null_handle_is_an_error_not_a_crash():
    L = rlsampler.lib()
    st = L.rl_sample_batch(None, None, 0, 1, 10, 10, None, None, 0, None, 0, None, None, None, None,
                           None, None)
    assert st == rlsampler.RL_ERR_INVALID_ARG
    assert "handle" in rlsampler.last_error()
    assert L.rl_sampler_destroy(None) == rlsampler.RL_OK


def test_create_without_device_reports_cuda_error():
    from conftest import HAS_GPU

    if HAS_GPU:
        pytest.skip("a device is present")
    h = ctypes.c_void_p()
    st = rlsampler.lib().rl_sampler_create(ctypes.byref(h), 0, 4, 1000, 16, 0)
    assert st in (rlsampler.RL_ERR_CUDA, rlsampler.RL_ERR_INVALID_ARG)
    assert rlsampler.last_error()


def test_error_message_is_thread_local():
    import threading

    L = rlsampler.lib()
    L.rl_sampler_create(None, 0, 1, 1, 0, 0)
    seen = {}

    def other():
        seen["msg"] = rlsampler.last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""
    assert rlsampler.last_error() != ""
