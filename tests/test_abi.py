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


def test_every_handle_entry_rejects_a_null_handle():
    """Each entry that takes a handle answers a NULL handle with
    RL_ERR_INVALID_ARG and a message, before touching any device."""
    L = rlsampler.lib()
    P = None
    calls = {
        "rl_decoder_sample": lambda: L.rl_decoder_sample(P, P, 1, 10, 10, P, P, P, P, P, P),
        "rl_decoder_sample_host": lambda: L.rl_decoder_sample_host(P, P, 1, 10, P, P, P, P, P),
        "rl_greedy_host": lambda: L.rl_greedy_host(P, P, 1, 10, P),
        "rl_grammar_greedy_host": lambda: L.rl_grammar_greedy_host(P, P, 1, 10, P, 1, P),
        "rl_specdec_sample": lambda: L.rl_specdec_sample(P, P, 1, 10, 10, P, P, P, P, P),
        "rl_specdec_verify": lambda: L.rl_specdec_verify(P, P, 1, 10, 10, P, 4, P, P, P, P, P, P, P),
        "rl_sample_sharded": lambda: L.rl_sample_sharded(P, P, P, 0, 1, 10, 10, 0, 10, P, P, 0, P, 0, P, P, P, P,
                                                         P, P),
        "rl_sampler_set_debug": lambda: L.rl_sampler_set_debug(P, 0),
        "rl_lmhead_logits": lambda: L.rl_lmhead_logits(P, P, 64, P, 64, 1, 64, 10, P, 0, 10, P),
        "rl_lmhead_greedy": lambda: L.rl_lmhead_greedy(P, P, 64, P, 64, 1, 64, 10, P, P, P, 10, P),
        "rl_lmhead_sample": lambda: L.rl_lmhead_sample(P, P, 64, P, 64, 1, 64, 10, P, P, 0, P, P, P, P, P, P),
    }
    for name, call in calls.items():
        st = call()
        assert st == rlsampler.RL_ERR_INVALID_ARG, (name, st)
        assert rlsampler.last_error(), name


def test_selfcheck_and_nccl_helpers_reject_bad_arguments():
    L = rlsampler.lib()
    assert L.rl_selfcheck_div(None, -1, None, 1, None, None, None) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_selfcheck_div(None, 0, None, 0, None, None, None) == rlsampler.RL_OK  # nothing to do
    assert L.rl_nccl_unique_id(None) == rlsampler.RL_ERR_INVALID_ARG
    comm = ctypes.c_void_p()
    uid = (ctypes.c_char * rlsampler.NCCL_ID_BYTES)()
    assert L.rl_nccl_comm_init(ctypes.byref(comm), 2, uid, 5) == rlsampler.RL_ERR_INVALID_ARG  # rank >= nranks
    assert L.rl_nccl_comm_init(None, 1, uid, 0) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_nccl_comm_destroy(None) == rlsampler.RL_OK


def test_gbnf_entries_reject_null_arguments():
    """The grammar entries are host-only: their argument checks need no GPU."""
    L = rlsampler.lib()
    P = None
    out = ctypes.c_void_p()
    assert L.rl_gbnf_create(b"root ::= \"a\"", b"root", 1, P, P, -1, ctypes.byref(out)) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_gbnf_state_create(P, ctypes.byref(out)) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_gbnf_mask(P, P, P, 1, P) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_gbnf_accept(P, P, 0) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_gbnf_mask_batch(P, P, 1, P, 1, P, 1) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_gbnf_accept_batch(P, P, P, 1, P, 1) == rlsampler.RL_ERR_INVALID_ARG
    assert L.rl_gbnf_accepting(P) == 0
    assert rlsampler.last_error()
