"""The expert-parallel layer's bounded host wait (jt_watchdog.c), on the CPU.

jt_b200_watchdog_selftest runs the same polling loop the forward uses for
the gathered expert counts, against fake operations: a completion after a
few polls, an asynchronous error reported by the communicator, and nothing
at all (the deadline passes).  On an error or a timeout the loop must abort
the communicator; on completion it must not.
"""
import ctypes as C
import time

from jimotono_b200 import lib


def _run(scenario, timeout_ms):
    aborted = C.c_int(-1)
    t0 = time.perf_counter()
    rc = lib().jt_b200_watchdog_selftest(scenario, timeout_ms, C.byref(aborted))
    return rc, aborted.value, time.perf_counter() - t0


def test_completion_is_not_aborted():
    rc, aborted, dt = _run(0, 10_000)
    assert (rc, aborted) == (0, 0)
    assert dt < 1.0


def test_async_error_aborts_before_the_deadline():
    rc, aborted, dt = _run(1, 10_000)
    assert (rc, aborted) == (1, 1)
    assert dt < 1.0


def test_deadline_aborts():
    rc, aborted, dt = _run(2, 200)
    assert (rc, aborted) == (2, 1)
    assert 0.2 <= dt < 5.0


def test_bad_arguments():
    assert lib().jt_b200_watchdog_selftest(3, 10, C.byref(C.c_int())) != 0
    assert lib().jt_b200_watchdog_selftest(0, 10, None) != 0
