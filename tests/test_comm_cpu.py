"""The communicator's host watchdog (bwpp_cuda_comm_watch), on CPU, driven by
a fake communicator: Python callbacks stand in for the last collective's CUDA
event, NCCL's asynchronous error state and ncclCommAbort.  The same function,
with the CUDA / NCCL callbacks, bounds every wait of the tiny_model step's
gradient allreduce (no reference counterpart: the reference has no
distributed code)."""
import ctypes as C
import time

import pytest

import bwpp

DONE = C.CFUNCTYPE(C.c_int, C.c_void_p)
ERR = C.CFUNCTYPE(C.c_int, C.c_void_p)
ABORT = C.CFUNCTYPE(None, C.c_void_p)


class FakeComm:
    """done_after: polls until the collective finishes (None: never);
    error_after: polls until NCCL reports an async error (None: never);
    in_progress: polls during which the error state reads "in progress"."""

    def __init__(self, done_after=0, error_after=None, in_progress=0, cuda_error=False):
        self.done_after, self.error_after, self.in_progress = done_after, error_after, in_progress
        self.cuda_error = cuda_error
        self.polls = self.err_polls = self.aborts = 0
        self.done_cb = DONE(self._done)
        self.err_cb = ERR(self._err)
        self.abort_cb = ABORT(self._abort)

    def _done(self, _):
        self.polls += 1
        if self.cuda_error:
            return -1
        return 1 if self.done_after is not None and self.polls > self.done_after else 0

    def _err(self, _):
        self.err_polls += 1
        if self.error_after is not None and self.err_polls > self.error_after:
            return 2
        return 1 if self.err_polls <= self.in_progress else 0

    def _abort(self, _):
        self.aborts += 1

    def watch(self, timeout_ms):
        lib = bwpp.load()
        t0 = time.perf_counter()
        rc = lib.bwpp_cuda_comm_watch(C.cast(self.done_cb, C.c_void_p), C.cast(self.err_cb, C.c_void_p),
                                      C.cast(self.abort_cb, C.c_void_p), None, timeout_ms)
        return rc, time.perf_counter() - t0


def test_finished_collective_returns_at_once():
    f = FakeComm(done_after=0)
    rc, dt = f.watch(1000)
    assert rc == bwpp.OK and f.aborts == 0 and dt < 0.5


def test_collective_that_finishes_later():
    f = FakeComm(done_after=20, in_progress=5)
    rc, _ = f.watch(2000)
    assert rc == bwpp.OK and f.aborts == 0 and f.polls == 21


def test_peer_that_never_joins_times_out_and_aborts_once():
    f = FakeComm(done_after=None)
    rc, dt = f.watch(300)
    assert rc == bwpp.ERR_TIMEOUT
    assert f.aborts == 1
    assert 0.3 <= dt < 1.5  # the bound holds (polls back off to 160 us, no more)


def test_async_nccl_error_aborts():
    f = FakeComm(done_after=None, error_after=3)
    rc, dt = f.watch(5000)
    assert rc == bwpp.ERR and f.aborts == 1 and dt < 1.0


def test_cuda_error_on_the_event_aborts():
    f = FakeComm(cuda_error=True)
    rc, _ = f.watch(1000)
    assert rc == bwpp.ERR_CUDA and f.aborts == 1


def test_watch_without_error_callback_and_bad_arguments():
    lib = bwpp.load()
    f = FakeComm(done_after=2)
    rc = lib.bwpp_cuda_comm_watch(C.cast(f.done_cb, C.c_void_p), None, C.cast(f.abort_cb, C.c_void_p),
                                  None, 1000)
    assert rc == bwpp.OK
    assert lib.bwpp_cuda_comm_watch(None, None, C.cast(f.abort_cb, C.c_void_p), None, 10) == bwpp.ERR_ARG
    assert lib.bwpp_cuda_comm_watch(C.cast(f.done_cb, C.c_void_p), None, None, None, 10) == bwpp.ERR_ARG
