"""The tensor-parallel host wait (llm-accel_b200/csrc/stream_watch.h) on the CPU.

A rank whose stream can hold NCCL collectives waits by polling the stream, the
communicator's asynchronous error and a deadline; on an error or expiry it
aborts the communicator (ncclCommAbort), which ends the NCCL kernels, instead of
blocking for good in cudaStreamSynchronize.  The loop is compiled here against
fakes of the stream query, the asynchronous-error query, the abort and the
clock, so every outcome is exercised without a GPU and without an NCCL kernel
left waiting on a missing peer.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "llm-accel_b200", "csrc")

HARNESS = r"""
#include <cstdio>
#include "stream_watch.h"
using namespace llmx;

// pending: polls until the stream reports idle (-1 = never); stream_err: the
// poll at which the stream reports a CUDA error (-1 = never); comm_err: the poll
// at which the communicator reports an asynchronous error (-1 = never); each
// poll advances the fake clock by step_ms.
static void run(const char *name, int pending, int stream_err, int comm_err, double step_ms, double timeout_ms) {
    int polls = 0, aborts = 0, comm_checks = 0;
    double clock = 0.0;
    const WatchOutcome w = watch_stream(
        [&] {
            const int n = polls++;
            clock += step_ms;
            if (stream_err >= 0 && n >= stream_err) return -1;
            return pending >= 0 && n >= pending ? 0 : 1;
        },
        [&] { return comm_err >= 0 && comm_checks++ >= comm_err; },
        [&] { aborts++; },
        [&] { return clock; },
        timeout_ms);
    std::printf("%s %d %d %d\n", name, (int)w, aborts, polls);
}

int main() {
    run("idle", 0, -1, -1, 0.001, 1000.0);
    run("finishes", 5000, -1, -1, 0.001, 1000.0);
    run("stream_error", -1, 7, -1, 0.001, 1000.0);
    run("comm_error", -1, -1, 3, 0.001, 1000.0);
    run("timeout", -1, -1, -1, 1.0, 50.0);
    run("finishes_before_deadline", 40, -1, -1, 1.0, 50.0);
    return 0;
}
"""


@pytest.fixture(scope="module")
def outcomes(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if not cxx:
        pytest.skip("no C++ compiler")
    d = tmp_path_factory.mktemp("watch")
    src, exe = d / "watch.cpp", d / "watch"
    src.write_text(HARNESS)
    subprocess.run([cxx, "-std=c++17", "-O1", "-I", CSRC, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    res = {}
    for line in out.split("\n"):
        if line.strip():
            name, w, aborts, polls = line.split()
            res[name] = (int(w), int(aborts), int(polls))
    return res


DONE, STREAM_ERROR, COMM_ERROR, TIMEOUT = 0, 1, 2, 3


def test_idle_stream_returns_at_once(outcomes):
    assert outcomes["idle"] == (DONE, 0, 1)


def test_pending_work_is_waited_for_without_abort(outcomes):
    assert outcomes["finishes"] == (DONE, 0, 5001)
    assert outcomes["finishes_before_deadline"] == (DONE, 0, 41)


def test_stream_error_is_reported_without_abort(outcomes):
    # a CUDA fault is the context's own error: the communicator is left alone
    assert outcomes["stream_error"] == (STREAM_ERROR, 0, 8)


def test_async_comm_error_aborts_once(outcomes):
    assert outcomes["comm_error"] == (COMM_ERROR, 1, 4)


def test_deadline_aborts_once(outcomes):
    w, aborts, polls = outcomes["timeout"]
    assert (w, aborts) == (TIMEOUT, 1)
    assert 50 <= polls <= 52  # one poll per fake millisecond until the deadline


def test_runtime_routes_collective_waits_through_the_watch():
    """Every host wait of the runtime goes through stream_wait (the watched wait
    while NCCL collectives can be pending), except the best-effort drain at
    release and llmx_time_kernel, which times single kernels and enqueues no
    collective."""
    src = open(os.path.join(CSRC, "runtime.cu")).read()
    body = src.split("int stream_wait(llmx_ctx *c) {", 1)[1]
    assert "ncclCommAbort" in body.split("\n}\n", 1)[0]
    plain = [ln for ln in src.split("\n") if "cudaStreamSynchronize(c->stream)" in ln]
    # inside stream_wait (no collective possible), release(), llmx_time_kernel
    assert len(plain) == 3, plain
