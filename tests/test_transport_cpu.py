"""The exl3b_vit serve worker's framing and error behaviour (the reference's
viterbi_esimd serve loop, viterbi_esimd.cpp:683-733), exercised without a
GPU: malformed requests answer rc 7 and the worker keeps serving, a bad magic
ends it with status 1, quit and EOF end it with 0."""
import os
import subprocess

import numpy as np
import pytest

from exl3b import transport as tp


@pytest.fixture()
def worker():
    if not os.path.exists(tp.worker_path()):
        pytest.skip("exl3b_vit not built")
    w = tp.ServeWorker()
    yield w
    w.close()


def test_malformed_requests_answer_rc7(worker):
    # op other than 0 / 1
    assert worker.request(2, 0, 0, 1, 1024, "mul1p") == (7, b"")
    # xbytes != nseq * 256 * 4
    assert worker.request(1, 0, 0, 2, 1024, "mul1p") == (7, b"")
    # nseq over 2^22
    assert worker.request(1, 0, 0, (1 << 22) + 1, ((1 << 22) + 1) * 1024, "mul1p") == (7, b"")
    # a well-formed request with an unsupported code fails inside xtq_vit_run
    # (no device here: rc 1; with one: rc 7) and the worker keeps serving
    x = np.zeros((3, 256), np.float32)
    rc, data = worker.request(1, 0, 0, 3, x.nbytes, "ih2x2", x)
    assert rc in (1, 7) and data == b""
    assert worker.request(2, 0, 0, 0, 0, "mul1p") == (7, b"")
    assert worker.close() == 0


def test_bad_magic_and_eof_end_the_worker():
    if not os.path.exists(tp.worker_path()):
        pytest.skip("exl3b_vit not built")
    frame = tp.REQ.pack(0x1234, 1, 0, 0, 0, 0, b"mul1p".ljust(16, b"\0"))
    r = subprocess.run([tp.worker_path(), "serve"], input=frame, capture_output=True,
                       timeout=60)
    assert r.returncode == 1 and r.stdout == b"" and b"frame magic" in r.stderr
    r = subprocess.run([tp.worker_path(), "serve"], input=b"", capture_output=True, timeout=60)
    assert r.returncode == 0 and r.stdout == b""
    # quit frame
    quit_ = tp.REQ.pack(tp.SERVE_MAGIC, 0, 0, 0, 0, 0, b"\0" * 16)
    r = subprocess.run([tp.worker_path(), "serve"], input=quit_, capture_output=True,
                       timeout=60)
    assert r.returncode == 0 and r.stdout == b""


def test_transport_argument_checks():
    import torch
    with pytest.raises(ValueError, match="K=4"):
        tp.tailbite_proc(torch.zeros(256, 2), K=5)
    with pytest.raises(ValueError, match="256-target"):
        tp.tailbite_proc(torch.zeros(128, 2))
