"""Out-of-process encoder transport: a persistent ``exl3b_vit serve`` child
on a framed stdin/stdout protocol (the reference's "proc" transport,
quantize.py:441-608, over viterbi_esimd.cpp:683-733).

The child gets XTQ_VIT_DEVIDX in its environment, so it can encode on a
different GPU than the parent process uses.  Frames (little endian):
request "<IIiiQQ16s" = magic, op (0 quit / 1 run), margin, pivot, nseq,
xbytes, code; then fp32 X [nseq][256].  Reply "<IiQ" = magic, rc, nbytes;
then int32 states [nseq][256] when rc == 0.

Env: XTQ_VIT_BIN (worker path; default exl3b/exl3b_vit next to the library),
XTQ_VIT_DEVIDX (device of the child), XTQ_VIT_MAXSEQ (sequences per frame,
default 1024)."""
from __future__ import annotations

import atexit
import os
import struct
import subprocess

import numpy as np
import torch

SERVE_MAGIC = 0x58545156
REQ = struct.Struct("<IIiiQQ16s")
REP = struct.Struct("<IiQ")
CODES = {"exl3_mul1": "mul1p"}


def worker_path() -> str:
    return os.environ.get("XTQ_VIT_BIN") or os.path.join(
        os.path.dirname(os.path.abspath(__file__)), "exl3b_vit")


class ServeError(RuntimeError):
    pass


class ServeWorker:
    """One ``exl3b_vit serve`` child process."""

    def __init__(self, devidx: int | None = None, binary: str | None = None):
        env = dict(os.environ)
        if devidx is not None:
            env["XTQ_VIT_DEVIDX"] = str(int(devidx))
        path = binary or worker_path()
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path}: worker not built (run csrc/build.py)")
        self.proc = subprocess.Popen([path, "serve"], stdin=subprocess.PIPE,
                                     stdout=subprocess.PIPE, env=env, bufsize=0)
        atexit.register(self.close)

    def _read(self, n: int) -> bytes:
        buf = bytearray()
        fd = self.proc.stdout.fileno()
        while len(buf) < n:
            chunk = os.read(fd, n - len(buf))
            if not chunk:
                raise ServeError("exl3b_vit worker closed its stdout")
            buf += chunk
        return bytes(buf)

    def _write(self, data) -> None:
        mv = memoryview(data).cast("B")
        fd = self.proc.stdin.fileno()
        off = 0
        while off < len(mv):
            off += os.write(fd, mv[off:])

    def request(self, op: int, margin: int, pivot: int, nseq: int, xbytes: int,
                code: str, payload=None) -> tuple[int, bytes]:
        """Send one raw frame (+ payload); returns (rc, reply bytes)."""
        self._write(REQ.pack(SERVE_MAGIC, op, margin, pivot, nseq, xbytes,
                             code.encode().ljust(16, b"\0")[:16]))
        if payload is not None:
            self._write(payload)
        magic, rc, nbytes = REP.unpack(self._read(REP.size))
        if magic != SERVE_MAGIC:
            raise ServeError(f"exl3b_vit serve: bad reply magic {magic:#x}")
        return rc, (self._read(nbytes) if nbytes else b"")

    def run(self, x: np.ndarray, code: str = "mul1p", margin: int = 0,
            pivot: int = 128) -> np.ndarray:
        """x [nseq][256] fp32 -> states [nseq][256] int32."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        nseq = x.shape[0]
        assert x.shape == (nseq, 256)
        rc, data = self.request(1, margin, pivot, nseq, x.nbytes, code, x)
        if rc:
            raise ServeError(f"exl3b_vit serve rc={rc}")
        if len(data) != nseq * 256 * 4:
            raise ServeError(f"exl3b_vit serve nbytes={len(data)} want={nseq * 1024}")
        return np.frombuffer(data, dtype=np.int32).reshape(nseq, 256).copy()

    def close(self) -> int | None:
        p = self.proc
        if p.poll() is None:
            try:
                self._write(REQ.pack(SERVE_MAGIC, 0, 0, 0, 0, 0, b"\0" * 16))
                p.stdin.close()
            except OSError:
                pass
            try:
                p.wait(timeout=30)
            except subprocess.TimeoutExpired:
                p.kill()
                p.wait()
        return p.returncode


_WORKER: ServeWorker | None = None


def _worker() -> ServeWorker:
    global _WORKER
    if _WORKER is None or _WORKER.proc.poll() is not None:
        dev = os.environ.get("XTQ_VIT_DEVIDX")
        _WORKER = ServeWorker(int(dev) if dev is not None else None)
    return _WORKER


def tailbite_proc(X: torch.Tensor, code: str = "exl3_mul1", K: int = 4, L: int = 16,
                  V: int = 1, pivot: int | None = None, margin: int = 0) -> torch.Tensor:
    """quantize.py:611-628 over the worker: X [256, nseq] fp32 -> states
    [256, nseq] int64, bit-exact with quantize_seq_tailbite(pivot, margin).
    The worker protocol carries the reference's K = 4 mul1 kernel."""
    kcode = CODES.get(code)
    if kcode is None or K != 4 or L != 16 or V != 1:
        raise ValueError(f"the worker transport encodes code exl3_mul1 at K=4, L=16, V=1; "
                         f"got {code!r} K={K} L={L} V={V}")
    T, nseq = X.shape
    if T != 256:
        raise ValueError(f"256-target sequences expected, got T={T}")
    pv = T // 2 if pivot is None else int(pivot)
    x = np.ascontiguousarray(X.detach().t().cpu().numpy(), dtype=np.float32)
    st = np.empty((nseq, T), dtype=np.int32)
    chunk = int(os.environ.get("XTQ_VIT_MAXSEQ", "1024"))
    w = _worker()
    for s0 in range(0, nseq, chunk):
        s1 = min(nseq, s0 + chunk)
        st[s0:s1] = w.run(x[s0:s1], kcode, margin, pv)
    return torch.from_numpy(st).t().contiguous().long()
