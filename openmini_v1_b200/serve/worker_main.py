"""Worker process entry: ``python -m openmini_v1_b200.serve.worker_main module:function``.

Reads command bytes from stdin (1 TASK + length-prefixed Task, 2 SHUTDOWN,
3 HEARTBEAT -> echoes 0x03, 4 LOAD_MODEL + length-prefixed model path) and
writes length-prefixed TaskResult frames to stdout. ``function(bytes) -> bytes``
handles a task; an exception becomes a failed result carrying the message.
Restates openmini-server/src/service/worker/worker.rs:178-283.
"""
from __future__ import annotations

import importlib
import struct
import sys


def _read_exact(f, n):
    buf = b""
    while len(buf) < n:
        chunk = f.read(n - len(buf))
        if not chunk:
            raise EOFError
        buf += chunk
    return buf


def echo_handler(data: bytes) -> bytes:
    """Default handler: returns the payload (used by tests and health probes)."""
    return data


def main(argv=None):
    argv = argv or sys.argv[1:]
    spec = argv[0] if argv else "openmini_v1_b200.serve.worker_main:echo_handler"
    mod, fn = spec.split(":")
    handler = getattr(importlib.import_module(mod), fn)
    from openmini_v1_b200 import _native
    rt = _native.rt()
    inp, out = sys.stdin.buffer, sys.stdout.buffer
    while True:
        try:
            cmd = _read_exact(inp, 1)[0]
        except EOFError:
            return 0
        if cmd == rt.WORKER_CMD_SHUTDOWN:
            return 0
        if cmd == rt.WORKER_CMD_HEARTBEAT:
            out.write(b"\x03")
            out.flush()
            continue
        n = struct.unpack("<I", _read_exact(inp, 4))[0]
        payload = _read_exact(inp, n)
        if cmd == rt.WORKER_CMD_LOAD_MODEL:
            continue
        if cmd != rt.WORKER_CMD_TASK:
            continue
        tid, data = rt.decode_task(payload)
        try:
            res, ok = handler(data), True
        except Exception as e:  # report, keep serving
            res, ok = f"{type(e).__name__}: {e}".encode(), False
        out.write(rt.encode_length_prefixed(rt.encode_result(tid, ok, res)))
        out.flush()


def crash_handler(data: bytes) -> bytes:
    """Test handler: exits the process when the payload is b"crash"."""
    if data == b"crash":
        import os
        os._exit(3)
    return data.upper()


if __name__ == "__main__":
    sys.exit(main())
