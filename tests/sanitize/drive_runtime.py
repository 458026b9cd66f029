"""Drives the C++ runtime module built with -fsanitize=address,undefined (directory in
argv[1]): random block-manager operations (allocate / append / fork / free, slot and
block-table queries), malformed IPC frames, and every truncation of a GGUF header.
Any sanitizer report aborts the process (non-zero exit)."""
import importlib.util
import os
import random
import sys

import numpy as np

D = sys.argv[1]
spec = importlib.util.spec_from_file_location("_rt", os.path.join(D, [f for f in os.listdir(D) if f.startswith("_rt.")][0]))
rt = importlib.util.module_from_spec(spec); spec.loader.exec_module(rt)
bm = rt.BlockManager(64, 16, True)
rng = random.Random(0)
live = {}
for it in range(2000):
    op = rng.random()
    if op < 0.4 and len(live) < 8:
        sid = it; toks = [rng.randrange(50) for _ in range(rng.randrange(1, 120))]
        if bm.can_allocate(len(toks) + 1):
            bm.allocate(sid, toks); live[sid] = len(toks)
    elif op < 0.7 and live:
        sid = rng.choice(list(live))
        if bm.can_append(sid, 1):
            bm.append(sid, [rng.randrange(50)]); live[sid] += 1
            bm.slots(sid, 0, live[sid])
            out = np.zeros(live[sid], dtype=np.int32)
    elif op < 0.8 and live:
        sid = rng.choice(list(live)); child = 100000 + it
        try:
            bm.fork(sid, child); live[child] = live[sid]
        except Exception:
            pass
    elif live:
        sid = rng.choice(list(live)); bm.free(sid); del live[sid]
    if live:
        sids = list(live)
        bt = np.zeros((len(sids), 16), dtype=np.int32)
        try:
            bm.fill_block_tables(sids, bt)
        except Exception:
            pass
        p = np.array([live[s] - 1 for s in sids], dtype=np.int32); o = np.zeros(len(sids), dtype=np.int32)
        bm.decode_slots(sids, p, o)
# malformed / random IPC input
for n in range(300):
    blob = bytes(rng.randrange(256) for _ in range(rng.randrange(0, 80)))
    for f in (rt.decode_task, rt.decode_result):
        try: f(blob)
        except Exception: pass
    d = rt.GatewayDecoder(1024)
    d.feed(blob)
    try: d.next()
    except Exception: pass
g = rt.encode_gateway(1, "sess", False, b"hello")
d = rt.GatewayDecoder(1024); d.feed(g); print("gateway", d.next() is not None)
# GGUF: a valid file, then every truncation of its header
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from openmini_v1_b200.gguf.writer import GGUFWriter
w = GGUFWriter(os.path.join(D, "t.gguf"), "llama"); w.add_kv("llama.block_count", 2); w.add_tensor("a", np.ones((4, 32), np.float32)); w.write()
rt.parse_gguf(os.path.join(D, "t.gguf"))
data = open(os.path.join(D, "t.gguf"), "rb").read()
bad = 0
for cut in range(0, min(len(data), 400), 3):
    open(os.path.join(D, "c.gguf"), "wb").write(data[:cut])
    try: rt.parse_gguf(os.path.join(D, "c.gguf"))
    except Exception: bad += 1
print("ok", bad)
