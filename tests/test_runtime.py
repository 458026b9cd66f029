"""C++ runtime: block manager (alloc / append / COW fork / prefix cache / LRU),
worker and gateway framing, GGUF index parsing."""
import struct

import numpy as np
import pytest

from openmini_v1_b200 import _native

rt = _native.rt()


def test_block_manager_alloc_append_free():
    bm = rt.BlockManager(8, 16, False)
    assert bm.allocate(1, list(range(20))) == 0
    assert bm.num_free() == 6
    assert bm.slots(1, 0, 2) == [bm.block_table(1)[0] * 16, bm.block_table(1)[0] * 16 + 1]
    bm.append(1, list(range(12)))
    assert bm.seq_len(1) == 32 and len(bm.block_table(1)) == 2
    bm.append(1, [7])
    assert len(bm.block_table(1)) == 3
    bm.free(1)
    assert bm.num_free() == 8
    with pytest.raises(RuntimeError):
        bm.allocate(2, list(range(16 * 9)))


def test_fork_copy_on_write():
    bm = rt.BlockManager(8, 16, False)
    bm.allocate(1, list(range(20)))
    bm.fork(1, 2)
    last = bm.block_table(1)[1]
    assert bm.ref_count(last) == 2
    cow = bm.append(2, [99])
    assert cow and cow[0][0] == last
    assert bm.block_table(2)[1] != last and bm.ref_count(last) == 1


def test_prefix_cache_hit_and_lru():
    bm = rt.BlockManager(6, 16, True)
    toks = list(range(40))
    assert bm.allocate(1, toks) == 0
    bm.free(1)
    assert bm.allocate(2, toks) == 32          # two full blocks reused
    assert bm.prefix_hit_rate() > 0
    bm.free(2)
    assert bm.allocate(3, [5] * 90) == 0       # evicts cached blocks under pressure
    fill = np.zeros((1, 8), dtype=np.int32)
    bm.fill_block_tables([3], fill)
    assert list(fill[0, :6]) == bm.block_table(3)


def test_reserve_then_append():
    bm = rt.BlockManager(8, 16, False)
    bm.allocate(1, list(range(15)))
    bm.reserve(1, 20)
    assert len(bm.block_table(1)) == 3
    bm.append(1, list(range(20)))
    assert len(bm.block_table(1)) == 3


def test_worker_framing_roundtrip():
    t = rt.encode_task(12345, b"hello")
    assert t[:8] == struct.pack("<Q", 12345) and t[8:12] == struct.pack("<I", 5)
    assert rt.decode_task(t) == (12345, b"hello")
    r = rt.encode_result(7, True, b"xy")
    assert rt.decode_result(r) == (7, True, b"xy")
    with pytest.raises(ValueError):
        rt.decode_task(struct.pack("<QI", 1, 1000))
    assert rt.encode_command(rt.WORKER_CMD_HEARTBEAT) == b"\x03"
    assert rt.encode_command(rt.WORKER_CMD_TASK, b"ab") == b"\x01" + struct.pack("<I", 2) + b"ab"


def test_gateway_decoder_incremental():
    f = rt.encode_gateway(1, "s" * 36, True, b"prompt text")
    d = rt.GatewayDecoder()
    d.feed(f[:10])
    assert d.next() is None
    d.feed(f[10:] + rt.encode_gateway(4, "h", False, b""))
    typ, sid, stream, payload = d.next()
    assert (typ, sid, stream, payload) == (1, "s" * 36, True, b"prompt text")
    assert d.next()[0] == 4
    big = rt.GatewayDecoder(16)
    big.feed(struct.pack(">I", 100))
    with pytest.raises(ValueError):
        big.next()


def test_gguf_index(tmp_path):
    from openmini_v1_b200.gguf.writer import GGUFWriter
    p = tmp_path / "m.gguf"
    w = GGUFWriter(str(p), "llama")
    w.add_kv("llama.block_count", 2)
    w.add_kv("general.name", "t")
    w.add_kv("tokenizer.ggml.tokens", ["a", "b"])
    w.add_tensor("x", np.arange(64, dtype=np.float32).reshape(2, 32))
    w.write()
    info = rt.parse_gguf(str(p))
    assert info["metadata"]["llama.block_count"] == 2
    assert info["metadata"]["tokenizer.ggml.tokens"] == ["a", "b"]
    name, dims, typ, off = info["tensors"][0]
    assert name == "x" and dims == [32, 2] and typ == 0
