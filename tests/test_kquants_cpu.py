"""GGUF block formats beyond Q4_0 / Q4_1 / Q8_0 / Q4_K: the vectorised readers
against element-by-element statements of the specification on random blocks,
and quantise -> dequantise round trips."""
import struct

import numpy as np
import pytest

from openmini_v1_b200.gguf import kquants as k
from openmini_v1_b200.gguf.constants import BLOCK_SIZES, GGMLType
from openmini_v1_b200.gguf.quants import dequantize


def _rand_blocks(nblk, nbytes, seed, f16_at=(), f32_at=()):
    rng = np.random.default_rng(seed)
    b = rng.integers(0, 256, size=(nblk, nbytes), dtype=np.uint8)
    for off in f16_at:  # keep scales finite and moderate
        b[:, off:off + 2] = np.frombuffer(
            rng.uniform(-0.1, 0.1, nblk).astype(np.float16).tobytes(), np.uint8).reshape(nblk, 2)
    for off in f32_at:
        b[:, off:off + 4] = np.frombuffer(
            rng.uniform(-0.1, 0.1, nblk).astype(np.float32).tobytes(), np.uint8).reshape(nblk, 4)
    return b


def _by(x):
    return np.asarray(x).astype(np.uint8).tobytes()


def _h(b, o):
    return float(np.frombuffer(_by(b[o:o + 2]), np.float16)[0])


def _scalar_q6k(blk):
    ql, qh, sc, d = blk[0:128], blk[128:192], np.frombuffer(_by(blk[192:208]), np.int8), _h(blk, 208)
    out = np.zeros(256, np.float32)
    for half in range(2):
        L, H, S = ql[64 * half:], qh[32 * half:], sc[8 * half:]
        for l in range(32):
            i = l // 16
            q1 = ((L[l] & 15) | (((H[l] >> 0) & 3) << 4)) - 32
            q2 = ((L[l + 32] & 15) | (((H[l] >> 2) & 3) << 4)) - 32
            q3 = ((L[l] >> 4) | (((H[l] >> 4) & 3) << 4)) - 32
            q4 = ((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32
            base = 128 * half
            out[base + l] = d * S[i] * q1
            out[base + l + 32] = d * S[i + 2] * q2
            out[base + l + 64] = d * S[i + 4] * q3
            out[base + l + 96] = d * S[i + 6] * q4
    return out


def _scalar_q2k(blk):
    sc, q, d, dm = blk[0:16], blk[16:80], _h(blk, 80), _h(blk, 82)
    out, e, g = np.zeros(256, np.float32), 0, 0
    for half in range(2):
        Q = q[32 * half:]
        for shift in (0, 2, 4, 6):
            for part in range(2):
                s = sc[g]
                g += 1
                for l in range(16):
                    out[e] = d * (s & 15) * ((Q[l + 16 * part] >> shift) & 3) - dm * (s >> 4)
                    e += 1
    return out


def _scalar_q3k(blk):
    hm, q, s12, d = blk[0:32], blk[32:96], blk[96:108], _h(blk, 108)
    a0, a1, tmp = struct.unpack("<III", _by(s12))
    m2, m1 = 0x0F0F0F0F, 0x03030303
    aux = [(a0 & m2) | (((tmp >> 0) & m1) << 4), (a1 & m2) | (((tmp >> 2) & m1) << 4),
           ((a0 >> 4) & m2) | (((tmp >> 4) & m1) << 4), ((a1 >> 4) & m2) | (((tmp >> 6) & m1) << 4)]
    scales = [b - 32 for b in struct.pack("<IIII", *aux)]
    out, e, g, mbit = np.zeros(256, np.float32), 0, 0, 1
    for half in range(2):
        Q = q[32 * half:]
        for shift in (0, 2, 4, 6):
            for part in range(2):
                dl = d * scales[g]
                g += 1
                for l in range(16):
                    i = l + 16 * part
                    out[e] = dl * (((Q[i] >> shift) & 3) - (0 if hm[i] & mbit else 4))
                    e += 1
            mbit <<= 1
    return out


def _scalar_q5k(blk):
    d, dm, sc, qh, ql = _h(blk, 0), _h(blk, 2), blk[4:16], blk[16:48], blk[48:176]

    def sm(j):
        if j < 4:
            return sc[j] & 63, sc[j + 4] & 63
        return (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4), (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4)
    out, e, u1, u2 = np.zeros(256, np.float32), 0, 1, 2
    for j in range(0, 8, 2):
        s1, m1 = sm(j)
        s2, m2 = sm(j + 1)
        Q = ql[16 * j:]
        for l in range(32):
            out[e] = d * s1 * ((Q[l] & 15) + (16 if qh[l] & u1 else 0)) - dm * m1
            e += 1
        for l in range(32):
            out[e] = d * s2 * ((Q[l] >> 4) + (16 if qh[l] & u2 else 0)) - dm * m2
            e += 1
        u1 <<= 2
        u2 <<= 2
    return out


def _scalar_q5_0(blk):
    d = _h(blk, 0)
    qh = struct.unpack("<I", _by(blk[2:6]))[0]
    qs = blk[6:22]
    out = np.zeros(32, np.float32)
    for j in range(16):
        out[j] = (((qs[j] & 15) | (((qh >> j) & 1) << 4)) - 16) * d
        out[j + 16] = (((qs[j] >> 4) | (((qh >> (j + 16)) & 1) << 4)) - 16) * d
    return out


def _scalar_iq4xs(blk):
    d = _h(blk, 0)
    sh = struct.unpack("<H", _by(blk[2:4]))[0]
    sl, qs = blk[4:8], blk[8:136]
    out = np.zeros(256, np.float32)
    for ib in range(8):
        ls = ((sl[ib // 2] >> (4 * (ib % 2))) & 15) | (((sh >> (2 * ib)) & 3) << 4)
        for j in range(16):
            out[32 * ib + j] = d * (ls - 32) * k.IQ4_BOOK[qs[16 * ib + j] & 15]
            out[32 * ib + j + 16] = d * (ls - 32) * k.IQ4_BOOK[qs[16 * ib + j] >> 4]
    return out


@pytest.mark.parametrize("typ,scalar,f16_at", [
    (GGMLType.Q6_K, _scalar_q6k, (208,)),
    (GGMLType.Q2_K, _scalar_q2k, (80, 82)),
    (GGMLType.Q3_K, _scalar_q3k, (108,)),
    (GGMLType.Q5_K, _scalar_q5k, (0, 2)),
    (GGMLType.Q5_0, _scalar_q5_0, (0,)),
    (GGMLType.IQ4_XS, _scalar_iq4xs, (0,)),
])
def test_reader_matches_spec_statement(typ, scalar, f16_at):
    per, nbytes = BLOCK_SIZES[typ]
    b = _rand_blocks(3, nbytes, seed=int(typ), f16_at=f16_at)
    got = dequantize(b.reshape(-1), typ, 3 * per)
    want = np.concatenate([scalar(b[i].astype(np.int64)) for i in range(3)])
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-7)


def test_q8k_q8_1_q5_1_readers():
    b = _rand_blocks(2, 292, 1, f32_at=(0,))
    d = np.frombuffer(bytes(b[:, 0:4]), np.float32)
    q = b[:, 4:260].view(np.int8).astype(np.float32)
    np.testing.assert_allclose(dequantize(b.reshape(-1), GGMLType.Q8_K, 512), (q * d[:, None]).reshape(-1))
    b = _rand_blocks(2, 36, 2, f16_at=(0, 2))
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    np.testing.assert_allclose(dequantize(b.reshape(-1), GGMLType.Q8_1, 64),
                               (b[:, 4:].view(np.int8).astype(np.float32) * d).reshape(-1))


@pytest.mark.parametrize("typ,quant,tol", [
    (GGMLType.Q5_0, k.quantize_q5_0, 1 / 16), (GGMLType.Q5_1, k.quantize_q5_1, 1 / 31),
    (GGMLType.Q6_K, k.quantize_q6_k, 1 / 31), (GGMLType.Q8_K, k.quantize_q8_k, 1 / 127),
    (GGMLType.IQ4_NL, k.quantize_iq4_nl, 0.15),
])
def test_round_trip(typ, quant, tol):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.02, 4096).astype(np.float32)
    y = dequantize(quant(x), typ, x.size)
    per = BLOCK_SIZES[typ][0]
    amax = np.repeat(np.abs(x).reshape(-1, per).max(-1), per)
    # each error stays within about one quantisation step of its block's range
    assert np.all(np.abs(y - x) <= tol * amax * 1.05 + 1e-6)
    assert np.corrcoef(x, y)[0, 1] > 0.99


def test_fp8_fp4_codecs():
    x = np.array([0, 1, -1, 0.5, 448, -448, 1000, 3.3e-3], np.float32)
    e4 = k.dequantize_fp8(k.quantize_fp8(x, "e4m3"), x.size, "e4m3")
    np.testing.assert_allclose(e4[:6], x[:6])
    assert e4[6] == 448  # saturates
    e5 = k.dequantize_fp8(k.quantize_fp8(x, "e5m2"), x.size, "e5m2")
    np.testing.assert_allclose(e5, x, rtol=0.13)
    v = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -6, -0.5, 5.2], np.float32)
    f4 = k.dequantize_fp4(k.quantize_fp4(v), v.size)
    np.testing.assert_array_equal(f4[:10], v[:10])
    assert f4[10] in (4.0, 6.0)


def _logits(m, T=7):
    from openmini_v1_b200.models.llama import ForwardBatch
    import torch
    i32 = dict(dtype=torch.int32)
    fb = ForwardBatch(torch.arange(50, 50 + T, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                      torch.arange(2, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                      torch.tensor([T - 1]))
    return m.logits(m(fb, m.allocate_kv(2)))


@pytest.mark.parametrize("quant,tol", [("f32", 1e-5), ("q6_k", 6e-2), ("q8_k", 3e-2)])
def test_moe_gguf_roundtrip(tmp_path, quant, tol):
    """A MoE decoder (routed + shared + zero-computation experts, dense first layer) is
    written with llama.cpp's stacked expert tensors and read back."""
    from openmini_v1_b200.models.config import MoEConfig, tiny
    from openmini_v1_b200.models.llama import DecoderLM
    from openmini_v1_b200.models.loader import load_gguf_model, save_gguf_model
    cfg = tiny()
    cfg.intermediate_size = 512
    cfg.moe = MoEConfig(num_experts=4, top_k=2, expert_ffn=256, num_shared_experts=1, num_zero_experts=1,
                        ffn_prefix_layers=1)
    m = DecoderLM(cfg, device="cpu", seed=3)
    ref = _logits(m)
    path = str(tmp_path / f"moe_{quant}.gguf")
    save_gguf_model(m, path, quant)
    m2 = load_gguf_model(path, device="cpu")
    assert m2.cfg.moe.num_experts == 4 and m2.cfg.moe.num_zero_experts == 1 and m2.cfg.moe.ffn_prefix_layers == 1
    assert "router" in m2.layers[1] and "gate_up" in m2.layers[0]
    out = _logits(m2)
    assert (out - ref).abs().max().item() < tol * max(1.0, ref.abs().max().item())
