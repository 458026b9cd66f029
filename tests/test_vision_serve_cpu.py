"""Image understanding through the serving stack on CPU: image features spliced
into the prompt through the engine match a full recompute with the same features,
image-derived placeholder ids keep the prefix cache per image, and the HTTP and
gRPC routes answer (501 / UNIMPLEMENTED without an encoder). Speech in and out:
the audio encoder, the Griffin-Lim vocoder against the speech front end, the TTS
model's durations / voices / limits, and the TTS HTTP and gRPC routes."""
import asyncio
import base64
import io

import numpy as np
import pytest
import torch
from fastapi.testclient import TestClient

from openmini_v1_b200.engine.async_engine import AsyncLLMEngine
from openmini_v1_b200.engine.engine import EngineConfig, LLMEngine
from openmini_v1_b200.engine.request import SamplingParams
from openmini_v1_b200.engine.tokenizer import ByteTokenizer
from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
from openmini_v1_b200.models.vision import VisionConfig, VisionEncoder
from openmini_v1_b200.serve.http import create_app
from openmini_v1_b200.serve.vision_service import ImageUnderstanding, image_ids


def _npy(seed):
    img = np.random.default_rng(seed).integers(0, 255, (40, 40, 3), dtype=np.uint8)
    b = io.BytesIO()
    np.save(b, img)
    return b.getvalue()


@pytest.fixture(scope="module")
def vstack():
    m = DecoderLM(tiny(), device="cpu", seed=0)
    eng = LLMEngine(m, EngineConfig(max_num_seqs=4, max_model_len=256, enable_prefix_cache=True))
    aeng = AsyncLLMEngine(eng)
    tok = ByteTokenizer()
    enc = VisionEncoder(VisionConfig(image_size=32, patch_size=16, hidden_size=128, num_layers=1, num_heads=2,
                                     mlp_size=256, lm_hidden=256), device="cpu", dtype=torch.float32)
    yield aeng, tok, m, ImageUnderstanding(aeng, tok, enc, default_max_tokens=4)
    aeng.shutdown()


def test_engine_image_rows_match_recompute(vstack):
    aeng, tok, m, vis = vstack
    ids, (p0, feats) = vis.prepare(_npy(1), "what is it?")
    eng = LLMEngine(m, EngineConfig(max_num_seqs=2, max_model_len=256, enable_prefix_cache=False))
    r = eng.add_request("a", ids, SamplingParams(temperature=0.0, max_tokens=3, ignore_eos=True),
                        image_embeds=(p0, feats))
    while eng.has_unfinished():
        eng.step()
    toks = list(ids)
    rows = torch.arange(p0, p0 + feats.shape[0])
    for _ in range(3):
        T = len(toks)
        i32 = dict(dtype=torch.int32)
        fb = ForwardBatch(torch.tensor(toks, **i32), torch.arange(T, **i32), torch.arange(T, **i32),
                          torch.arange(16, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32), T,
                          torch.tensor([T - 1]), embed_override=(rows, feats))
        toks.append(int(m.logits(m(fb, m.allocate_kv(16))).argmax(-1)))
    assert r.output_token_ids == toks[len(ids):]


def test_image_ids_differ_per_image():
    a, b = image_ids(_npy(1), 4, 32000), image_ids(_npy(2), 4, 32000)
    assert a != b and a == image_ids(_npy(1), 4, 32000) and min(a + b) >= 256


def test_http_and_grpc_image_routes(vstack):
    aeng, tok, m, vis = vstack
    c = TestClient(create_app(aeng, tok, "tiny", vision=vis))
    r = c.post("/api/v1/image/understand", json={"image": base64.b64encode(_npy(3)).decode(), "question": "?",
                                                 "max_tokens": 3})
    assert r.status_code == 200, r.text
    assert r.json()["usage"]["completion_tokens"] == 3
    assert c.post("/api/v1/image/understand", json={"image": "AAAA"}).status_code == 400
    assert TestClient(create_app(aeng, tok, "tiny")).post("/api/v1/image/understand",
                                                          json={"image": ""}).status_code == 501
    import grpc
    from openmini_v1_b200.serve import proto
    from openmini_v1_b200.serve.grpc_server import OpenMiniServicer, start_grpc_server

    async def run():
        server, port = await start_grpc_server(OpenMiniServicer(aeng, tok, vision=vis), "127.0.0.1:0")
        try:
            async with grpc.aio.insecure_channel(f"127.0.0.1:{port}") as ch:
                req = proto.ImageRequest(session_id="s", image_data=_npy(4), question="?")
                ser = proto.message("ImageRequest").SerializeToString
                de = proto.message("ImageResponse").FromString
                one = await ch.unary_unary(f"/{proto.SERVICE}/ImageUnderstanding", request_serializer=ser,
                                           response_deserializer=de)(req)
                assert one.finished and one.session_id == "s"
                outs = [o async for o in ch.unary_stream(f"/{proto.SERVICE}/ImageUnderstandingStream",
                                                         request_serializer=ser, response_deserializer=de)(req)]
                assert len(outs) == 4 and outs[-1].finished and "".join(o.token for o in outs) == one.token
        finally:
            await server.stop(1)
    asyncio.run(run())


def _wav(seconds=0.5, rate=22050, seed=0):
    import wave
    t = np.arange(int(seconds * rate)) / rate
    x = 0.3 * np.sin(2 * np.pi * 440 * t) + 0.05 * np.random.default_rng(seed).normal(size=t.size)
    b = io.BytesIO()
    with wave.open(b, "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(rate)
        w.writeframes((x * 32767).astype(np.int16).tobytes())
    return b.getvalue()


def test_audio_features_and_speech_routes(vstack):
    from openmini_v1_b200.models.audio import AudioConfig, AudioEncoder, decode_audio, log_mel, mel_filterbank
    from openmini_v1_b200.serve.vision_service import SpeechToText
    aeng, tok, m, vis = vstack
    fb = mel_filterbank(16000, 400, 80)
    freqs = torch.linspace(0, 8000, 201)
    centre = (fb @ freqs) / fb.sum(1)  # filter centroids do not fall with the band index
    assert fb.shape == (80, 201) and (fb >= 0).all() and bool((centre[1:] >= centre[:-1] - 1e-3).all()) and centre[-1] > 7000
    wav = decode_audio(_wav(), 16000)
    assert abs(wav.numel() - 8000) <= 1 and wav.abs().max() < 1.0
    lm = log_mel(wav, AudioConfig())
    assert lm.shape == (51, 80)
    # the 440 Hz tone is the loudest band
    assert abs(float(centre[int(lm.mean(0).argmax())]) - 440) < 100
    enc = AudioEncoder(AudioConfig(hidden_size=128, num_layers=1, num_heads=2, mlp_size=256, lm_hidden=256),
                       device="cpu", dtype=torch.float32)
    feats = enc.encode(wav)
    assert feats.shape == (26, 256) and torch.isfinite(feats).all()
    stt = SpeechToText(aeng, tok, enc, default_max_tokens=3)
    c = TestClient(create_app(aeng, tok, "tiny", speech=stt))
    r = c.post("/api/v1/stt", json={"audio": base64.b64encode(_wav()).decode()})
    assert r.status_code == 200 and r.json()["tokens"] == 3
    assert TestClient(create_app(aeng, tok, "tiny")).post("/api/v1/stt", json={"audio": ""}).status_code == 501
    import grpc
    from openmini_v1_b200.serve import proto
    from openmini_v1_b200.serve.grpc_server import OpenMiniServicer, start_grpc_server

    async def run():
        server, port = await start_grpc_server(OpenMiniServicer(aeng, tok, speech=stt), "127.0.0.1:0")
        try:
            async with grpc.aio.insecure_channel(f"127.0.0.1:{port}") as ch:
                data = _wav(seed=1)
                reqs = [proto.SpeechToTextRequest(session_id="a", audio_data=data[i:i + 4000])
                        for i in range(0, len(data), 4000)]

                async def gen():
                    for q in reqs:
                        yield q
                call = ch.stream_stream(f"/{proto.SERVICE}/SpeechToText",
                                        request_serializer=proto.message("SpeechToTextRequest").SerializeToString,
                                        response_deserializer=proto.message("SpeechToTextResponse").FromString)
                outs = [o async for o in call(gen())]
                assert len(outs) == 3 and outs[-1].finished and 0 < outs[-1].confidence <= 1
        finally:
            await server.stop(1)
    asyncio.run(run())


# ----------------------------------------------------------------------------- text to speech

def _small_tts():
    from openmini_v1_b200.models.tts import TTSConfig, TTSModel
    return TTSModel(TTSConfig(hidden_size=128, num_heads=1, mlp_size=256, gl_iters=8), dtype=torch.float32)


def test_griffin_lim_vocoder_inverts_the_speech_front_end():
    """log-mel of a chirp plus a tone -> vocoder -> log-mel again stays close to the
    original (much closer than noise), and a +12 semitone shift moves a 440 Hz tone's
    loudest band to about 880 Hz."""
    import math
    from openmini_v1_b200.models.audio import AudioConfig, log_mel, mel_filterbank
    from openmini_v1_b200.models.tts import TTSConfig, TTSModel
    m = TTSModel(TTSConfig(gl_iters=32), dtype=torch.float32)
    ac = AudioConfig()
    t = torch.arange(16000) / 16000
    sig = 0.5 * torch.sin(2 * math.pi * (200 * t + 300 * t * t)) + 0.3 * torch.sin(2 * math.pi * 1200 * t)
    lm = log_mel(sig, ac)
    lm2 = log_mel(m.vocode(lm), ac)
    n = min(lm.shape[0], lm2.shape[0])
    err = float((lm[:n] - lm2[:n]).abs().mean())
    noise = float((lm[:n] - log_mel(torch.randn(16000) * 0.1, ac)[:n]).abs().mean())
    assert err < 0.3 and err < noise / 3, (err, noise)
    fb = mel_filterbank(16000, 400, 80)
    centre = (fb @ torch.linspace(0, 8000, 201)) / fb.sum(1).clamp(min=1e-9)
    tone = log_mel(0.5 * torch.sin(2 * math.pi * 440 * t), ac)
    up = log_mel(m.vocode(tone, pitch=12.0), ac)
    f = float(centre[int(up.mean(0).argmax())])
    assert 700 < f < 1050, f


def test_tts_durations_voices_and_limits():
    import wave
    from openmini_v1_b200.models.tts import MAX_TEXT
    m = _small_tts()
    _, d1 = m.durations("hello there", speed=1.0)
    _, d2 = m.durations("hello there", speed=2.0)
    assert d1.numel() == len(b"hello there") and (d1 >= 1).all()
    assert abs(int(d2.sum()) - int(d1.sum()) / 2) <= d1.numel()
    wav = m.synthesize("hello there")
    assert wav.numel() == (int(d1.sum()) - 1) * m.cfg.hop and torch.isfinite(wav).all()
    a, b, c = (m.synthesize_wav("hi", voice=v) for v in ("alice", "alice", "bob"))
    assert a == b and a != c
    with wave.open(io.BytesIO(a)) as w:
        assert (w.getframerate(), w.getnchannels(), w.getsampwidth()) == (16000, 1, 2) and w.getnframes() > 0
    for bad in (dict(text=""), dict(text="x" * (MAX_TEXT + 1)), dict(text="a", speed=5.0),
                dict(text="a", pitch=-21.0)):
        with pytest.raises(ValueError):
            m.synthesize(**bad)


def test_tts_http_and_grpc_routes(vstack):
    import wave
    import grpc
    from openmini_v1_b200.serve import proto
    from openmini_v1_b200.serve.grpc_server import OpenMiniServicer, start_grpc_server
    from openmini_v1_b200.serve.vision_service import TextToSpeech
    aeng, tok, m, vis = vstack
    tts = TextToSpeech(_small_tts(), chunk_bytes=4000)
    c = TestClient(create_app(aeng, tok, "tiny", tts=tts))
    r = c.post("/api/v1/tts", json={"text": "good morning", "voice": "v1", "speed": 1.5})
    assert r.status_code == 200, r.text
    wav = base64.b64decode(r.json()["audio_data"])
    with wave.open(io.BytesIO(wav)) as w:
        assert abs(w.getnframes() / 16000 - r.json()["duration_s"]) < 1e-6
    assert c.post("/api/v1/tts", json={"text": ""}).status_code == 400
    assert c.post("/api/v1/tts", json={"text": "a", "speed": 9}).status_code == 400
    assert TestClient(create_app(aeng, tok, "tiny")).post("/api/v1/tts", json={"text": "a"}).status_code == 501

    async def run():
        server, port = await start_grpc_server(OpenMiniServicer(aeng, tok, tts=tts), "127.0.0.1:0")
        try:
            async with grpc.aio.insecure_channel(f"127.0.0.1:{port}") as ch:
                call = ch.unary_stream(f"/{proto.SERVICE}/TextToSpeech",
                                       request_serializer=proto.message("TextToSpeechRequest").SerializeToString,
                                       response_deserializer=proto.message("TextToSpeechResponse").FromString)
                outs = [o async for o in call(proto.TextToSpeechRequest(session_id="s", text="good morning",
                                                                        voice="v1", speed=1.5))]
                assert len(outs) > 1 and outs[-1].finished and not any(o.finished for o in outs[:-1])
                assert b"".join(o.audio_data for o in outs) == wav and outs[0].session_id == "s"
                with pytest.raises(grpc.aio.AioRpcError) as e:
                    _ = [o async for o in call(proto.TextToSpeechRequest(text=""))]
                assert e.value.code() == grpc.StatusCode.INVALID_ARGUMENT
        finally:
            await server.stop(1)
    asyncio.run(run())


def test_pan_and_scan_tiles_large_images(vstack):
    from openmini_v1_b200.models.vision import pan_and_scan, pan_scan_layout
    assert pan_scan_layout(800, 600) == [(0, 0, 800, 600)]
    tiles = pan_scan_layout(2000, 900, base_size=896, overlap=14)
    assert len(tiles) == 3 * 2 and tiles[1] == (882, 0, 896, 896) and tiles[2] == (1764, 0, 236, 896)
    covered = np.zeros((900, 2000), dtype=bool)
    for x, y, w, h in tiles:
        covered[y:y + h, x:x + w] = True
    assert covered.all()
    aeng, tok, m, vis = vstack
    cfg = vis.enc.cfg
    img = np.random.default_rng(5).integers(0, 255, (60, 130, 3), dtype=np.uint8)
    crops = pan_and_scan(img, cfg, base_size=48, overlap=4)
    assert crops[0].shape == (60, 130, 3) and len(crops) == 1 + 3 * 2
    assert len(pan_and_scan(img, cfg, base_size=48, overlap=4, max_tokens=3 * cfg.num_patches)) == 3
    b = io.BytesIO()
    np.save(b, img)
    ps = ImageUnderstanding(aeng, tok, vis.enc, default_max_tokens=2, pan_scan=True, pan_scan_base=48,
                            pan_scan_max_tokens=4 * cfg.num_patches)
    ids, (pos, feats) = ps.prepare(b.getvalue(), "what?")
    assert feats.shape[0] == 4 * cfg.num_patches and len(ids) > feats.shape[0]
    text, pt, n = asyncio.run(ps.answer(b.getvalue(), "what?"))
    assert n == 2 and pt == len(ids)
