"""Image understanding for the serving API: decode the uploaded image, run the
vision encoder, splice its features into the prompt and generate with the engine.

The features replace ``num_patches`` placeholder positions of the prompt. The ids
written at those positions are derived from the image bytes (a hash per position),
so the engine's prefix cache, which keys on ids, reuses a cached prefix only for
the same image and never across different images.

Reference counterpart: the ImageUnderstanding / ImageUnderstandingStream RPCs and
/api/v1/image/understand of openmini-server/src/service/grpc/server.rs:385-515 and
service/http; the reference answers them with placeholder text.
"""
from __future__ import annotations

import hashlib
import io

import numpy as np

from ..engine.request import SamplingParams
from ..engine.tokenizer import IncrementalDecoder


def decode_image(data: bytes) -> np.ndarray:
    """Encoded image bytes (PNG, JPEG, ... via Pillow) or a raw .npy [H, W, 3] array -> uint8 RGB."""
    if data[:6] == b"\x93NUMPY":
        return np.load(io.BytesIO(data))
    from PIL import Image
    return np.asarray(Image.open(io.BytesIO(data)).convert("RGB"))


def image_ids(data: bytes, n: int, vocab: int, reserved: int = 256) -> list:
    h = hashlib.blake2b(data, digest_size=16).digest()
    base = int.from_bytes(h[:8], "little")
    return [reserved + (base + i * 0x9E3779B97F4A7C15) % (vocab - reserved) for i in range(n)]


class ImageUnderstanding:
    """``pan_scan``: large images are tiled (``models.vision.pan_and_scan``: the whole
    image plus base_size tiles) and the features of every crop are spliced in order."""

    def __init__(self, aengine, tokenizer, encoder, default_max_tokens: int = 256, pan_scan: bool = False,
                 pan_scan_base: int = 896, pan_scan_max_tokens: int = 16384):
        self.aengine, self.tok, self.enc = aengine, tokenizer, encoder
        self.default_max = default_max_tokens
        self.vocab = aengine.engine.model.cfg.vocab_size
        self.pan_scan, self.ps_base, self.ps_max = pan_scan, pan_scan_base, pan_scan_max_tokens

    def prepare(self, image_bytes: bytes, question: str):
        """-> (prompt ids, (first image position, features [P, hidden]))."""
        img = decode_image(image_bytes)
        if self.pan_scan:
            import torch
            from ..models.vision import pan_and_scan
            crops = pan_and_scan(img, self.enc.cfg, self.ps_base, max_tokens=self.ps_max)
            feats = torch.cat([self.enc(c)[0] for c in crops])
        else:
            feats = self.enc(img)[0]
        P = feats.shape[0]
        head = self.tok.encode("user: <image>\n")
        tail = self.tok.encode(f"{question}\nassistant:", add_bos=False)
        ids = head + image_ids(image_bytes, P, self.vocab) + tail
        return ids, (len(head), feats)

    async def stream(self, image_bytes: bytes, question: str, max_tokens: int = 0, temperature: float = 0.0):
        """Async iterator of (text piece, finished, prompt tokens, generated tokens)."""
        ids, img = self.prepare(image_bytes, question)
        sp = SamplingParams(temperature=max(temperature, 0.0), max_tokens=max_tokens or self.default_max)
        dec, n = IncrementalDecoder(self.tok), 0
        async for out in self.aengine.generate(ids, sp, image_embeds=img):
            n += 1
            yield dec.push(out.new_token_ids[0]), out.finished, len(ids), n

    async def answer(self, image_bytes: bytes, question: str, max_tokens: int = 0, temperature: float = 0.0):
        text, pt, n = [], 0, 0
        async for piece, fin, pt, n in self.stream(image_bytes, question, max_tokens, temperature):
            text.append(piece)
        return "".join(text), pt, n


class SpeechToText:
    """Speech input: decode the audio, run the audio encoder, splice the features into a
    transcription prompt (placeholder ids derived from the audio bytes, as for images)
    and generate."""

    def __init__(self, aengine, tokenizer, encoder, default_max_tokens: int = 128):
        self.aengine, self.tok, self.enc = aengine, tokenizer, encoder
        self.default_max = default_max_tokens
        self.vocab = aengine.engine.model.cfg.vocab_size

    def prepare(self, audio_bytes: bytes, language: str = ""):
        from ..models.audio import decode_audio
        feats = self.enc.encode(decode_audio(audio_bytes, self.enc.cfg.sample_rate))
        head = self.tok.encode("user: <audio>\n")
        tail = self.tok.encode(f"transcribe{(' (' + language + ')') if language else ''}:\nassistant:",
                               add_bos=False)
        return head + image_ids(audio_bytes, feats.shape[0], self.vocab) + tail, (len(head), feats)

    async def stream(self, audio_bytes: bytes, language: str = "", max_tokens: int = 0):
        ids, feats = self.prepare(audio_bytes, language)
        sp = SamplingParams(temperature=0.0, max_tokens=max_tokens or self.default_max, logprobs=True)
        dec, n = IncrementalDecoder(self.tok), 0
        async for out in self.aengine.generate(ids, sp, image_embeds=feats):
            n += 1
            lp = out.logprobs[-1] if getattr(out, "logprobs", None) else 0.0
            yield dec.push(out.new_token_ids[0]), out.finished, lp


class TextToSpeech:
    """Speech output: the TTS model synthesises the whole clip (off the event loop), and
    the WAV bytes are sent in chunks whose concatenation is one WAV file (header first).
    An empty voice is "default" and a zero speed (the protobuf default) is 1.0."""

    def __init__(self, model, chunk_bytes: int = 32000):
        self.model, self.chunk = model, chunk_bytes

    @staticmethod
    def _args(voice, speed):
        return voice or "default", float(speed) if speed else 1.0

    async def synthesize(self, text: str, voice: str = "", speed: float = 0.0, pitch: float = 0.0) -> bytes:
        import asyncio
        voice, speed = self._args(voice, speed)
        return await asyncio.to_thread(self.model.synthesize_wav, text, voice, speed, float(pitch))

    async def stream(self, text: str, voice: str = "", speed: float = 0.0, pitch: float = 0.0):
        wav = await self.synthesize(text, voice, speed, pitch)
        for i in range(0, len(wav), self.chunk):
            yield wav[i:i + self.chunk], i + self.chunk >= len(wav)
