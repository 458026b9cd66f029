"""Text-to-speech: a non-autoregressive acoustic model plus a Griffin-Lim vocoder.

    text (UTF-8 bytes) -> byte embedding + sinusoidal positions + voice embedding
    -> encoder blocks (bidirectional) -> duration head: frames per byte
       d = clamp(round(exp(w . x + log base) / speed), 1, max_dur)
    -> length regulator (each byte's hidden state repeated d times)
    -> + frame positions -> decoder blocks -> linear to n_mels
    -> normalised log-mel in [-1, 1] (the scale of ``audio.log_mel``)
    -> mel power -> linear power by the pseudo-inverse of the mel filterbank
    -> optional pitch shift (the magnitude spectrum resampled along frequency by
       2^(pitch / 12), pitch in semitones)
    -> Griffin-Lim phase reconstruction (Griffin & Lim, "Signal estimation from
       modified short-time Fourier transform", IEEE TASSP 1984), with the momentum
       of Perraudin, Balazs and Sondergaard, "A fast Griffin-Lim algorithm"
       (WASPAA 2013)
    -> 16 kHz mono waveform -> 16-bit PCM WAV.

The acoustic model shares its blocks with the audio encoder (``audio.run_blocks``:
every linear is the tcgen05 GEMM on the GPU, LayerNorm / GELU are the norm kernels,
attention the FlashAttention kernel when head_dim is 128). The vocoder uses torch's
STFT / inverse STFT. The STFT settings are those of the speech-input front end, so
``log_mel(synthesize(...))`` is on the scale the model was asked to produce. Weights
are random-init (no checkpoint on this box): the waveform is well formed (length
from the durations, peak-normalised PCM, valid WAV) but not intelligible speech.

Request limits follow the reference's TextToSpeech handler: text 1 to 10000
characters, speed 0.25 to 4.0, pitch -20 to 20.

Reference counterparts: TextToSpeech (openmini-server/src/service/grpc/server.rs:943-1000,
which streams a synthetic sine) and POST /api/v1/tts (openmini-server/src/service/http/
handlers.rs:225-265, types.rs:133-162: {text, voice, language, speed, pitch} ->
{audio_data: base64}).
"""
from __future__ import annotations

import hashlib
import io
import math
import wave
from dataclasses import dataclass

import torch

from .. import ops
from .audio import _sinusoids, init_blocks, mel_filterbank, run_blocks

MAX_TEXT = 10000


@dataclass
class TTSConfig:
    sample_rate: int = 16000
    n_fft: int = 400
    hop: int = 160
    n_mels: int = 80
    hidden_size: int = 256
    num_heads: int = 2            # head_dim 128
    enc_layers: int = 2
    dec_layers: int = 2
    mlp_size: int = 1024
    base_frames: float = 6.0      # frames per byte at speed 1 before the learned duration (60 ms)
    max_dur: int = 40
    max_frames: int = 60000       # 10 minutes
    gl_iters: int = 32
    ln_eps: float = 1e-5


def validate_request(text: str, speed: float, pitch: float):
    if not text:
        raise ValueError("text is empty")
    if len(text) > MAX_TEXT:
        raise ValueError(f"text is longer than {MAX_TEXT} characters")
    if not 0.25 <= speed <= 4.0:
        raise ValueError("speed must be in [0.25, 4.0]")
    if not -20.0 <= pitch <= 20.0:
        raise ValueError("pitch must be in [-20, 20]")


def mel_to_power(norm_log_mel: torch.Tensor, fb_pinv: torch.Tensor) -> torch.Tensor:
    """[frames, n_mels] normalised log-mel (``audio.log_mel`` scale) -> [n_fft/2+1, frames] power."""
    mel_power = torch.pow(10.0, norm_log_mel.float() * 4.0 - 4.0).t()
    return (fb_pinv @ mel_power).clamp(min=0.0)


def pitch_shift(mag: torch.Tensor, semitones: float) -> torch.Tensor:
    """Resample a [bins, frames] magnitude spectrogram along frequency by 2^(semitones/12)."""
    if semitones == 0.0:
        return mag
    r = 2.0 ** (semitones / 12.0)
    F = mag.shape[0]
    src = torch.arange(F, device=mag.device, dtype=torch.float32) / r
    i0 = src.floor().long()
    w = (src - i0).unsqueeze(1)
    ok = (i0 + 1 < F).unsqueeze(1)
    i0c, i1c = i0.clamp(max=F - 1), (i0 + 1).clamp(max=F - 1)
    return torch.where(ok, mag[i0c] * (1 - w) + mag[i1c] * w, torch.zeros_like(mag[i0c]))


def griffin_lim(mag: torch.Tensor, n_fft: int, hop: int, iters: int = 32, momentum: float = 0.99,
                length: int | None = None, seed: int = 0) -> torch.Tensor:
    """[n_fft/2+1, frames] STFT magnitude -> waveform whose STFT magnitude approximates it."""
    win = torch.hann_window(n_fft, device=mag.device)
    g = torch.Generator(device="cpu").manual_seed(seed)
    phase = torch.exp(2j * math.pi * torch.rand(mag.shape, generator=g)).to(mag.device)
    spec = mag * phase
    prev = torch.zeros_like(spec)
    for _ in range(iters):
        y = torch.istft(spec, n_fft, hop, window=win, length=length)
        proj = torch.stft(y, n_fft, hop, window=win, return_complex=True)
        accel = proj + momentum * (proj - prev) if momentum else proj
        prev = proj
        spec = mag * accel / accel.abs().clamp(min=1e-8)
    return torch.istft(spec, n_fft, hop, window=win, length=length)


def to_wav(wav: torch.Tensor, sr: int) -> bytes:
    """Float waveform -> 16-bit PCM mono WAV bytes, peak-normalised to 0.9."""
    x = wav.detach().float().cpu()
    peak = float(x.abs().max()) if x.numel() else 0.0
    if peak > 0:
        x = x * (0.9 / peak)
    pcm = (x.clamp(-1, 1) * 32767.0).round().to(torch.int16).numpy().tobytes()
    buf = io.BytesIO()
    with wave.open(buf, "wb") as w:
        w.setnchannels(1)
        w.setsampwidth(2)
        w.setframerate(sr)
        w.writeframes(pcm)
    return buf.getvalue()


class TTSModel:
    def __init__(self, cfg: TTSConfig | None = None, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                 std: float = 0.02):
        self.cfg = cfg = cfg or TTSConfig()
        self.device, self.dtype = torch.device(device), dtype
        g = torch.Generator().manual_seed(seed)
        rnd = lambda *s: (torch.randn(*s, generator=g) * std).to(self.device, dtype)  # noqa: E731
        D = cfg.hidden_size
        one = lambda: torch.ones(D, dtype=dtype, device=self.device)  # noqa: E731
        zero = lambda: torch.zeros(D, dtype=dtype, device=self.device)  # noqa: E731
        self.embed = rnd(257, D)                         # byte values 0..255 and a pad row
        self.enc = init_blocks(cfg.enc_layers, D, cfg.mlp_size, rnd, one, zero)
        self.dur_w = rnd(1, D)
        self.dec = init_blocks(cfg.dec_layers, D, cfg.mlp_size, rnd, one, zero)
        self.post_w, self.post_b = one(), zero()
        self.mel_w = rnd(cfg.n_mels, D)
        self.pos = _sinusoids(4096, D).to(self.device)
        fb = mel_filterbank(cfg.sample_rate, cfg.n_fft, cfg.n_mels).double()
        self.fb_pinv = torch.linalg.pinv(fb).float().to(self.device)

    def _positions(self, n: int) -> torch.Tensor:
        """Sinusoidal rows for n positions (the table repeats past its 4096 rows)."""
        idx = torch.arange(n, device=self.device) % self.pos.shape[0]
        return self.pos[idx]

    def voice_vector(self, voice: str) -> torch.Tensor:
        """A fixed speaker embedding per voice name (seeded by a hash of the name)."""
        seed = int.from_bytes(hashlib.sha256(voice.encode()).digest()[:7], "little")
        g = torch.Generator().manual_seed(seed)
        return (torch.randn(self.cfg.hidden_size, generator=g) * 0.02).to(self.device)

    @torch.no_grad()
    def durations(self, text: str, voice: str = "default", speed: float = 1.0):
        """Encoder states [n, D] and frames per byte [n] (int64)."""
        cfg = self.cfg
        ids = torch.tensor(list(text.encode("utf-8")), dtype=torch.long, device=self.device)
        n = ids.numel()
        x = (ops.embedding(ids.to(torch.int32), self.embed).float() + self._positions(n)
             + self.voice_vector(voice)).to(self.dtype)
        x = run_blocks(x, self.enc, cfg.num_heads, cfg.ln_eps)
        logd = (x.float() @ self.dur_w.float().t()).squeeze(1) + math.log(cfg.base_frames)  # one output: a GEMV
        d = torch.clamp(torch.round(torch.exp(logd) / speed), 1, cfg.max_dur).long()
        return x, d

    @torch.no_grad()
    def mel(self, text: str, voice: str = "default", speed: float = 1.0, d: torch.Tensor | None = None) -> torch.Tensor:
        """[frames, n_mels] normalised log-mel; ``d`` overrides the predicted frames per byte."""
        cfg = self.cfg
        x, dp = self.durations(text, voice, speed)
        d = dp if d is None else d.to(dp.device, torch.long)
        h = torch.repeat_interleave(x, d, dim=0)[: cfg.max_frames]
        h = (h.float() + self._positions(h.shape[0])).to(self.dtype)
        h = run_blocks(h, self.dec, cfg.num_heads, cfg.ln_eps)
        h = ops.layernorm(h, self.post_w, self.post_b, cfg.ln_eps)
        return torch.tanh(ops.linear(h, self.mel_w).float())

    @torch.no_grad()
    def vocode(self, norm_log_mel: torch.Tensor, pitch: float = 0.0, seed: int = 0) -> torch.Tensor:
        cfg = self.cfg
        mag = mel_to_power(norm_log_mel.to(self.device), self.fb_pinv).sqrt()
        mag = pitch_shift(mag, pitch)
        n = (mag.shape[1] - 1) * cfg.hop
        return griffin_lim(mag, cfg.n_fft, cfg.hop, cfg.gl_iters, length=n, seed=seed)

    def synthesize(self, text: str, voice: str = "default", speed: float = 1.0, pitch: float = 0.0) -> torch.Tensor:
        """Float waveform at ``cfg.sample_rate``."""
        validate_request(text, speed, pitch)
        return self.vocode(self.mel(text, voice, speed), pitch)

    def synthesize_wav(self, text: str, voice: str = "default", speed: float = 1.0, pitch: float = 0.0) -> bytes:
        return to_wav(self.synthesize(text, voice, speed, pitch), self.cfg.sample_rate)
