"""Audio encoder (Whisper-style) for speech input to the language model.

    wave (16 kHz mono) -> log-mel spectrogram (n_mels bands, 25 ms window, 10 ms hop)
    -> two 1-D convolutions (kernel 3; the second with stride 2) with GELU
    -> sinusoidal positions -> pre-norm transformer blocks (bidirectional attention)
    -> LayerNorm -> linear projector to the LM hidden size

The convolutions run as GEMMs over unfolded frames, every linear is the tcgen05 GEMM
on the GPU (``ops.linear``), LayerNorm / GELU are the norm kernels, and attention is
the FlashAttention kernel (``parallel.ring_attention.attend``, bidirectional). The
mel filterbank is built from the HTK mel formula (mel = 2595 log10(1 + f / 700)) with
triangular filters. Features replace placeholder positions of the prompt exactly as
image features do (``LLMEngine.add_request(image_embeds=...)``).

Reference counterparts: the audio path of MultimodalTransformer
(openmini-server/src/model/inference/model.rs:2713-3350) and the SpeechToText RPC
(openmini-server/src/service/grpc/server.rs); the reference answers with placeholders.
"""
from __future__ import annotations

import io
import math
import wave
from dataclasses import dataclass

import numpy as np
import torch

from .. import ops


@dataclass
class AudioConfig:
    sample_rate: int = 16000
    n_fft: int = 400
    hop: int = 160
    n_mels: int = 80
    hidden_size: int = 512
    num_layers: int = 4
    num_heads: int = 4           # head_dim 128
    mlp_size: int = 2048
    max_frames: int = 3000       # 30 s
    lm_hidden: int = 4096
    ln_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


def mel_filterbank(sr: int, n_fft: int, n_mels: int) -> torch.Tensor:
    """[n_mels, n_fft // 2 + 1] triangular filters equally spaced on the HTK mel scale."""
    mel = lambda f: 2595.0 * math.log10(1.0 + f / 700.0)  # noqa: E731
    inv = lambda m: 700.0 * (10 ** (m / 2595.0) - 1.0)  # noqa: E731
    pts = torch.tensor([inv(m) for m in np.linspace(mel(0.0), mel(sr / 2), n_mels + 2)], dtype=torch.float64)
    freqs = torch.linspace(0, sr / 2, n_fft // 2 + 1, dtype=torch.float64)
    fb = torch.zeros(n_mels, freqs.numel(), dtype=torch.float64)
    for i in range(n_mels):
        lo, c, hi = pts[i], pts[i + 1], pts[i + 2]
        up = (freqs - lo) / (c - lo)
        down = (hi - freqs) / (hi - c)
        fb[i] = torch.clamp(torch.minimum(up, down), min=0.0)
    return fb.float()


def log_mel(wav: torch.Tensor, cfg: AudioConfig) -> torch.Tensor:
    """[samples] float -> [frames, n_mels] log10 power, floored at max - 8 and scaled to ~[-1, 1]."""
    win = torch.hann_window(cfg.n_fft, device=wav.device)
    spec = torch.stft(wav.float(), cfg.n_fft, cfg.hop, window=win, return_complex=True).abs().pow(2)
    mel = mel_filterbank(cfg.sample_rate, cfg.n_fft, cfg.n_mels).to(wav.device) @ spec  # [n_mels, frames]
    lm = torch.log10(mel.clamp(min=1e-10))
    lm = torch.maximum(lm, lm.max() - 8.0)
    return ((lm + 4.0) / 4.0).t()[: cfg.max_frames].contiguous()


def decode_audio(data: bytes, sr: int = 16000) -> torch.Tensor:
    """WAV (PCM 8 / 16 / 32-bit, any rate, mono or stereo) or a .npy float array -> mono float at ``sr``."""
    if data[:6] == b"\x93NUMPY":
        x = np.load(io.BytesIO(data)).astype(np.float32).reshape(-1)
        rate = sr
    else:
        with wave.open(io.BytesIO(data)) as w:
            rate, ch, width = w.getframerate(), w.getnchannels(), w.getsampwidth()
            raw = w.readframes(w.getnframes())
        dt = {1: np.uint8, 2: np.int16, 4: np.int32}[width]
        x = np.frombuffer(raw, dtype=dt).astype(np.float32)
        x = (x - 128.0) / 128.0 if width == 1 else x / float(2 ** (8 * width - 1))
        x = x.reshape(-1, ch).mean(1)
    t = torch.from_numpy(x)
    if rate != sr:  # linear resampling
        n = int(round(len(t) * sr / rate))
        pos = torch.linspace(0, len(t) - 1, n)
        i0 = pos.floor().long().clamp(max=len(t) - 1)
        i1 = (i0 + 1).clamp(max=len(t) - 1)
        t = t[i0] + (t[i1] - t[i0]) * (pos - i0)
    return t


def _sinusoids(n: int, d: int) -> torch.Tensor:
    inc = math.log(10000) / (d // 2 - 1)
    inv = torch.exp(-inc * torch.arange(d // 2))
    a = torch.arange(n)[:, None] * inv[None]
    return torch.cat([a.sin(), a.cos()], 1)


def attention_full(qkv: torch.Tensor, n: int, H: int, Dh: int) -> torch.Tensor:
    """Bidirectional multi-head attention over ``n`` rows of a fused [n, 3 H Dh] QKV:
    the FlashAttention kernel on the GPU when Dh is 128, fp32 softmax attention otherwise."""
    if qkv.is_cuda and Dh == 128:
        from ..parallel.ring_attention import attend
        q, k, v = (qkv[:, i * H * Dh:(i + 1) * H * Dh].reshape(n, H, Dh).contiguous() for i in range(3))
        out, _ = attend(q, k, v, 1 / math.sqrt(Dh), causal=False)
        return out.to(qkv.dtype).reshape(n, H * Dh)
    q, k, v = (qkv[:, i * H * Dh:(i + 1) * H * Dh].float().reshape(n, H, Dh).transpose(0, 1) for i in range(3))
    p = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(Dh), -1)
    return (p @ v).transpose(0, 1).reshape(n, H * Dh).to(qkv.dtype)


def init_blocks(n: int, D: int, mlp: int, rnd, one, zero) -> list:
    """Weights of ``n`` pre-LayerNorm transformer blocks (``rnd(*shape)`` draws a weight)."""
    return [{"ln1_w": one(), "ln1_b": zero(), "qkv": rnd(3 * D, D), "o": rnd(D, D),
             "ln2_w": one(), "ln2_b": zero(), "fc1": rnd(mlp, D), "fc2": rnd(D, mlp)} for _ in range(n)]


def run_blocks(x: torch.Tensor, layers: list, H: int, eps: float) -> torch.Tensor:
    """Pre-LayerNorm blocks with bidirectional attention and a GELU MLP, residuals in fp32."""
    n, D = x.shape
    for L in layers:
        a = ops.layernorm(x, L["ln1_w"], L["ln1_b"], eps)
        att = attention_full(ops.linear(a, L["qkv"]), n, H, D // H)
        x = (x.float() + ops.linear(att, L["o"]).float()).to(x.dtype)
        m = ops.layernorm(x, L["ln2_w"], L["ln2_b"], eps)
        x = (x.float() + ops.linear(ops.gelu(ops.linear(m, L["fc1"])), L["fc2"]).float()).to(x.dtype)
    return x


class AudioEncoder:
    def __init__(self, cfg: AudioConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0, std: float = 0.02):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        g = torch.Generator().manual_seed(seed)
        rnd = lambda *s: (torch.randn(*s, generator=g) * std).to(self.device, dtype)  # noqa: E731
        D = cfg.hidden_size
        one = lambda: torch.ones(D, dtype=dtype, device=self.device)  # noqa: E731
        zero = lambda: torch.zeros(D, dtype=dtype, device=self.device)  # noqa: E731
        self.conv1 = rnd(D, cfg.n_mels * 3)
        self.conv2 = rnd(D, D * 3)
        self.pos = _sinusoids(cfg.max_frames // 2 + 1, D).to(self.device, dtype)
        self.layers = init_blocks(cfg.num_layers, D, cfg.mlp_size, rnd, one, zero)
        self.post_w, self.post_b = one(), zero()
        self.proj = rnd(cfg.lm_hidden, D)

    @staticmethod
    def _conv(x, w, stride):
        """x [T, C] -> [T', O]: kernel-3 convolution (padding 1) as unfold + GEMM."""
        xp = torch.nn.functional.pad(x.t()[None], (1, 1))[0].t()            # [T + 2, C]
        cols = xp.unfold(0, 3, stride)                                        # [T', C, 3]
        return ops.linear(cols.transpose(1, 2).reshape(cols.shape[0], -1).contiguous(), w)

    def encode(self, wav: torch.Tensor) -> torch.Tensor:
        """[samples] -> projected features [frames / 2, lm_hidden]."""
        cfg = self.cfg
        mel = log_mel(wav.to(self.device), cfg).to(self.dtype)
        x = ops.gelu(self._conv(mel, self.conv1, 1))
        x = ops.gelu(self._conv(x, self.conv2, 2))
        n = x.shape[0]
        x = (x.float() + self.pos[:n].float()).to(self.dtype)
        x = run_blocks(x, self.layers, cfg.num_heads, cfg.ln_eps)
        x = ops.layernorm(x, self.post_w, self.post_b, cfg.ln_eps)
        return ops.linear(x, self.proj)
