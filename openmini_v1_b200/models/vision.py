"""Vision encoder (SigLIP-style ViT), image preprocessing and the projector into the
language model's embedding space.

Reference counterparts: the SigLIP encoder and Gemma image processor
(openmini-server/src/model/inference/vision/*, image_preprocess.rs: resize to a
square, rescale to [0, 1], normalise with mean = std = 0.5, non-overlapping
patches) and the vision path of MultimodalTransformer
(openmini-server/src/model/inference/model.rs:2713-3350), where image features
replace placeholder tokens of the prompt.

Per layer (pre-norm):  x += Wo · attn(LN1(x))   (bidirectional, all patches)
                       x += W2 · gelu(W1 · LN2(x))
then a final LayerNorm and a linear projector to the LM hidden size. On the GPU
every linear is the tcgen05 GEMM, LayerNorm / GELU are the norm kernels, and the
bidirectional attention is the tcgen05 FlashAttention kernel with every key
visible to every row (head_dim 128); on CPU the same ops run as fp32 statements.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .. import ops


@dataclass
class VisionConfig:
    image_size: int = 224
    patch_size: int = 16
    hidden_size: int = 1024
    num_layers: int = 4
    num_heads: int = 8           # head_dim = hidden / heads = 128
    mlp_size: int = 4096
    ln_eps: float = 1e-6
    lm_hidden: int = 4096        # projector output width
    mean: float = 0.5
    std: float = 0.5

    @property
    def num_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads


def preprocess(images, cfg: VisionConfig) -> torch.Tensor:
    """uint8 / float images [B, H, W, 3] (or one [H, W, 3]) -> patches [B, P, 3 * p * p] fp32."""
    x = torch.as_tensor(images)
    if x.dim() == 3:
        x = x[None]
    x = x.float()
    if x.max() > 1.5:
        x = x / 255.0
    x = x.permute(0, 3, 1, 2)
    x = F.interpolate(x, size=(cfg.image_size, cfg.image_size), mode="bilinear", align_corners=False)
    x = (x - cfg.mean) / cfg.std
    p = cfg.patch_size
    B, C, H, W = x.shape
    x = x.reshape(B, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (H // p) * (W // p), C * p * p).contiguous()


class VisionEncoder:
    def __init__(self, cfg: VisionConfig, device="cpu", dtype=torch.bfloat16, seed: int = 0, std: float = 0.02):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        g = torch.Generator().manual_seed(seed)

        def rnd(*shape):
            return (torch.randn(*shape, generator=g) * std).to(dtype).to(self.device)

        D, Pd = cfg.hidden_size, 3 * cfg.patch_size ** 2
        one = lambda: torch.ones(D, dtype=dtype, device=self.device)  # noqa: E731
        zero = lambda: torch.zeros(D, dtype=dtype, device=self.device)  # noqa: E731
        self.patch_w = rnd(D, Pd)
        self.pos = rnd(cfg.num_patches, D)
        self.layers = [{"ln1_w": one(), "ln1_b": zero(), "qkv": rnd(3 * D, D), "o": rnd(D, D),
                        "ln2_w": one(), "ln2_b": zero(), "fc1": rnd(cfg.mlp_size, D), "fc2": rnd(D, cfg.mlp_size)}
                       for _ in range(cfg.num_layers)]
        self.post_w, self.post_b = one(), zero()
        self.proj = rnd(cfg.lm_hidden, D)

    def _attention(self, qkv, n):
        cfg = self.cfg
        H, Dh = cfg.num_heads, cfg.head_dim
        if qkv.is_cuda:
            from ..parallel.ring_attention import attend
            q = qkv[:, :H * Dh].reshape(n, H, Dh)
            k = qkv[:, H * Dh:2 * H * Dh].reshape(n, H, Dh)
            v = qkv[:, 2 * H * Dh:].reshape(n, H, Dh)
            out, _ = attend(q.contiguous(), k.contiguous(), v.contiguous(), 1 / math.sqrt(Dh), causal=False)
            return out.to(qkv.dtype).reshape(n, H * Dh)
        q, k, v = (qkv[:, i * H * Dh:(i + 1) * H * Dh].float().reshape(n, H, Dh).transpose(0, 1) for i in range(3))
        p = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(Dh), -1)
        return (p @ v).transpose(0, 1).reshape(n, H * Dh).to(qkv.dtype)

    def encode(self, patches: torch.Tensor) -> torch.Tensor:
        """patches [P, 3 p p] (one image) -> projected features [P, lm_hidden]."""
        cfg = self.cfg
        x = ops.linear(patches.to(self.device, self.dtype).contiguous(), self.patch_w)
        x = (x.float() + self.pos.float()).to(self.dtype)
        n = x.shape[0]
        for L in self.layers:
            a = ops.layernorm(x, L["ln1_w"], L["ln1_b"], cfg.ln_eps)
            att = self._attention(ops.linear(a, L["qkv"]), n)
            x = ops.linear(att, L["o"], resid=x) if x.is_cuda else (x.float() + ops.linear(att, L["o"]).float()).to(
                self.dtype)
            m = ops.layernorm(x, L["ln2_w"], L["ln2_b"], cfg.ln_eps)
            h = ops.gelu(ops.linear(m, L["fc1"]))
            x = ops.linear(h, L["fc2"], resid=x) if x.is_cuda else (x.float() + ops.linear(h, L["fc2"]).float()).to(
                self.dtype)
        x = ops.layernorm(x, self.post_w, self.post_b, cfg.ln_eps)
        return ops.linear(x, self.proj)

    def __call__(self, images) -> list:
        return [self.encode(p) for p in preprocess(images, self.cfg)]


def pan_scan_layout(width: int, height: int, base_size: int = 896, overlap: int = 14) -> list:
    """Tiles (x, y, w, h) covering an image: one tile when it fits in base_size x
    base_size, else a grid of base_size windows stepped by base_size - overlap (edge
    tiles are cut at the border). Reference: calculate_patch_layout of
    openmini-server/src/model/inference/vision/pan_scan.rs:39-82."""
    if width <= base_size and height <= base_size:
        return [(0, 0, width, height)]
    step = max(1, base_size - overlap)
    return [(x, y, min(base_size, width - x), min(base_size, height - y))
            for y in range(0, height, step) for x in range(0, width, step)]


def pan_and_scan(image, cfg: "VisionConfig", base_size: int = 896, overlap: int = 14, max_tokens: int = 16384,
                 include_global: bool = True) -> list:
    """[H, W, 3] image -> list of crops [h, w, 3] to encode: the whole image first (when
    ``include_global`` and it is tiled), then the tiles of ``pan_scan_layout`` in row
    order, stopping before the encoder tokens (``cfg.num_patches`` per crop) would pass
    ``max_tokens``. Each crop is resized to the encoder's input by ``preprocess``."""
    x = torch.as_tensor(image)
    H, W = int(x.shape[0]), int(x.shape[1])
    tiles = pan_scan_layout(W, H, base_size, overlap)
    crops = [x] if include_global and len(tiles) > 1 else []
    crops += [x[ty:ty + th, tx:tx + tw] for tx, ty, tw, th in tiles]
    keep = max(1, max_tokens // cfg.num_patches)
    return crops[:keep]


def splice_image(prompt_ids: list, image_token_id: int, num_patches: int) -> tuple:
    """Expand the single ``image_token_id`` of a prompt into ``num_patches`` placeholder
    positions. Returns (ids, rows): the rows whose embeddings the image features replace."""
    i = prompt_ids.index(image_token_id)
    ids = prompt_ids[:i] + [image_token_id] * num_patches + prompt_ids[i + 1:]
    return ids, list(range(i, i + num_patches))
