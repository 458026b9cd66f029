"""Vision encoder: preprocessing shapes, the encoder against an independent
torch.nn.functional statement of the same ViT, and image features spliced into
the language model's embeddings."""
import math

import torch
import torch.nn.functional as F

from openmini_v1_b200.models.config import tiny
from openmini_v1_b200.models.llama import DecoderLM, ForwardBatch
from openmini_v1_b200.models.vision import VisionConfig, VisionEncoder, preprocess, splice_image


def _ref(enc, patches):
    c = enc.cfg
    x = patches.float() @ enc.patch_w.float().t() + enc.pos.float()
    for L in enc.layers:
        a = F.layer_norm(x, (c.hidden_size,), L["ln1_w"].float(), L["ln1_b"].float(), c.ln_eps)
        qkv = a @ L["qkv"].float().t()
        q, k, v = qkv.split(c.hidden_size, -1)
        sh = lambda t: t.view(-1, c.num_heads, c.head_dim).transpose(0, 1)  # noqa: E731
        o = F.scaled_dot_product_attention(sh(q), sh(k), sh(v)).transpose(0, 1).reshape(-1, c.hidden_size)
        x = x + o @ L["o"].float().t()
        m = F.layer_norm(x, (c.hidden_size,), L["ln2_w"].float(), L["ln2_b"].float(), c.ln_eps)
        x = x + F.gelu(m @ L["fc1"].float().t(), approximate="tanh") @ L["fc2"].float().t()
    x = F.layer_norm(x, (c.hidden_size,), enc.post_w.float(), enc.post_b.float(), c.ln_eps)
    return x @ enc.proj.float().t()


def test_vision_encoder_and_splice():
    cfg = VisionConfig(image_size=64, patch_size=16, hidden_size=256, num_layers=2, num_heads=2, mlp_size=512,
                       lm_hidden=256)
    enc = VisionEncoder(cfg, dtype=torch.float32, seed=1)
    img = (torch.rand(50, 70, 3) * 255).to(torch.uint8)
    patches = preprocess(img, cfg)
    assert patches.shape == (1, 16, 3 * 16 * 16) and patches.min() >= -1.001 and patches.max() <= 1.001
    feats = enc(img)[0]
    assert feats.shape == (16, 256)
    assert torch.allclose(feats, _ref(enc, patches[0]), atol=1e-4)
    # splice into the LM
    lm = DecoderLM(tiny(), device="cpu", seed=0, dtype=torch.float32)
    ids, rows = splice_image([5, 7, 999, 9], 999, 16)
    assert len(ids) == 19 and rows == list(range(2, 18))
    T = len(ids)
    i32 = dict(dtype=torch.int32)
    mk = lambda ov: ForwardBatch(torch.tensor(ids, **i32), torch.arange(T, **i32), torch.arange(T, **i32),  # noqa
                                 torch.arange(2, **i32)[None], torch.zeros(T, **i32), torch.arange(1, T + 1, **i32),
                                 T, torch.tensor([T - 1]), embed_override=ov)
    plain = lm.logits(lm(mk(None), lm.allocate_kv(2)))
    withimg = lm.logits(lm(mk((torch.tensor(rows), feats)), lm.allocate_kv(2)))
    assert not torch.allclose(plain, withimg)
    assert math.isfinite(float(withimg.sum()))
