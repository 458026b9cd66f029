"""Supervised training on CPU: safetensors format, LR schedules, SFT data
masking, a trainer that lowers the loss, checkpoint keep-last-N and exact
resume, and data-parallel gradient averaging on 2 gloo ranks."""
import json
import os
import socket
import struct

import torch
import torch.multiprocessing as mp

from openmini_v1_b200.engine.tokenizer import ByteTokenizer
from openmini_v1_b200.models.config import ModelConfig
from openmini_v1_b200.models.policy import Policy
from openmini_v1_b200.train.data import DataLoader, TokenizedDataset
from openmini_v1_b200.train.loss import IGNORE, causal_lm_loss
from openmini_v1_b200.train.optim import CosineWithWarmup, LinearWithWarmup
from openmini_v1_b200.train.safetensors import load_file, save_file
from openmini_v1_b200.train.trainer import Trainer, TrainingConfig


def _cfg():
    return ModelConfig(name="t", vocab_size=259, hidden_size=32, num_layers=1, num_heads=2, num_kv_heads=1,
                       head_dim=16, intermediate_size=64, dtype="float32")


def test_safetensors_roundtrip(tmp_path):
    t = {"a": torch.randn(3, 4), "b": torch.arange(5, dtype=torch.int64), "c": torch.randn(2, 2).bfloat16()}
    p = str(tmp_path / "x.safetensors")
    save_file(t, p, {"k": "v"})
    raw = open(p, "rb").read()
    (n,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + n])
    assert hdr["a"]["dtype"] == "F32" and hdr["a"]["shape"] == [3, 4] and hdr["__metadata__"] == {"k": "v"}
    assert hdr["c"]["dtype"] == "BF16"
    back = load_file(p)
    for k in t:
        assert torch.equal(back[k], t[k])


def test_schedules():
    c = CosineWithWarmup(10, 110, 1e-6, 1e-3)
    assert c.get_lr(0) == 0.0 and abs(c.get_lr(5) - 5e-4) < 1e-12
    assert abs(c.get_lr(10) - 1e-3) < 1e-12 and abs(c.get_lr(110) - 1e-6) < 1e-12
    assert abs(c.get_lr(60) - (1e-6 + 0.5 * (1e-3 - 1e-6))) < 1e-12
    lin = LinearWithWarmup(10, 110, 0.0, 1.0)
    assert lin.get_lr(60) == 0.5 and lin.get_lr(500) == 0.0


def test_sft_masking():
    tok = ByteTokenizer()
    ds = TokenizedDataset([{"prompt": "hi", "response": "yo"}, {"text": "plain text"}], tok, 64)
    ids, labels = ds.samples[0]
    n_resp = len("yo") + 1  # + eos
    assert labels[-n_resp:] == ids[-n_resp:] and all(x == IGNORE for x in labels[:-n_resp])
    assert ds.samples[1][0] == ds.samples[1][1]
    lg = torch.zeros(1, 4, 10)
    assert float(causal_lm_loss(lg, torch.full((1, 4), IGNORE))) == 0.0


def _data(n=24):
    tok = ByteTokenizer()
    recs = [{"prompt": f"q{i % 3}", "response": "abcabc"} for i in range(n)]
    return TokenizedDataset(recs, tok, 64)


def test_trainer_learns_checkpoints_and_resumes(tmp_path):
    torch.manual_seed(0)
    ds = _data()
    cfg = TrainingConfig(num_train_epochs=4, per_device_train_batch_size=4, gradient_accumulation_steps=2,
                         learning_rate=1e-2, warmup_steps=2, output_dir=str(tmp_path / "ck"), save_steps=3,
                         save_total_limit=2, logging_steps=1, lr_scheduler="cosine")
    m = Policy(_cfg(), seed=1)
    tr = Trainer(m, cfg, DataLoader(ds, 4, seed=1), DataLoader(ds, 8, shuffle=False))
    first = tr.evaluate()
    st = tr.train()
    assert st.status == "finished" and st.global_step == 12
    assert tr.evaluate() < first * 0.8
    dirs = sorted(d for d in os.listdir(tmp_path / "ck") if d.startswith("checkpoint_"))
    assert len(dirs) <= 3  # keep-last-2 plus the best
    assert {"training_state.json", "optimizer_state.bin", "model.safetensors"} <= set(
        os.listdir(tmp_path / "ck" / dirs[-1]))
    # resume: a fresh trainer loads the latest checkpoint exactly
    m2 = Policy(_cfg(), seed=7)
    tr2 = Trainer(m2, cfg, DataLoader(ds, 4, seed=1))
    assert tr2.resume_from_checkpoint()
    assert tr2.state.global_step == 12
    for (k, a), (_, b) in zip(m.state_dict().items(), m2.state_dict().items()):
        assert torch.equal(a, b), k


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dp_worker(rank, world, port, q):
    import torch.distributed as dist
    from openmini_v1_b200.train.ddp import GradReducer
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        m = Policy(_cfg(), seed=1)
        red = GradReducer(m.parameters(), bucket_mb=0.01)
        ids = torch.randint(0, 259, (2, 9), generator=torch.Generator().manual_seed(rank))
        red.begin(True)
        causal_lm_loss(m(ids), ids).backward()
        red.finish()
        g = torch.cat([p.grad.reshape(-1) for p in m.parameters()])
        q.put((rank, g))
    finally:
        dist.destroy_process_group()


def test_dp_grad_average():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    # reference: average of the two ranks' single-process gradients
    grads = []
    for r in range(world):
        torch.manual_seed(0)
        m = Policy(_cfg(), seed=1)
        ids = torch.randint(0, 259, (2, 9), generator=torch.Generator().manual_seed(r))
        causal_lm_loss(m(ids), ids).backward()
        grads.append(torch.cat([p.grad.reshape(-1) for p in m.parameters()]))
    want = (grads[0] + grads[1]) / 2
    assert torch.allclose(res[0], want, atol=1e-6) and torch.allclose(res[1], want, atol=1e-6)


def test_training_rest_api(tmp_path):
    import time
    from fastapi import FastAPI
    from fastapi.testclient import TestClient
    from openmini_v1_b200.serve.training_api import mount_training

    def factory(body):
        ds = _data(8)
        cfg = TrainingConfig(num_train_epochs=int(body.get("epochs", 50)), per_device_train_batch_size=4,
                             output_dir=str(tmp_path / "api"), save_steps=0, logging_steps=1)
        return Trainer(Policy(_cfg(), seed=2), cfg, DataLoader(ds, 4))

    app = FastAPI()
    mount_training(app, factory)
    c = TestClient(app)
    assert c.get("/api/v1/training/status").status_code == 404
    assert c.post("/api/v1/training/start", json={"epochs": 50}).json()["status"] == "started"
    time.sleep(0.5)
    c.post("/api/v1/training/pause")
    time.sleep(0.2)
    s1 = c.get("/api/v1/training/status").json()
    time.sleep(0.3)
    s2 = c.get("/api/v1/training/status").json()
    assert s1["status"] == "paused" and s1["global_step"] == s2["global_step"]
    c.post("/api/v1/training/resume")
    assert c.post("/api/v1/training/stop").json()["status"] in ("stopped", "finished")
    m = c.get("/api/v1/training/metrics").json()
    assert len(m["history"]) > 0
