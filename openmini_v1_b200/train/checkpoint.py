"""Training checkpoints.

Layout (same directory and file names as the reference's CheckpointManager,
openmini-server/src/training/checkpoint.rs:45-240, so tooling that looks for
them keeps working):

    <output_dir>/checkpoint_<step:08>/training_state.json   epoch, global_step, losses, lr, config
    <output_dir>/checkpoint_<step:08>/optimizer_state.bin   optimizer + scaler + RNG state (torch.save)
    <output_dir>/checkpoint_<step:08>/model.safetensors     fp32 master weights

``save_total_limit`` keeps the newest N checkpoints (the best one by validation
loss is never deleted). ``load_latest`` / ``load`` restore everything needed to
resume bit-exactly on the same world size.
"""
from __future__ import annotations

import json
import os
import shutil
import time

import torch

from .safetensors import load_file, save_file


class CheckpointManager:
    def __init__(self, output_dir: str, save_total_limit: int = 5):
        self.output_dir = output_dir
        self.save_total_limit = save_total_limit
        os.makedirs(output_dir, exist_ok=True)
        self.checkpoints = self._scan()
        self.best = None  # (val_loss, path)
        for c in self.checkpoints:
            vl = c.get("val_loss")
            if vl is not None and (self.best is None or vl < self.best[0]):
                self.best = (vl, c["path"])

    def _scan(self):
        out = []
        for d in sorted(os.listdir(self.output_dir)):
            p = os.path.join(self.output_dir, d)
            f = os.path.join(p, "training_state.json")
            if d.startswith("checkpoint_") and os.path.isfile(f):
                with open(f) as fh:
                    st = json.load(fh)
                out.append({"path": p, "step": st.get("global_step", 0), "val_loss": st.get("val_loss")})
        out.sort(key=lambda c: c["step"])
        return out

    def save(self, model, optimizer, state: dict, extra: dict | None = None, val_loss: float | None = None) -> str:
        step = int(state["global_step"])
        path = os.path.join(self.output_dir, f"checkpoint_{step:08d}")
        tmp = path + ".partial"
        if os.path.exists(tmp):
            shutil.rmtree(tmp)
        os.makedirs(tmp)
        st = dict(state)
        st["val_loss"] = val_loss
        st["created_at"] = time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())
        with open(os.path.join(tmp, "training_state.json"), "w") as f:
            json.dump(st, f, indent=2)
        weights = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
        save_file(weights, os.path.join(tmp, "model.safetensors"), {"global_step": step})
        blob = {"optimizer": optimizer.state_dict() if optimizer is not None else None,
                "torch_rng": torch.get_rng_state(), "extra": extra or {}}
        if torch.cuda.is_available():
            blob["cuda_rng"] = torch.cuda.get_rng_state_all()
        torch.save(blob, os.path.join(tmp, "optimizer_state.bin"))
        if os.path.exists(path):
            shutil.rmtree(path)
        os.replace(tmp, path)
        self.checkpoints = [c for c in self.checkpoints if c["path"] != path]
        self.checkpoints.append({"path": path, "step": step, "val_loss": val_loss})
        if val_loss is not None and (self.best is None or val_loss < self.best[0]):
            self.best = (val_loss, path)
        self._cleanup()
        return path

    def _cleanup(self):
        while len(self.checkpoints) > self.save_total_limit:
            victim = next((c for c in self.checkpoints if not (self.best and c["path"] == self.best[1])), None)
            if victim is None:
                break
            shutil.rmtree(victim["path"], ignore_errors=True)
            self.checkpoints.remove(victim)

    def latest(self) -> str | None:
        return self.checkpoints[-1]["path"] if self.checkpoints else None

    def load(self, path: str, model=None, optimizer=None, map_location="cpu") -> dict:
        with open(os.path.join(path, "training_state.json")) as f:
            state = json.load(f)
        if model is not None:
            w = load_file(os.path.join(path, "model.safetensors"))
            sd = model.state_dict()
            for k, v in sd.items():
                if k not in w:
                    raise KeyError(f"checkpoint {path} misses {k}")
                v.copy_(w[k].to(v.dtype))
        blob = torch.load(os.path.join(path, "optimizer_state.bin"), map_location=map_location, weights_only=False)
        if optimizer is not None and blob.get("optimizer") is not None:
            optimizer.load_state_dict(blob["optimizer"])
        torch.set_rng_state(blob["torch_rng"])
        if "cuda_rng" in blob and torch.cuda.is_available():
            torch.cuda.set_rng_state_all(blob["cuda_rng"])
        state["extra"] = blob.get("extra", {})
        return state

    def load_latest(self, model=None, optimizer=None) -> dict | None:
        p = self.latest()
        return self.load(p, model, optimizer) if p else None
