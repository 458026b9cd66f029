"""Training control REST API: /api/v1/training/{start,pause,resume,stop,status,metrics}.

``start`` builds a :class:`~openmini_v1_b200.train.trainer.Trainer` through the
server's ``trainer_factory(body)`` and runs ``train()`` in a background thread;
the other routes drive and observe it. One training run at a time.

Reference: openmini-server/src/api/training.rs:40-48 (routes declared there but
not compiled into the server).
"""
from __future__ import annotations

import threading

from fastapi import FastAPI, HTTPException, Request


def mount_training(app: FastAPI, trainer_factory):
    run = {"trainer": None, "thread": None, "error": None}

    def _cur():
        t = run["trainer"]
        if t is None:
            raise HTTPException(404, "no training run")
        return t

    @app.post("/api/v1/training/start")
    async def start(req: Request):
        if run["thread"] is not None and run["thread"].is_alive():
            raise HTTPException(409, "a training run is active")
        body = await req.json() if (await req.body()) else {}
        if trainer_factory is None:
            raise HTTPException(501, "this server has no training data / model configured")
        t = trainer_factory(body)
        run.update(trainer=t, error=None)

        def go():
            try:
                t.train()
            except Exception as e:  # surfaced through /status
                run["error"] = repr(e)
                t.state.status = "failed"

        th = threading.Thread(target=go, daemon=True, name="trainer")
        run["thread"] = th
        th.start()
        return {"status": "started", "total_steps": t.total_steps}

    @app.post("/api/v1/training/pause")
    async def pause():
        _cur().pause()
        return {"status": _cur().state.status}

    @app.post("/api/v1/training/resume")
    async def resume():
        _cur().resume()
        return {"status": _cur().state.status}

    @app.post("/api/v1/training/stop")
    async def stop():
        t = _cur()
        t.stop()
        if run["thread"] is not None:
            run["thread"].join(timeout=30)
        return {"status": t.state.status}

    @app.get("/api/v1/training/status")
    async def status():
        s = _cur().status()
        s["error"] = run["error"]
        return s

    @app.get("/api/v1/training/metrics")
    async def metrics():
        h = _cur().state.history
        return {"history": h[-200:], "last_loss": _cur().state.last_loss, "lr": _cur().state.lr}
