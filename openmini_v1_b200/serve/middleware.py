"""HTTP middleware: request id + access log with secrets masked, CORS, request
body limit and per-request timeout.

Reference: openmini-server/src/service/http/middleware.rs:23-153 (logging,
CORS, RequestBodyLimitLayer, TimeoutLayer -> 408) and sensitive_filter.rs
(API keys, bearer tokens, passwords and "sk-" keys masked before logging).
"""
from __future__ import annotations

import asyncio
import re
import time
import uuid

from fastapi import FastAPI
from fastapi.middleware.cors import CORSMiddleware
from starlette.responses import JSONResponse

# bearer tokens first, so "Authorization: Bearer <tok>" loses the token and not only the word "Bearer"
_SENSITIVE = [
    re.compile(r"(?i)Bearer\s+\S+"),
    re.compile(r"(?i)sk-[a-zA-Z0-9]{20,}"),
    re.compile(r"(?i)(api[_\-]?key|authorization|token|password|secret|apikey)[=:]\s*\S+"),
]
MASK = "***MASKED***"


def mask_sensitive_data(text: str) -> str:
    for p in _SENSITIVE:
        text = p.sub(MASK, text)
    return text


def apply_middlewares(app: FastAPI, log=None, cors_origins=None, max_body_bytes: int = 10 * 1024 * 1024,
                      request_timeout_s: float = 300.0):
    app.add_middleware(CORSMiddleware, allow_origins=cors_origins or ["*"], allow_methods=["*"],
                       allow_headers=["*"])

    @app.middleware("http")
    async def _limits_and_log(request, call_next):
        rid = request.headers.get("x-request-id") or uuid.uuid4().hex
        n = request.headers.get("content-length")
        if n is not None and n.isdigit() and int(n) > max_body_bytes:
            return JSONResponse({"error": "request body too large"}, status_code=413,
                                headers={"x-request-id": rid})
        t0 = time.time()
        try:
            resp = await asyncio.wait_for(call_next(request), timeout=request_timeout_s)
        except asyncio.TimeoutError:
            resp = JSONResponse({"error": "request timed out"}, status_code=408)
        resp.headers["x-request-id"] = rid
        if log is not None:
            auth = request.headers.get("authorization")
            log("http", request_id=rid, method=request.method, path=request.url.path, status=resp.status_code,
                ms=round((time.time() - t0) * 1e3, 2), authorization=mask_sensitive_data(auth) if auth else None,
                query=mask_sensitive_data(str(request.url.query)) if request.url.query else None)
        return resp

    return app
