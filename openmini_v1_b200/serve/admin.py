"""Admin service: users with roles (RBAC), signed session tokens, API keys, audit log,
alert rules, SLA tracking, model / session / config administration.

Reference counterparts: the admin REST surface ``/admin/{service,model,sessions,
metrics,apikeys,users,alerts,audit,config,auth}`` (openmini-admin/src/api/mod.rs:20-205)
with JWT auth and SQLite storage, and the enterprise module (RBAC, audit log, SLA
monitor; openmini-server/src/enterprise/*). OAuth2 / OIDC federation needs an
external identity provider and is not part of this server.

Storage is SQLite (stdlib ``sqlite3``, WAL when on disk). Tokens are
``base64(payload).hmac_sha256`` with an expiry, verified with ``hmac.compare_digest``.
Passwords and API keys are stored as salted PBKDF2 / SHA-256 digests only.

Roles: ``admin`` (everything), ``operator`` (model, sessions, alerts, service
actions), ``viewer`` (read-only). Every mutating call is written to the audit log.
"""
from __future__ import annotations

import base64
import hashlib
import hmac
import json
import os
import secrets
import sqlite3
import threading
import time
from dataclasses import dataclass

from fastapi import APIRouter, Depends, FastAPI, Header, HTTPException, Request

ROLES = {"admin": 3, "operator": 2, "viewer": 1}


def _hash_pw(pw: str, salt: bytes | None = None) -> str:
    salt = salt or os.urandom(16)
    return salt.hex() + "$" + hashlib.pbkdf2_hmac("sha256", pw.encode(), salt, 100_000).hex()


def _check_pw(pw: str, stored: str) -> bool:
    salt, _ = stored.split("$", 1)
    return hmac.compare_digest(_hash_pw(pw, bytes.fromhex(salt)), stored)


class AdminStore:
    def __init__(self, path: str = ":memory:"):
        self.db = sqlite3.connect(path, check_same_thread=False)
        self.lock = threading.Lock()
        with self.lock:
            if path != ":memory:":
                self.db.execute("PRAGMA journal_mode=WAL")
            self.db.executescript("""
                CREATE TABLE IF NOT EXISTS users (name TEXT PRIMARY KEY, pw TEXT, role TEXT, created REAL);
                CREATE TABLE IF NOT EXISTS apikeys (id TEXT PRIMARY KEY, digest TEXT, owner TEXT, role TEXT,
                                                    created REAL, revoked INTEGER DEFAULT 0);
                CREATE TABLE IF NOT EXISTS audit (ts REAL, actor TEXT, action TEXT, target TEXT, detail TEXT);
                CREATE TABLE IF NOT EXISTS alerts (id INTEGER PRIMARY KEY AUTOINCREMENT, name TEXT, metric TEXT,
                                                   op TEXT, threshold REAL, enabled INTEGER DEFAULT 1);
            """)
            self.db.commit()

    def q(self, sql, args=()):
        with self.lock:
            cur = self.db.execute(sql, args)
            self.db.commit()
            return cur.fetchall()

    def audit(self, actor, action, target="", detail=None):
        self.q("INSERT INTO audit VALUES (?, ?, ?, ?, ?)",
               (time.time(), actor, action, target, json.dumps(detail or {})))


@dataclass
class Principal:
    name: str
    role: str


class SLAMonitor:
    """Rolling window of request latencies against a p99 target and an error-rate target."""

    def __init__(self, p99_ms: float = 2000.0, max_error_rate: float = 0.01, window: int = 1000):
        self.p99_ms, self.max_error_rate, self.window = p99_ms, max_error_rate, window
        self.lat, self.err = [], []

    def record(self, latency_ms: float, ok: bool = True):
        self.lat.append(latency_ms)
        self.err.append(0 if ok else 1)
        del self.lat[:-self.window], self.err[:-self.window]

    def report(self) -> dict:
        if not self.lat:
            return {"requests": 0, "compliant": True}
        s = sorted(self.lat)
        p99 = s[min(len(s) - 1, int(0.99 * (len(s) - 1) + 0.5))]
        er = sum(self.err) / len(self.err)
        return {"requests": len(s), "p99_ms": p99, "error_rate": er, "p99_target_ms": self.p99_ms,
                "compliant": p99 <= self.p99_ms and er <= self.max_error_rate}


class AdminService:
    def __init__(self, secret: bytes | None = None, store: AdminStore | None = None, token_ttl_s: int = 3600,
                 bootstrap_admin: tuple | None = ("admin", "admin")):
        self.secret = secret or secrets.token_bytes(32)
        self.store = store or AdminStore()
        self.ttl = token_ttl_s
        self.sla = SLAMonitor()
        self.hooks = {}  # "model_status", "model_reload", "sessions", "metrics", "config", "service_action"
        self.oidc = None  # serve.oidc.OIDCVerifier: bearer JWTs from an identity provider
        self.oidc_login = None  # serve.oidc.OIDCLogin: browser login through the provider
        if bootstrap_admin and not self.store.q("SELECT 1 FROM users"):
            self.create_user(*bootstrap_admin, role="admin", actor="bootstrap")

    # ------------------------------------------------------------------ identities
    def create_user(self, name, pw, role="viewer", actor="system"):
        if role not in ROLES:
            raise ValueError(f"unknown role {role}")
        self.store.q("INSERT INTO users VALUES (?, ?, ?, ?)", (name, _hash_pw(pw), role, time.time()))
        self.store.audit(actor, "user.create", name, {"role": role})

    def issue_token(self, name: str, role: str) -> str:
        body = base64.urlsafe_b64encode(json.dumps({"sub": name, "role": role,
                                                    "exp": time.time() + self.ttl}).encode()).decode()
        sig = hmac.new(self.secret, body.encode(), hashlib.sha256).hexdigest()
        return f"{body}.{sig}"

    def verify_token(self, token: str) -> Principal | None:
        try:
            body, sig = token.rsplit(".", 1)
        except ValueError:
            return None
        if not hmac.compare_digest(hmac.new(self.secret, body.encode(), hashlib.sha256).hexdigest(), sig):
            return None
        p = json.loads(base64.urlsafe_b64decode(body.encode()))
        if p["exp"] < time.time():
            return None
        return Principal(p["sub"], p["role"])

    def login(self, name, pw) -> str | None:
        rows = self.store.q("SELECT pw, role FROM users WHERE name=?", (name,))
        if not rows or not _check_pw(pw, rows[0][0]):
            self.store.audit(name, "auth.fail")
            return None
        self.store.audit(name, "auth.login")
        return self.issue_token(name, rows[0][1])

    def create_apikey(self, owner: str, role: str) -> tuple:
        kid = secrets.token_hex(6)
        key = f"om-{kid}-{secrets.token_urlsafe(24)}"
        self.store.q("INSERT INTO apikeys VALUES (?, ?, ?, ?, ?, 0)",
                     (kid, hashlib.sha256(key.encode()).hexdigest(), owner, role, time.time()))
        return kid, key

    def check_apikey(self, key: str) -> Principal | None:
        parts = key.split("-")
        if len(parts) < 3 or parts[0] != "om":
            return None
        rows = self.store.q("SELECT digest, owner, role, revoked FROM apikeys WHERE id=?", (parts[1],))
        if not rows or rows[0][3] or not hmac.compare_digest(rows[0][0], hashlib.sha256(key.encode()).hexdigest()):
            return None
        return Principal(rows[0][1], rows[0][2])

    # ------------------------------------------------------------------ alerts
    def evaluate_alerts(self, metrics: dict) -> list:
        fired = []
        for aid, name, metric, op, thr, en in self.store.q("SELECT * FROM alerts"):
            v = metrics.get(metric)
            if not en or v is None:
                continue
            if (op == ">" and v > thr) or (op == "<" and v < thr) or (op == ">=" and v >= thr) or (
                    op == "<=" and v <= thr):
                fired.append({"id": aid, "name": name, "metric": metric, "value": v, "threshold": thr})
        return fired

    def _oidc_principal(self, tok: str):
        from .oidc import OIDCError
        try:
            claims = self.oidc.verify(tok)
        except OIDCError:
            return None
        role = self.oidc.role_of(claims)
        if role is None:
            return None
        return Principal(claims.get("preferred_username") or claims.get("email") or claims.get("sub", "oidc"), role)

    # ------------------------------------------------------------------ HTTP
    def principal(self, authorization: str | None = Header(None), x_api_key: str | None = Header(None)):
        p = None
        if authorization and authorization.lower().startswith("bearer "):
            tok = authorization[7:]
            p = self.verify_token(tok)
            if p is None and self.oidc is not None and tok.count(".") == 2:
                p = self._oidc_principal(tok)
        elif x_api_key:
            p = self.check_apikey(x_api_key)
        if p is None:
            raise HTTPException(401, "authentication required")
        return p

    def require(self, role: str):
        def dep(p: Principal = Depends(self.principal)):
            if ROLES.get(p.role, 0) < ROLES[role]:
                raise HTTPException(403, f"{role} role required")
            return p
        return dep

    def router(self) -> APIRouter:
        r = APIRouter(prefix="/admin")
        view, oper, admin = self.require("viewer"), self.require("operator"), self.require("admin")

        @r.post("/auth/login")
        async def login(body: dict):
            tok = self.login(body.get("username", ""), body.get("password", ""))
            if tok is None:
                raise HTTPException(401, "bad credentials")
            return {"token": tok, "expires_in": self.ttl}

        @r.get("/auth/oidc/login")
        async def oidc_login():
            """Redirect the browser to the identity provider (authorization-code flow, PKCE)."""
            if self.oidc_login is None:
                raise HTTPException(404, "OIDC login is not configured")
            from fastapi.responses import RedirectResponse
            url, _ = self.oidc_login.start()
            return RedirectResponse(url, status_code=302)

        @r.get("/auth/oidc/callback")
        async def oidc_callback(code: str = "", state: str = "", error: str = ""):
            """The provider's redirect: exchange the code, verify the ID token, issue a session token."""
            if self.oidc_login is None:
                raise HTTPException(404, "OIDC login is not configured")
            if error or not code:
                raise HTTPException(400, f"login failed at the provider: {error or 'no code'}")
            import asyncio
            from .oidc import OIDCError
            try:
                claims = await asyncio.to_thread(self.oidc_login.finish, code, state)
            except OIDCError as e:
                self.store.audit("oidc", "auth.fail", "", {"reason": str(e)})
                raise HTTPException(400, str(e))
            role = self.oidc_login.verifier.role_of(claims)
            name = claims.get("preferred_username") or claims.get("email") or claims.get("sub", "oidc")
            if role is None:
                self.store.audit(name, "auth.fail", "", {"reason": "no role"})
                raise HTTPException(403, "the identity provider grants this user no admin role")
            self.store.audit(name, "auth.oidc", "", {"role": role})
            return {"token": self.issue_token(name, role), "expires_in": self.ttl, "user": name, "role": role}

        @r.get("/auth/me")
        async def me(p: Principal = Depends(view)):
            return {"user": p.name, "role": p.role}

        @r.get("/users")
        async def users(p: Principal = Depends(admin)):
            return [{"name": n, "role": ro, "created": c} for n, ro, c in
                    self.store.q("SELECT name, role, created FROM users")]

        @r.post("/users")
        async def add_user(body: dict, p: Principal = Depends(admin)):
            try:
                self.create_user(body["username"], body["password"], body.get("role", "viewer"), actor=p.name)
            except (sqlite3.IntegrityError, ValueError, KeyError) as e:
                raise HTTPException(400, str(e))
            return {"ok": True}

        @r.delete("/users/{name}")
        async def del_user(name: str, p: Principal = Depends(admin)):
            self.store.q("DELETE FROM users WHERE name=?", (name,))
            self.store.audit(p.name, "user.delete", name)
            return {"ok": True}

        @r.get("/apikeys")
        async def keys(p: Principal = Depends(admin)):
            return [{"id": i, "owner": o, "role": ro, "created": c, "revoked": bool(rv)} for i, o, ro, c, rv in
                    self.store.q("SELECT id, owner, role, created, revoked FROM apikeys")]

        @r.post("/apikeys")
        async def new_key(body: dict, p: Principal = Depends(admin)):
            role = body.get("role", "viewer")
            if role not in ROLES:
                raise HTTPException(400, "unknown role")
            kid, key = self.create_apikey(body.get("owner", p.name), role)
            self.store.audit(p.name, "apikey.create", kid, {"role": role})
            return {"id": kid, "key": key}

        @r.delete("/apikeys/{kid}")
        async def revoke(kid: str, p: Principal = Depends(admin)):
            self.store.q("UPDATE apikeys SET revoked=1 WHERE id=?", (kid,))
            self.store.audit(p.name, "apikey.revoke", kid)
            return {"ok": True}

        @r.get("/audit")
        async def audit(limit: int = 100, p: Principal = Depends(admin)):
            rows = self.store.q("SELECT ts, actor, action, target, detail FROM audit ORDER BY ts DESC LIMIT ?",
                                (limit,))
            return [{"ts": t, "actor": a, "action": ac, "target": tg, "detail": json.loads(d)}
                    for t, a, ac, tg, d in rows]

        @r.get("/alerts")
        async def alerts(p: Principal = Depends(view)):
            rules = [{"id": i, "name": n, "metric": m, "op": o, "threshold": t, "enabled": bool(e)}
                     for i, n, m, o, t, e in self.store.q("SELECT * FROM alerts")]
            metrics = self.hooks["metrics"]() if "metrics" in self.hooks else {}
            return {"rules": rules, "firing": self.evaluate_alerts(metrics)}

        @r.post("/alerts")
        async def add_alert(body: dict, p: Principal = Depends(oper)):
            if body.get("op") not in (">", "<", ">=", "<="):
                raise HTTPException(400, "op must be one of > < >= <=")
            self.store.q("INSERT INTO alerts (name, metric, op, threshold) VALUES (?, ?, ?, ?)",
                         (body["name"], body["metric"], body["op"], float(body["threshold"])))
            self.store.audit(p.name, "alert.create", body["name"], body)
            return {"ok": True}

        @r.get("/metrics")
        async def metrics(p: Principal = Depends(view)):
            m = self.hooks["metrics"]() if "metrics" in self.hooks else {}
            return {"metrics": m, "sla": self.sla.report()}

        @r.get("/service")
        async def service(p: Principal = Depends(view)):
            return {"uptime_s": time.monotonic(), "sla": self.sla.report(),
                    "model": self.hooks["model_status"]() if "model_status" in self.hooks else None}

        @r.post("/service/{action}")
        async def service_action(action: str, p: Principal = Depends(oper)):
            if "service_action" not in self.hooks:
                raise HTTPException(501, "no service controller attached")
            out = self.hooks["service_action"](action)
            self.store.audit(p.name, f"service.{action}")
            return out

        @r.get("/model")
        async def model(p: Principal = Depends(view)):
            return self.hooks["model_status"]() if "model_status" in self.hooks else {}

        @r.post("/model/reload")
        async def reload(body: dict, p: Principal = Depends(oper)):
            if "model_reload" not in self.hooks:
                raise HTTPException(501, "no hot reloader attached")
            out = self.hooks["model_reload"](body)
            self.store.audit(p.name, "model.reload", body.get("name", ""), body)
            return out

        @r.get("/sessions")
        async def sessions(p: Principal = Depends(view)):
            return self.hooks["sessions"]() if "sessions" in self.hooks else []

        @r.get("/config")
        async def config(p: Principal = Depends(view)):
            return self.hooks["config"]() if "config" in self.hooks else {}

        return r

    def mount(self, app: FastAPI):
        app.include_router(self.router())

        @app.get("/admin/ui")
        async def admin_ui():
            """Static single-page admin console over the /admin REST API (no build step)."""
            from fastapi.responses import HTMLResponse
            import pathlib
            return HTMLResponse((pathlib.Path(__file__).parent / "static" / "admin.html").read_text())

        @app.middleware("http")
        async def _sla(request: Request, call_next):
            t0 = time.perf_counter()
            resp = await call_next(request)
            if not request.url.path.startswith("/admin"):
                self.sla.record((time.perf_counter() - t0) * 1e3, resp.status_code < 500)
            return resp
        return app
