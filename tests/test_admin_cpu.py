"""Admin service: login tokens, RBAC, API keys (create / use / revoke), audit log,
alert rules against live metrics, SLA report, hooks for model reload and sessions."""
from fastapi import FastAPI
from fastapi.testclient import TestClient

from openmini_v1_b200.serve.admin import AdminService, SLAMonitor


def test_admin_rbac_keys_audit_alerts():
    svc = AdminService(secret=b"k" * 32)
    reloads = []
    svc.hooks.update(metrics=lambda: {"queue_length": 12.0, "p99_ms": 50.0},
                     model_reload=lambda body: reloads.append(body) or {"version": 2},
                     sessions=lambda: [{"id": "s1"}], model_status=lambda: {"name": "tiny"})
    app = FastAPI()

    @app.get("/ping")
    async def ping():
        return {"ok": 1}

    svc.mount(app)
    c = TestClient(app)
    assert c.get("/admin/users").status_code == 401
    assert c.post("/admin/auth/login", json={"username": "admin", "password": "bad"}).status_code == 401
    tok = c.post("/admin/auth/login", json={"username": "admin", "password": "admin"}).json()["token"]
    A = {"Authorization": f"Bearer {tok}"}
    assert c.get("/admin/auth/me", headers=A).json() == {"user": "admin", "role": "admin"}
    assert c.post("/admin/users", json={"username": "op", "password": "pw", "role": "operator"}, headers=A).json()
    assert c.post("/admin/users", json={"username": "v", "password": "pw", "role": "viewer"}, headers=A).json()
    assert c.post("/admin/users", json={"username": "x", "password": "pw", "role": "god"},
                  headers=A).status_code == 400
    vt = c.post("/admin/auth/login", json={"username": "v", "password": "pw"}).json()["token"]
    V = {"Authorization": f"Bearer {vt}"}
    assert c.get("/admin/model", headers=V).json() == {"name": "tiny"}
    assert c.post("/admin/model/reload", json={"name": "m2"}, headers=V).status_code == 403
    assert c.get("/admin/users", headers=V).status_code == 403
    # API key with operator role
    k = c.post("/admin/apikeys", json={"owner": "ci", "role": "operator"}, headers=A).json()
    K = {"X-API-Key": k["key"]}
    assert c.post("/admin/model/reload", json={"name": "m2"}, headers=K).json() == {"version": 2}
    assert reloads == [{"name": "m2"}]
    assert c.post("/admin/alerts", json={"name": "q", "metric": "queue_length", "op": ">", "threshold": 10},
                  headers=K).json()
    al = c.get("/admin/alerts", headers=V).json()
    assert al["firing"] and al["firing"][0]["name"] == "q"
    assert c.delete(f"/admin/apikeys/{k['id']}", headers=A).json()
    assert c.post("/admin/model/reload", json={}, headers=K).status_code == 401
    # tampered token
    assert c.get("/admin/auth/me", headers={"Authorization": f"Bearer {tok[:-2]}00"}).status_code == 401
    acts = [e["action"] for e in c.get("/admin/audit", headers=A).json()]
    for a in ("auth.login", "user.create", "apikey.create", "model.reload", "alert.create", "apikey.revoke",
              "auth.fail"):
        assert a in acts, a
    assert c.get("/admin/sessions", headers=V).json() == [{"id": "s1"}]
    for _ in range(5):
        c.get("/ping")
    assert c.get("/admin/metrics", headers=V).json()["sla"]["requests"] == 5


def test_sla_monitor():
    s = SLAMonitor(p99_ms=100, max_error_rate=0.1)
    for i in range(100):
        s.record(10.0)
    assert s.report()["compliant"]
    for i in range(5):
        s.record(500.0, ok=False)
    r = s.report()
    assert not r["compliant"] and r["p99_ms"] == 500.0


def test_admin_web_console_served_and_wired():
    """The console page is served and every view it opens is a route of the admin API."""
    import re
    svc = AdminService(secret=b"k" * 32)
    app = FastAPI()
    svc.mount(app)
    c = TestClient(app)
    r = c.get("/admin/ui")
    assert r.status_code == 200 and r.headers["content-type"].startswith("text/html")
    html = r.text
    assert "/admin/auth/login" in html and "Bearer" in html
    routes = {getattr(rt, "path", "") for rt in app.routes}
    for view in re.findall(r'data-view="([a-z]+)"', html):
        assert f"/admin/{view}" in routes, view
    tok = c.post("/admin/auth/login", json={"username": "admin", "password": "admin"}).json()["token"]
    for view in re.findall(r'data-view="([a-z]+)"', html):
        assert c.get(f"/admin/{view}", headers={"Authorization": f"Bearer {tok}"}).status_code == 200, view
