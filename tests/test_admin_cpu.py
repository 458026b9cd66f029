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


def _jwt(key, alg, claims, kid="k1"):
    import json
    from cryptography.hazmat.primitives import hashes
    from cryptography.hazmat.primitives.asymmetric import ec, padding
    from cryptography.hazmat.primitives.asymmetric.utils import decode_dss_signature
    from openmini_v1_b200.serve.oidc import b64url_encode
    h = b64url_encode(json.dumps({"alg": alg, "kid": kid, "typ": "JWT"}).encode())
    p = b64url_encode(json.dumps(claims).encode())
    msg = f"{h}.{p}".encode()
    if alg == "RS256":
        sig = key.sign(msg, padding.PKCS1v15(), hashes.SHA256())
    else:
        r, s = decode_dss_signature(key.sign(msg, ec.ECDSA(hashes.SHA256())))
        sig = r.to_bytes(32, "big") + s.to_bytes(32, "big")
    return f"{h}.{p}.{b64url_encode(sig)}"


def test_oidc_bearer_tokens():
    import time
    from cryptography.hazmat.primitives.asymmetric import ec, rsa
    from openmini_v1_b200.serve.oidc import OIDCVerifier, b64url_encode
    rk = rsa.generate_private_key(public_exponent=65537, key_size=2048)
    ek = ec.generate_private_key(ec.SECP256R1())
    rn, en = rk.public_key().public_numbers(), ek.public_key().public_numbers()
    b = lambda i, n: b64url_encode(i.to_bytes(n, "big"))  # noqa: E731
    jwks = {"keys": [{"kty": "RSA", "kid": "k1", "n": b(rn.n, 256), "e": b(rn.e, 3)},
                     {"kty": "EC", "crv": "P-256", "kid": "k2", "x": b(en.x, 32), "y": b(en.y, 32)}]}
    svc = AdminService(secret=b"k" * 32)
    svc.oidc = OIDCVerifier("https://idp.example", "openmini", jwks=jwks, role_map={"ops-team": "operator"})
    app = FastAPI()
    svc.mount(app)
    c = TestClient(app)
    now = time.time()
    good = {"iss": "https://idp.example", "aud": "openmini", "exp": now + 60, "sub": "u1",
            "preferred_username": "alice", "groups": ["eng", "ops-team"]}
    for key, alg, kid in ((rk, "RS256", "k1"), (ek, "ES256", "k2")):
        t = _jwt(key, alg, good, kid)
        assert c.get("/admin/auth/me", headers={"Authorization": f"Bearer {t}"}).json() == \
            {"user": "alice", "role": "operator"}
    bad = [dict(good, exp=now - 100), dict(good, aud="other"), dict(good, iss="evil"), dict(good, groups=["eng"])]
    for claims in bad:
        t = _jwt(rk, "RS256", claims)
        assert c.get("/admin/auth/me", headers={"Authorization": f"Bearer {t}"}).status_code == 401, claims
    forged = _jwt(rsa.generate_private_key(public_exponent=65537, key_size=2048), "RS256", good)
    assert c.get("/admin/auth/me", headers={"Authorization": f"Bearer {forged}"}).status_code == 401


def test_oidc_browser_login_code_flow_with_pkce():
    """Authorization-code login against a fake provider: the redirect carries state,
    nonce and an S256 code challenge; the callback's token request carries the matching
    verifier; the ID token's nonce must match; states are single use; a user without a
    mapped role is refused; discovery reads the endpoints."""
    import hashlib
    import time
    import urllib.parse
    from cryptography.hazmat.primitives.asymmetric import rsa
    from openmini_v1_b200.serve.oidc import OIDCLogin, OIDCVerifier, b64url_encode
    rk = rsa.generate_private_key(public_exponent=65537, key_size=2048)
    rn = rk.public_key().public_numbers()
    b = lambda i, n: b64url_encode(i.to_bytes(n, "big"))  # noqa: E731
    jwks = {"keys": [{"kty": "RSA", "kid": "k1", "n": b(rn.n, 256), "e": b(rn.e, 3)}]}
    issued = {}   # code -> (challenge, nonce, groups)
    seen = []

    def provider_token(url, form):
        seen.append((url, dict(form)))
        challenge, nonce, groups = issued.pop(form["code"])
        if b64url_encode(hashlib.sha256(form["code_verifier"].encode()).digest()) != challenge:
            return {"error": "invalid_grant"}
        claims = {"iss": "https://idp.example", "aud": "openmini", "exp": time.time() + 60, "sub": "u7",
                  "preferred_username": "bob", "groups": groups, "nonce": nonce}
        return {"id_token": _jwt(rk, "RS256", claims), "token_type": "Bearer"}

    verifier = OIDCVerifier("https://idp.example", "openmini", jwks=jwks, role_map={"ops-team": "operator"})
    doc = {"issuer": "https://idp.example", "authorization_endpoint": "https://idp.example/authorize",
           "token_endpoint": "https://idp.example/token", "jwks_uri": "https://idp.example/jwks"}
    login = OIDCLogin.from_discovery(verifier, "openmini", "https://admin.local/admin/auth/oidc/callback",
                                     http_get=lambda url: doc, http_post=provider_token, client_secret="s3")
    svc = AdminService(secret=b"k" * 32)
    svc.oidc_login = login
    app = FastAPI()
    svc.mount(app)
    c = TestClient(app)

    def authorize(groups, nonce_override=None):
        r = c.get("/admin/auth/oidc/login", follow_redirects=False)
        assert r.status_code == 302
        url = urllib.parse.urlparse(r.headers["location"])
        q = dict(urllib.parse.parse_qsl(url.query))
        assert url.netloc == "idp.example" and url.path == "/authorize"
        assert q["response_type"] == "code" and q["code_challenge_method"] == "S256" and q["client_id"] == "openmini"
        code = "c" + q["state"][:8]
        issued[code] = (q["code_challenge"], nonce_override or q["nonce"], groups)
        return code, q["state"]

    code, state = authorize(["ops-team"])
    r = c.get("/admin/auth/oidc/callback", params={"code": code, "state": state})
    assert r.status_code == 200, r.text
    assert r.json()["user"] == "bob" and r.json()["role"] == "operator"
    assert c.get("/admin/auth/me", headers={"Authorization": f"Bearer {r.json()['token']}"}).json() == \
        {"user": "bob", "role": "operator"}
    assert seen[-1][0] == "https://idp.example/token" and seen[-1][1]["client_secret"] == "s3"
    assert seen[-1][1]["grant_type"] == "authorization_code"
    # the state was used up
    issued["again"] = issued.get("again", ("x", "y", []))
    assert c.get("/admin/auth/oidc/callback", params={"code": "again", "state": state}).status_code == 400
    # a nonce that is not the issued one is refused
    code, state = authorize(["ops-team"], nonce_override="forged")
    assert c.get("/admin/auth/oidc/callback", params={"code": code, "state": state}).status_code == 400
    # a user whose groups map to no role is refused
    code, state = authorize(["eng"])
    assert c.get("/admin/auth/oidc/callback", params={"code": code, "state": state}).status_code == 403
    # an unknown state, and an error from the provider
    assert c.get("/admin/auth/oidc/callback", params={"code": "x", "state": "nope"}).status_code == 400
    assert c.get("/admin/auth/oidc/callback", params={"error": "access_denied"}).status_code == 400
    # an expired state
    login.ttl = -1.0
    code, state = authorize(["ops-team"])
    assert c.get("/admin/auth/oidc/callback", params={"code": code, "state": state}).status_code == 400
    # not configured
    svc2 = AdminService(secret=b"k" * 32)
    app2 = FastAPI()
    svc2.mount(app2)
    assert TestClient(app2).get("/admin/auth/oidc/login", follow_redirects=False).status_code == 404


def test_server_entry_mounts_admin(monkeypatch):
    """``serve.main.mount_admin``: the /admin API on the server's app, with the admin
    password from the environment and the model status hook wired."""
    from types import SimpleNamespace
    from openmini_v1_b200.config.settings import load_config
    from openmini_v1_b200.serve.main import mount_admin
    monkeypatch.setenv("OPENMINI_ADMIN_PASSWORD", "pw-123")
    eng = SimpleNamespace(model=SimpleNamespace(cfg=SimpleNamespace(name="tiny", num_layers=2, vocab_size=512)),
                          device="cpu")
    args = SimpleNamespace(admin_db=None, oidc_issuer=None, oidc_client_id="openmini", oidc_audience=None,
                           oidc_redirect_uri=None)
    app = FastAPI()
    mount_admin(app, eng, load_config(None), args)
    c = TestClient(app)
    assert c.post("/admin/auth/login", json={"username": "admin", "password": "nope"}).status_code == 401
    tok = c.post("/admin/auth/login", json={"username": "admin", "password": "pw-123"}).json()["token"]
    h = {"Authorization": f"Bearer {tok}"}
    assert c.get("/admin/model", headers=h).json()["name"] == "tiny"
    assert c.get("/admin/ui").status_code == 200
