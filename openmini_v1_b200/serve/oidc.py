"""OAuth2 / OpenID Connect bearer tokens for the admin API.

An identity provider signs JWTs (RS256 or ES256); the server verifies them with the
provider's JSON Web Key Set (a dict given at start-up, or fetched from ``jwks_uri``
and cached), checks issuer, audience, expiry and not-before (with ``leeway_s``), and
maps the token to an admin role: the first of ``role_claims`` present (a string or a
list of groups) looked up in ``role_map``, else ``default_role`` (None: reject).

``OIDCLogin`` is the browser login: the authorization-code flow (RFC 6749 section
4.1) with PKCE (RFC 7636, S256) and the OpenID Connect nonce. ``start`` returns the
provider's authorization URL with a fresh state, code challenge and nonce; ``finish``
takes the code and state from the redirect, sends the code with its verifier to the
token endpoint, verifies the returned ID token with ``OIDCVerifier`` and checks that its
nonce is the one issued. Each state is single use and expires after ``state_ttl_s``.
``from_discovery`` reads the endpoints from the issuer's
``/.well-known/openid-configuration``. The HTTP calls go through ``http_post`` /
``http_get`` (urllib by default), which tests replace with a fake provider.

Reference counterpart: the enterprise SSO settings of openmini-admin (OAuth2 / OIDC
login); the reference configures them, this verifies the tokens and runs the login.
"""
from __future__ import annotations

import base64
import hashlib
import json
import secrets
import threading
import time
import urllib.parse
import urllib.request

from cryptography.hazmat.primitives import hashes
from cryptography.hazmat.primitives.asymmetric import ec, padding, rsa
from cryptography.hazmat.primitives.asymmetric.utils import encode_dss_signature


def b64url_decode(s: str) -> bytes:
    return base64.urlsafe_b64decode(s + "=" * (-len(s) % 4))


def b64url_encode(b: bytes) -> str:
    return base64.urlsafe_b64encode(b).rstrip(b"=").decode()


def _int(s: str) -> int:
    return int.from_bytes(b64url_decode(s), "big")


def _public_key(jwk: dict):
    if jwk.get("kty") == "RSA":
        return rsa.RSAPublicNumbers(_int(jwk["e"]), _int(jwk["n"])).public_key()
    if jwk.get("kty") == "EC" and jwk.get("crv") == "P-256":
        return ec.EllipticCurvePublicNumbers(_int(jwk["x"]), _int(jwk["y"]), ec.SECP256R1()).public_key()
    raise ValueError(f"unsupported JWK {jwk.get('kty')}/{jwk.get('crv')}")


class OIDCError(Exception):
    pass


class OIDCVerifier:
    def __init__(self, issuer: str, audience: str, jwks: dict | None = None, jwks_uri: str | None = None,
                 role_claims=("roles", "groups"), role_map: dict | None = None, default_role: str | None = None,
                 leeway_s: float = 30.0, cache_s: float = 3600.0, clock=time.time):
        self.issuer, self.audience = issuer, audience
        self.jwks_uri, self.role_claims = jwks_uri, tuple(role_claims)
        self.role_map = role_map or {"admin": "admin", "operator": "operator", "viewer": "viewer"}
        self.default_role, self.leeway, self.cache_s, self.clock = default_role, leeway_s, cache_s, clock
        self._keys: dict = {}
        self._fetched = 0.0
        if jwks:
            self._load(jwks)

    def _load(self, jwks: dict):
        self._keys = {k.get("kid", str(i)): k for i, k in enumerate(jwks.get("keys", []))}

    def _key(self, kid: str | None):
        if self.jwks_uri and (not self._keys or self.clock() - self._fetched > self.cache_s or kid not in self._keys):
            with urllib.request.urlopen(self.jwks_uri, timeout=5) as r:
                self._load(json.loads(r.read()))
            self._fetched = self.clock()
        if kid is None and len(self._keys) == 1:
            return next(iter(self._keys.values()))
        if kid not in self._keys:
            raise OIDCError(f"unknown signing key {kid!r}")
        return self._keys[kid]

    def verify(self, token: str) -> dict:
        try:
            h64, p64, s64 = token.split(".")
            header, claims = json.loads(b64url_decode(h64)), json.loads(b64url_decode(p64))
            sig = b64url_decode(s64)
        except (ValueError, json.JSONDecodeError) as e:
            raise OIDCError(f"malformed token: {e}") from e
        alg = header.get("alg")
        jwk = self._key(header.get("kid"))
        key = _public_key(jwk)
        msg = f"{h64}.{p64}".encode()
        try:
            if alg == "RS256" and isinstance(key, rsa.RSAPublicKey):
                key.verify(sig, msg, padding.PKCS1v15(), hashes.SHA256())
            elif alg == "ES256" and isinstance(key, ec.EllipticCurvePublicKey):
                if len(sig) != 64:
                    raise OIDCError("bad ES256 signature length")
                der = encode_dss_signature(int.from_bytes(sig[:32], "big"), int.from_bytes(sig[32:], "big"))
                key.verify(der, msg, ec.ECDSA(hashes.SHA256()))
            else:
                raise OIDCError(f"algorithm {alg!r} not accepted for this key")
        except OIDCError:
            raise
        except Exception as e:
            raise OIDCError("bad signature") from e
        now = self.clock()
        if claims.get("iss") != self.issuer:
            raise OIDCError("wrong issuer")
        aud = claims.get("aud")
        if self.audience not in (aud if isinstance(aud, list) else [aud]):
            raise OIDCError("wrong audience")
        if "exp" not in claims or now > float(claims["exp"]) + self.leeway:
            raise OIDCError("expired")
        if "nbf" in claims and now + self.leeway < float(claims["nbf"]):
            raise OIDCError("not yet valid")
        return claims

    def role_of(self, claims: dict) -> str | None:
        ranks = {"viewer": 1, "operator": 2, "admin": 3}
        best = None
        for c in self.role_claims:
            v = claims.get(c)
            for item in ([v] if isinstance(v, str) else (v or [])):
                r = self.role_map.get(item)
                if r and (best is None or ranks.get(r, 0) > ranks.get(best, 0)):
                    best = r
            if best:
                return best
        return self.default_role


def _urllib_post(url: str, form: dict) -> dict:
    data = urllib.parse.urlencode(form).encode()
    req = urllib.request.Request(url, data=data, headers={"Content-Type": "application/x-www-form-urlencoded",
                                                          "Accept": "application/json"})
    with urllib.request.urlopen(req, timeout=10) as r:
        return json.loads(r.read())


def _urllib_get(url: str) -> dict:
    with urllib.request.urlopen(url, timeout=10) as r:
        return json.loads(r.read())


class OIDCLogin:
    def __init__(self, verifier: OIDCVerifier, authorization_endpoint: str, token_endpoint: str, client_id: str,
                 redirect_uri: str, client_secret: str | None = None, scope: str = "openid profile email",
                 state_ttl_s: float = 600.0, http_post=_urllib_post, clock=time.time):
        self.verifier, self.auth_ep, self.token_ep = verifier, authorization_endpoint, token_endpoint
        self.client_id, self.client_secret, self.redirect_uri, self.scope = client_id, client_secret, redirect_uri, scope
        self.ttl, self.post, self.clock = state_ttl_s, http_post, clock
        self._pending: dict = {}  # state -> (code verifier, nonce, created)
        self._lock = threading.Lock()

    @classmethod
    def from_discovery(cls, verifier: OIDCVerifier, client_id: str, redirect_uri: str, http_get=_urllib_get, **kw):
        doc = http_get(verifier.issuer.rstrip("/") + "/.well-known/openid-configuration")
        if doc.get("issuer") != verifier.issuer:
            raise OIDCError("discovery document names another issuer")
        if doc.get("jwks_uri") and not verifier._keys:
            verifier.jwks_uri = doc["jwks_uri"]
        return cls(verifier, doc["authorization_endpoint"], doc["token_endpoint"], client_id, redirect_uri, **kw)

    def start(self) -> tuple:
        """-> (authorization URL, state)."""
        state, nonce = secrets.token_urlsafe(24), secrets.token_urlsafe(24)
        code_verifier = secrets.token_urlsafe(48)
        challenge = b64url_encode(hashlib.sha256(code_verifier.encode()).digest())
        now = self.clock()
        with self._lock:
            for k in [k for k, v in self._pending.items() if now - v[2] > self.ttl]:
                del self._pending[k]
            self._pending[state] = (code_verifier, nonce, now)
        q = {"response_type": "code", "client_id": self.client_id, "redirect_uri": self.redirect_uri,
             "scope": self.scope, "state": state, "nonce": nonce, "code_challenge": challenge,
             "code_challenge_method": "S256"}
        sep = "&" if "?" in self.auth_ep else "?"
        return self.auth_ep + sep + urllib.parse.urlencode(q), state

    def finish(self, code: str, state: str) -> dict:
        """Code and state from the provider's redirect -> verified ID-token claims."""
        with self._lock:
            entry = self._pending.pop(state, None)
        if entry is None:
            raise OIDCError("unknown or already used login state")
        code_verifier, nonce, created = entry
        if self.clock() - created > self.ttl:
            raise OIDCError("login state expired")
        form = {"grant_type": "authorization_code", "code": code, "redirect_uri": self.redirect_uri,
                "client_id": self.client_id, "code_verifier": code_verifier}
        if self.client_secret:
            form["client_secret"] = self.client_secret
        try:
            resp = self.post(self.token_ep, form)
        except Exception as e:
            raise OIDCError(f"token endpoint: {e}") from e
        if "id_token" not in resp:
            raise OIDCError(f"token endpoint returned no id_token: {resp.get('error', resp)}")
        claims = self.verifier.verify(resp["id_token"])
        if claims.get("nonce") != nonce:
            raise OIDCError("nonce mismatch")
        return claims
