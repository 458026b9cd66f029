"""OAuth2 / OpenID Connect bearer tokens for the admin API.

An identity provider signs JWTs (RS256 or ES256); the server verifies them with the
provider's JSON Web Key Set (a dict given at start-up, or fetched from ``jwks_uri``
and cached), checks issuer, audience, expiry and not-before (with ``leeway_s``), and
maps the token to an admin role: the first of ``role_claims`` present (a string or a
list of groups) looked up in ``role_map``, else ``default_role`` (None: reject).

Reference counterpart: the enterprise SSO settings of openmini-admin (OAuth2 / OIDC
login); the reference configures them, this verifies the tokens.
"""
from __future__ import annotations

import base64
import json
import time
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
