"""Ops artefacts: the CI workflow and Dockerfile point at files that exist, and the
TypeScript client calls routes the HTTP server serves."""
import pathlib
import re

import yaml

ROOT = pathlib.Path(__file__).resolve().parents[1]


def test_ci_and_dockerfile():
    wf = yaml.safe_load((ROOT / ".github/workflows/ci.yml").read_text())
    steps = " ".join(s.get("run", "") for s in wf["jobs"]["cpu"]["steps"])
    assert "pytest tests" in steps and "build()" in steps
    df = (ROOT / "Dockerfile").read_text()
    for src in re.findall(r"^COPY (.+) \S+$", df, re.M):
        for f in src.split():
            assert (ROOT / f).exists(), f
    assert "openmini_v1_b200.serve.main" in df


def test_typescript_client_routes_exist():
    from openmini_v1_b200.serve.http import create_app
    ts = (ROOT / "bindings/typescript/openmini.ts").read_text()

    class _E:
        engine = None
    app = create_app(_E(), None, "x")
    routes = {getattr(r, "path", "") for r in app.routes}
    used = set(re.findall(r'"(/(?:v1|api/v1|health)[a-z/_]*)"', ts))
    assert used and used <= routes, used - routes
