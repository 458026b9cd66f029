"""Server entry point.

    python -m openmini_v1_b200.serve.main [--config server.toml] [--preset tiny]
        [--model path.gguf] [--http-port 8080] [--grpc-port 50051] [--gateway-port 0]

Start-up mirrors openmini-server/src/main.rs:76-247 (logging, hardware report,
config load + validation warnings, engine, servers, signal-driven shutdown),
but the engine is the real one: a model from GGUF (or a random-init preset),
the paged-KV continuous-batching engine, then HTTP (uvicorn), gRPC and the
raw-TCP gateway on one event loop.
"""
from __future__ import annotations

import argparse
import asyncio
import logging
import signal

import torch

from ..config.settings import load_config
from ..engine.async_engine import AsyncLLMEngine
from ..engine.engine import EngineConfig, LLMEngine
from ..engine.tokenizer import ByteTokenizer, GGUFTokenizer
from ..models.config import preset
from ..models.llama import DecoderLM
from ..utils.logging import init_logging
from .gateway import Gateway
from .grpc_server import OpenMiniServicer, SessionStore, start_grpc_server
from .http import create_app
from .metrics import Metrics

log = logging.getLogger("openmini.server")


def build_engine(cfg, preset_name=None, model_path=None, device=None):
    device = device or ("cuda" if torch.cuda.is_available() else "cpu")
    fmt = cfg.model.weight_format if device != "cpu" else "bf16"
    tokenizer = None
    if model_path or (not preset_name and cfg.model.path and not cfg.model.preset):
        from ..gguf.reader import GGUFReader
        from ..models.loader import load_gguf_model
        path = model_path or cfg.model.path
        model = load_gguf_model(path, device=device, weight_format=fmt)
        reader = GGUFReader(path)
        if "tokenizer.ggml.tokens" in reader.metadata:
            tokenizer = GGUFTokenizer.from_gguf(reader)
    else:
        mc = preset(preset_name or cfg.model.preset or "tiny")
        if device == "cpu":
            mc.dtype = "float32"
        elif mc.dtype == "float32":
            mc.dtype = "bfloat16"
        model = DecoderLM(mc, device=device, weight_format=fmt)
    tokenizer = tokenizer or ByteTokenizer(model.cfg.vocab_size)
    e = cfg.engine
    ecfg = EngineConfig(max_num_seqs=e.max_num_seqs, max_num_batched_tokens=e.max_num_batched_tokens,
                        max_model_len=min(cfg.model.context_length, model.cfg.max_position),
                        gpu_memory_utilization=e.gpu_memory_utilization, enable_prefix_cache=e.enable_prefix_cache,
                        use_cuda_graph=e.use_cuda_graph and device != "cpu",
                        eos_token_id=getattr(tokenizer, "eos_id", None))
    return LLMEngine(model, ecfg), tokenizer


def mount_admin(app, eng, cfg, args):
    """The /admin API and console. The admin password comes from $OPENMINI_ADMIN_PASSWORD
    (a random one is generated and logged when it is unset); with --oidc-issuer the
    provider's bearer tokens are accepted and /admin/auth/oidc/login runs the browser
    login (client secret from $OPENMINI_OIDC_CLIENT_SECRET)."""
    import os
    import secrets
    from .admin import AdminService, AdminStore
    pw = os.environ.get("OPENMINI_ADMIN_PASSWORD")
    if not pw:
        pw = secrets.token_urlsafe(12)
        log.warning("admin user 'admin' created with password %s (set OPENMINI_ADMIN_PASSWORD)", pw)
    svc = AdminService(store=AdminStore(args.admin_db or ":memory:"), bootstrap_admin=("admin", pw))
    svc.hooks["model_status"] = lambda: {"name": eng.model.cfg.name, "device": str(eng.device),
                                         "layers": eng.model.cfg.num_layers, "vocab": eng.model.cfg.vocab_size}
    svc.hooks["config"] = lambda: {"server": vars(cfg.server), "model": eng.model.cfg.name}
    if args.oidc_issuer:
        from .oidc import OIDCLogin, OIDCVerifier
        verifier = OIDCVerifier(args.oidc_issuer, args.oidc_audience or args.oidc_client_id)
        svc.oidc = verifier
        if args.oidc_redirect_uri:
            svc.oidc_login = OIDCLogin.from_discovery(verifier, args.oidc_client_id, args.oidc_redirect_uri,
                                                      client_secret=os.environ.get("OPENMINI_OIDC_CLIENT_SECRET"))
    svc.mount(app)
    return svc


async def serve(args):
    cfg = load_config(args.config)
    for w in cfg.validate():
        log.warning("config: %s", w)
    eng, tok = build_engine(cfg, args.preset, args.model)
    aeng = AsyncLLMEngine(eng)
    metrics = Metrics()
    vision = None
    if args.vision:
        from ..models.vision import VisionConfig, VisionEncoder
        from .vision_service import ImageUnderstanding
        vc = VisionConfig(lm_hidden=eng.model.cfg.hidden_size)
        if eng.device.type == "cpu":
            vc.hidden_size, vc.num_layers, vc.mlp_size, vc.num_heads = 256, 2, 512, 2
        vision = ImageUnderstanding(aeng, tok, VisionEncoder(vc, device=eng.device, dtype=eng.model.dtype),
                                    pan_scan=args.pan_scan)
    speech = None
    if args.audio:
        from ..models.audio import AudioConfig, AudioEncoder
        from .vision_service import SpeechToText
        ac = AudioConfig(lm_hidden=eng.model.cfg.hidden_size)
        if eng.device.type == "cpu":
            ac.hidden_size, ac.num_layers, ac.mlp_size, ac.num_heads = 256, 2, 512, 2
        speech = SpeechToText(aeng, tok, AudioEncoder(ac, device=eng.device, dtype=eng.model.dtype))
    tts = None
    if args.tts:
        from ..models.tts import TTSModel
        from .vision_service import TextToSpeech
        tts = TextToSpeech(TTSModel(device=eng.device, dtype=eng.model.dtype))
    app = create_app(aeng, tok, model_name=eng.model.cfg.name, metrics=metrics, config=cfg, vision=vision,
                     speech=speech, tts=tts)
    if args.admin:
        mount_admin(app, eng, cfg, args)
    import uvicorn
    http = uvicorn.Server(uvicorn.Config(app, host=cfg.server.host, port=args.http_port or cfg.server.http_port,
                                         log_level="warning"))
    store = SessionStore(cfg.database.path if args.db else ":memory:")
    servicer = OpenMiniServicer(aeng, tok, store, metrics, vision=vision, speech=speech, tts=tts)
    grpc_server, gport = await start_grpc_server(servicer,
                                                 f"{cfg.server.host}:{args.grpc_port or cfg.server.port}",
                                                 cfg.grpc.max_message_size_mb)
    gw = Gateway(aeng, tok, cfg.server.max_connections)
    gw_port = await gw.start(cfg.server.host, args.gateway_port) if args.gateway_port is not None else None
    log.info("serving %s: http :%s grpc :%s gateway :%s", eng.model.cfg.name, http.config.port, gport, gw_port)
    stop = asyncio.Event()
    loop = asyncio.get_running_loop()
    for sig in (signal.SIGINT, signal.SIGTERM):
        try:
            loop.add_signal_handler(sig, stop.set)
        except NotImplementedError:
            pass
    http_task = asyncio.create_task(http.serve())
    await stop.wait()
    http.should_exit = True
    await http_task
    await grpc_server.stop(5)
    await gw.stop()
    aeng.shutdown()


def main(argv=None):
    p = argparse.ArgumentParser(description="openmini_v1_b200 server")
    p.add_argument("--config", default=None)
    p.add_argument("--preset", default=None)
    p.add_argument("--model", default=None)
    p.add_argument("--http-port", type=int, default=None)
    p.add_argument("--grpc-port", type=int, default=None)
    p.add_argument("--gateway-port", type=int, default=None)
    p.add_argument("--db", action="store_true", help="persist chat sessions to [database].path")
    p.add_argument("--vision", action="store_true",
                   help="load a vision encoder (random-init weights) and serve image understanding")
    p.add_argument("--pan-scan", action="store_true", help="with --vision: tile large images (pan and scan)")
    p.add_argument("--audio", action="store_true",
                   help="load an audio encoder (random-init weights) and serve speech-to-text")
    p.add_argument("--tts", action="store_true",
                   help="load a text-to-speech model (random-init weights) with a Griffin-Lim vocoder")
    p.add_argument("--admin", action="store_true", help="serve the /admin API and console")
    p.add_argument("--admin-db", default=None, help="SQLite file of the admin store (default: in memory)")
    p.add_argument("--oidc-issuer", default=None, help="accept bearer tokens of this OpenID Connect issuer")
    p.add_argument("--oidc-client-id", default="openmini")
    p.add_argument("--oidc-audience", default=None, help="expected audience (default: the client id)")
    p.add_argument("--oidc-redirect-uri", default=None,
                   help="with --oidc-issuer: enable the browser login; the URL of /admin/auth/oidc/callback")
    p.add_argument("--dump-config", action="store_true",
                   help="print the effective configuration (file, defaults and OPENMINI__ overrides) as TOML")
    args = p.parse_args(argv)
    if args.dump_config:
        print(load_config(args.config).to_toml(), end="")
        return
    init_logging()
    asyncio.run(serve(args))


if __name__ == "__main__":
    main()
