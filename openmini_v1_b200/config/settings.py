"""Server configuration with the section / key names and defaults of the
reference's ``server.toml`` (openmini-server/src/config/settings.rs:20-480,
config/server.toml), loaded with ``tomllib``.

Unknown keys are kept (``extra``) rather than rejected, missing keys take the
defaults, and environment variables ``OPENMINI__<SECTION>__<KEY>=value``
override file values (e.g. ``OPENMINI__SERVER__PORT=8080``).
"""
from __future__ import annotations

import dataclasses
import os
import tomllib
import typing
from dataclasses import dataclass, field


@dataclass
class ServerSettings:
    host: str = "0.0.0.0"
    port: int = 50051
    http_port: int = 8080
    max_connections: int = 10000
    request_timeout_ms: int = 60000


@dataclass
class SchedulerSettings:
    max_concurrent: int = field(default_factory=lambda: max(1, os.cpu_count() or 1))
    queue_capacity: int = 1000
    worker_type: str = "auto"          # blocking | async | auto
    batch_size: int = 8
    batch_timeout_ms: int = 5


@dataclass
class ThreadPoolSettings:
    size: int = field(default_factory=lambda: os.cpu_count() or 1)
    stack_size_kb: int = 8192


@dataclass
class MemorySettings:
    max_memory_gb: int = 12
    model_memory_gb: int = 6
    cache_memory_gb: int = 4
    arena_size_mb: int = 256


@dataclass
class ModelSettings:
    path: str = "models/openmini-v1-q4_k_m.gguf"
    quantization: str = "Q4_K_M"
    context_length: int = 4096
    architecture: str = "native"
    preset: str = ""                   # build a random-init preset instead of loading `path`
    weight_format: str = "bf16"        # device weight format: bf16 | q4 | int8


@dataclass
class MoESettings:
    strategy: str = "cyclic"
    cycle_period: int = 3
    ffn_prefix_layers: int = 3
    num_routing_experts: int = 8
    num_shared_experts: int = 0
    top_k: int = 2
    capacity_factor: float = 1.25
    load_balance: bool = True


@dataclass
class VisionSettings:
    encoder: str = "none"
    image_size: int = 224
    num_image_tokens: int = 256


@dataclass
class EngineSettings:
    gemm_backend: str = "auto"
    enable_arena: bool = True
    arena_size_mb: int = 64
    fp8_kv_cache: bool = False
    target_device: str = "auto"
    dsa_threshold: int = 1024
    max_batch_size: int = 1
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 8192
    gpu_memory_utilization: float = 0.9
    enable_prefix_cache: bool = True
    use_cuda_graph: bool = True


@dataclass
class DistributedInferenceSettings:
    enabled: bool = False
    strategy: str = "tensor"           # tensor | pipeline | hybrid | sequence
    backend: str = "nccl"              # nccl | gloo
    tp_degree: int = 1
    pp_degree: int = 1
    dp_degree: int = 1
    ep_degree: int = 1
    sequence_chunk_size: int = 4096
    master_addr: str = "127.0.0.1"
    master_port: int = 29500


@dataclass
class WorkerSettings:
    count: int = 1
    restart_on_failure: bool = True
    health_check_interval_ms: int = 5000


@dataclass
class PerCoreSettings:
    max_concurrent: int = 5000
    kv_cache_mb: int = 2048


@dataclass
class CoreSettings:
    count: int = 2
    binding: bool = True
    strategy: str = "round_robin"
    per_core: PerCoreSettings = field(default_factory=PerCoreSettings)


@dataclass
class GrpcSettings:
    max_message_size_mb: int = 100
    keepalive_time_ms: int = 30000
    keepalive_timeout_ms: int = 10000


@dataclass
class DatabaseSettings:
    path: str = "data/openmini.db"
    pool_size: int = 10
    busy_timeout_ms: int = 5000


@dataclass
class TrainingSettings:
    enable: bool = False
    mode: str = "causal_lm"
    model: dict = field(default_factory=dict)
    hyperparams: dict = field(default_factory=dict)
    optimizer: dict = field(default_factory=dict)
    scheduler: dict = field(default_factory=dict)
    data: dict = field(default_factory=dict)
    checkpoint: dict = field(default_factory=dict)
    logging: dict = field(default_factory=dict)
    early_stopping: dict = field(default_factory=dict)
    sft: dict = field(default_factory=dict)


@dataclass
class ServerConfig:
    server: ServerSettings = field(default_factory=ServerSettings)
    scheduler: SchedulerSettings = field(default_factory=SchedulerSettings)
    thread_pool: ThreadPoolSettings = field(default_factory=ThreadPoolSettings)
    memory: MemorySettings = field(default_factory=MemorySettings)
    model: ModelSettings = field(default_factory=ModelSettings)
    moe: MoESettings = field(default_factory=MoESettings)
    vision: VisionSettings = field(default_factory=VisionSettings)
    engine: EngineSettings = field(default_factory=EngineSettings)
    distributed_inference: DistributedInferenceSettings = field(default_factory=DistributedInferenceSettings)
    worker: WorkerSettings = field(default_factory=WorkerSettings)
    core: CoreSettings = field(default_factory=CoreSettings)
    grpc: GrpcSettings = field(default_factory=GrpcSettings)
    database: DatabaseSettings = field(default_factory=DatabaseSettings)
    training: TrainingSettings = field(default_factory=TrainingSettings)
    extra: dict = field(default_factory=dict)

    # ------------------------------------------------------------ loading
    @staticmethod
    def from_dict(d: dict) -> "ServerConfig":
        return _build(ServerConfig, d)

    @staticmethod
    def from_file(path: str, env: dict | None = None) -> "ServerConfig":
        with open(path, "rb") as f:
            d = tomllib.load(f)
        cfg = ServerConfig.from_dict(d)
        cfg.apply_env(os.environ if env is None else env)
        return cfg

    @staticmethod
    def from_str(text: str) -> "ServerConfig":
        return ServerConfig.from_dict(tomllib.loads(text))

    def apply_env(self, env):
        for k, v in env.items():
            if not k.startswith("OPENMINI__"):
                continue
            parts = k[len("OPENMINI__"):].lower().split("__")
            obj = self
            for p in parts[:-1]:
                obj = getattr(obj, p, None)
                if obj is None:
                    break
            if obj is None or not hasattr(obj, parts[-1]):
                continue
            cur = getattr(obj, parts[-1])
            setattr(obj, parts[-1], _coerce(v, type(cur)))

    def validate(self) -> list:
        """Warnings (not errors) for suspicious settings, like the reference's start-up check."""
        w = []
        di = self.distributed_inference
        if di.tp_degree < 1 or di.pp_degree < 1:
            w.append("parallel degrees must be >= 1")
        if self.server.port <= 0 or self.server.port > 65535:
            w.append(f"invalid port {self.server.port}")
        if self.model.context_length <= 0:
            w.append("context_length must be positive")
        if self.engine.gpu_memory_utilization <= 0 or self.engine.gpu_memory_utilization > 1:
            w.append("gpu_memory_utilization must be in (0, 1]")
        if self.moe.top_k > self.moe.num_routing_experts:
            w.append("moe.top_k exceeds num_routing_experts")
        return w

    def to_dict(self):
        return dataclasses.asdict(self)

    def to_toml(self) -> str:
        """The whole configuration as TOML that ``from_str`` reads back to an equal object
        (unknown keys kept in ``extra`` are written at the top level)."""
        d = self.to_dict()
        extra = d.pop("extra", {})
        return _toml_table(extra, []) + "".join(_toml_table(v, [k]) for k, v in d.items())


def _toml_key(k: str) -> str:
    return k if k and all(c.isalnum() or c in "-_" for c in k) else _toml_str(k)


def _toml_str(s: str) -> str:
    out = ['"']
    for ch in s:
        if ch in '"\\':
            out.append("\\" + ch)
        elif ord(ch) < 0x20 or ord(ch) == 0x7F:
            out.append(f"\\u{ord(ch):04x}")
        else:
            out.append(ch)
    return "".join(out) + '"'


def _toml_value(v) -> str:
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, float):
        if v != v:
            return "nan"
        if v in (float("inf"), float("-inf")):
            return "inf" if v > 0 else "-inf"
        return repr(v)
    if isinstance(v, str):
        return _toml_str(v)
    if isinstance(v, (list, tuple)):
        return "[" + ", ".join(_toml_value(x) for x in v) + "]"
    if isinstance(v, dict):
        return "{" + ", ".join(f"{_toml_key(k)} = {_toml_value(x)}" for k, x in v.items()) + "}"
    if v is None:
        raise ValueError("TOML has no null value")
    raise TypeError(f"cannot write {type(v).__name__} as TOML")


def _toml_table(d: dict, path: list) -> str:
    tables = [(k, v) for k, v in d.items() if isinstance(v, dict) and v]
    scalars = [(k, v) for k, v in d.items() if not (isinstance(v, dict) and v)]
    out = []
    if path and (scalars or not tables):
        out.append("[" + ".".join(_toml_key(p) for p in path) + "]\n")
    out += [f"{_toml_key(k)} = {_toml_value(v)}\n" for k, v in scalars if v is not None]
    if out:
        out.append("\n")
    for k, v in tables:
        out.append(_toml_table(v, path + [k]))
    return "".join(out)


def _coerce(v: str, typ):
    if typ is bool:
        return str(v).lower() in ("1", "true", "yes", "on")
    if typ is int:
        return int(v)
    if typ is float:
        return float(v)
    return v


def _build(cls, d: dict):
    hints = typing.get_type_hints(cls)
    kwargs, extra = {}, {}
    for k, v in (d or {}).items():
        if k in hints and k != "extra":
            t = hints[k]
            if dataclasses.is_dataclass(t) and isinstance(v, dict):
                kwargs[k] = _build(t, v)
            elif t is float and isinstance(v, int):
                kwargs[k] = float(v)
            else:
                kwargs[k] = v
        else:
            extra[k] = v
    obj = cls(**kwargs)
    if extra and hasattr(obj, "extra"):
        obj.extra.update(extra)
    return obj


def load_config(path: str | None = None) -> ServerConfig:
    """Load ``path`` (or $OPENMINI_CONFIG, or config/server.toml if present), else defaults."""
    path = path or os.environ.get("OPENMINI_CONFIG")
    if path is None and os.path.exists("config/server.toml"):
        path = "config/server.toml"
    if path is None:
        cfg = ServerConfig()
        cfg.apply_env(os.environ)
        return cfg
    return ServerConfig.from_file(path)
