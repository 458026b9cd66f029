"""Error model: one exception hierarchy with stable error-code prefixes.

Reference: AppError {Engine (ENG), Worker (WRK), Training (TRN), Hardware
(HW), ...} and InferenceError (openmini-server/src/error.rs:1-545,
model/inference/error.rs:1-735). ``http_status`` maps each class to the HTTP
status the server answers with.
"""
from __future__ import annotations


class OpenMiniError(Exception):
    code_prefix = "APP"
    http_status = 500

    def __init__(self, message: str, code: int = 0, **context):
        super().__init__(message)
        self.message = message
        self.code = f"{self.code_prefix}{code:03d}"
        self.context = context

    def to_dict(self) -> dict:
        return {"error": self.message, "code": self.code, "type": type(self).__name__, **self.context}


class EngineError(OpenMiniError):
    code_prefix = "ENG"


class KVCacheExhausted(EngineError):
    http_status = 503


class InferenceError(EngineError):
    code_prefix = "INF"


class InvalidRequest(OpenMiniError):
    code_prefix = "REQ"
    http_status = 400


class WorkerError(OpenMiniError):
    code_prefix = "WRK"
    http_status = 503


class TrainingError(OpenMiniError):
    code_prefix = "TRN"


class HardwareError(OpenMiniError):
    code_prefix = "HW"


class DeviceStatusError(HardwareError):
    """A bounded device wait gave up (kernel status word set)."""


class ConfigError(OpenMiniError):
    code_prefix = "CFG"
    http_status = 400


class ModelLoadError(OpenMiniError):
    code_prefix = "MDL"
