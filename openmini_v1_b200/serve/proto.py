"""The ``openmini`` protobuf package (messages and the ``OpenMini`` service of
openmini-proto/proto/openmini.proto), built at import time from a
FileDescriptorProto so no protoc / grpc_tools step is needed.

Field names, numbers and types match the public .proto so existing clients
(openmini-client/client.py) interoperate.
"""
from __future__ import annotations

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

_F = descriptor_pb2.FieldDescriptorProto
_T = {"string": _F.TYPE_STRING, "bytes": _F.TYPE_BYTES, "bool": _F.TYPE_BOOL, "int32": _F.TYPE_INT32,
      "float": _F.TYPE_FLOAT}

# message -> [(name, number, type or message name, repeated?, oneof index or None)]
MESSAGES = {
    "UsageInfo": [("prompt_tokens", 1, "int32"), ("completion_tokens", 2, "int32"), ("total_tokens", 3, "int32")],
    "Message": [("role", 1, "string"), ("content", 2, "string"), ("image_data", 3, "bytes"),
                ("audio_data", 4, "bytes"), ("video_data", 5, "bytes")],
    "ChatRequest": [("session_id", 1, "string"), ("messages", 2, ".openmini.Message", True),
                    ("stream", 3, "bool"), ("max_tokens", 4, "int32"), ("temperature", 5, "float")],
    "ChatResponse": [("session_id", 1, "string"), ("token", 2, "string"), ("finished", 3, "bool"),
                     ("usage", 4, ".openmini.UsageInfo")],
    "ImageRequest": [("session_id", 1, "string"), ("image_data", 2, "bytes"), ("question", 3, "string"),
                     ("stream", 4, "bool")],
    "ImageResponse": [("session_id", 1, "string"), ("token", 2, "string"), ("finished", 3, "bool")],
    "HealthRequest": [],
    "HealthResponse": [("healthy", 1, "bool"), ("message", 2, "string")],
    "OmniChatRequest": [("session_id", 1, "string"), ("text", 2, "string", False, 0),
                        ("audio_data", 3, "bytes", False, 0), ("video_data", 4, "bytes", False, 0),
                        ("image_data", 5, "bytes", False, 0), ("stream", 6, "bool"), ("max_tokens", 7, "int32"),
                        ("temperature", 8, "float")],
    "OmniChatResponse": [("session_id", 1, "string"), ("text", 2, "string", False, 0),
                         ("audio_data", 3, "bytes", False, 0), ("finished", 4, "bool"),
                         ("usage", 5, ".openmini.UsageInfo")],
    "SpeechToTextRequest": [("session_id", 1, "string"), ("audio_data", 2, "bytes"), ("language", 3, "string"),
                            ("stream", 4, "bool")],
    "SpeechToTextResponse": [("session_id", 1, "string"), ("text", 2, "string"), ("finished", 3, "bool"),
                             ("confidence", 4, "float")],
    "TextToSpeechRequest": [("session_id", 1, "string"), ("text", 2, "string"), ("voice", 3, "string"),
                            ("language", 4, "string"), ("speed", 5, "float"), ("pitch", 6, "float")],
    "TextToSpeechResponse": [("session_id", 1, "string"), ("audio_data", 2, "bytes"), ("finished", 3, "bool")],
}
ONEOFS = {"OmniChatRequest": ["input"], "OmniChatResponse": ["output"]}

# rpc -> (request, response, client streaming, server streaming)
METHODS = {
    "Chat": ("ChatRequest", "ChatResponse", True, True),
    "ImageUnderstanding": ("ImageRequest", "ImageResponse", False, False),
    "ImageUnderstandingStream": ("ImageRequest", "ImageResponse", False, True),
    "HealthCheck": ("HealthRequest", "HealthResponse", False, False),
    "OmniChat": ("OmniChatRequest", "OmniChatResponse", True, True),
    "SpeechToText": ("SpeechToTextRequest", "SpeechToTextResponse", True, True),
    "TextToSpeech": ("TextToSpeechRequest", "TextToSpeechResponse", False, True),
}
SERVICE = "openmini.OpenMini"


def _build():
    fd = descriptor_pb2.FileDescriptorProto(name="openmini.proto", package="openmini", syntax="proto3")
    for name, fields in MESSAGES.items():
        m = fd.message_type.add(name=name)
        for o in ONEOFS.get(name, []):
            m.oneof_decl.add(name=o)
        for f in fields:
            fname, num, typ = f[0], f[1], f[2]
            rep = len(f) > 3 and f[3]
            oneof = f[4] if len(f) > 4 else None
            fp = m.field.add(name=fname, number=num)
            fp.label = _F.LABEL_REPEATED if rep else _F.LABEL_OPTIONAL
            if typ.startswith("."):
                fp.type = _F.TYPE_MESSAGE
                fp.type_name = typ
            else:
                fp.type = _T[typ]
            if oneof is not None:
                fp.oneof_index = oneof
    svc = fd.service.add(name="OpenMini")
    for mname, (req, resp, cs, ss) in METHODS.items():
        svc.method.add(name=mname, input_type=f".openmini.{req}", output_type=f".openmini.{resp}",
                       client_streaming=cs, server_streaming=ss)
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    classes = {}
    for name in MESSAGES:
        classes[name] = message_factory.GetMessageClass(pool.FindMessageTypeByName(f"openmini.{name}"))
    return classes


_CLASSES = _build()
globals().update(_CLASSES)


def message(name: str):
    return _CLASSES[name]
