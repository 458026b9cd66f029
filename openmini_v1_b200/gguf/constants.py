"""GGML tensor type ids and block geometry (public GGUF specification).

The reference keeps the same table (openmini-server/src/model/inference/gguf.rs:73-445);
note the reference maps BF16 to id 29 and dequantises it to zeros
(openmini-server/src/model/inference/quant.rs:56-79); here BF16 is id 30 as in
the GGUF specification and is read exactly.
"""
import enum


class GGMLType(enum.IntEnum):
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    IQ4_NL = 20
    IQ4_XS = 23
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    BF16 = 30


# type -> (elements per block, bytes per block)
BLOCK_SIZES = {
    GGMLType.F32: (1, 4), GGMLType.F16: (1, 2), GGMLType.BF16: (1, 2),
    GGMLType.Q4_0: (32, 18), GGMLType.Q4_1: (32, 20), GGMLType.Q5_0: (32, 22), GGMLType.Q5_1: (32, 24),
    GGMLType.Q8_0: (32, 34), GGMLType.Q8_1: (32, 36),
    GGMLType.Q2_K: (256, 84), GGMLType.Q3_K: (256, 110), GGMLType.Q4_K: (256, 144), GGMLType.Q5_K: (256, 176),
    GGMLType.Q6_K: (256, 210), GGMLType.Q8_K: (256, 292),
    GGMLType.IQ4_NL: (32, 18), GGMLType.IQ4_XS: (256, 136),
    GGMLType.I8: (1, 1), GGMLType.I16: (1, 2), GGMLType.I32: (1, 4), GGMLType.I64: (1, 8), GGMLType.F64: (1, 8),
}

# metadata value types
KV_UINT8, KV_INT8, KV_UINT16, KV_INT16, KV_UINT32, KV_INT32, KV_FLOAT32, KV_BOOL, KV_STRING, KV_ARRAY, \
    KV_UINT64, KV_INT64, KV_FLOAT64 = range(13)

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3

