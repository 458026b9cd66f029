"""GGUF checkpoint support: tensor type table, reader (C++ index + numpy
memory map), writer, and block (de)quantisers for F32 / F16 / BF16 / Q4_0 /
Q8_0 plus the per-channel INT8 layout (an I8 tensor with a companion
``<name>.scale`` F16 tensor)."""
from .constants import GGMLType, BLOCK_SIZES  # noqa: F401
